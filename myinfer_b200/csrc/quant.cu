// MLX affine group quantization on the device (mx.quantize / mx.dequantize).
//
// The quantizer is the one the reference runs for its KV cache
// (m5engine/attention.py:111-112 -> QuantizedKVCache) and that produced every
// MLX 4-bit weight.  It must be bit-exact with the CPU restatement, so every
// step below is an IEEE-rounded fp32 operation in the same order: no fused
// multiply-adds, IEEE division (__fdiv_rn), round-half-to-even (rintf).
#include <mutex>

#include "common.cuh"
#include "quant_impl.cuh"

namespace m5 {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return M5_ERR_CUDA;
}

// Off unless M5_PDL=1: measured on B200, letting the next GEMV's CTAs start
// early made the decode step slower (they compete for HBM and SM slots with
// the tail of the previous kernel and gain nothing while their activations
// are not ready).
bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("M5_PDL");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// One warp per group of 64 elements (2 per lane), one group per warp-iteration.
template <int BITS, typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                       int64_t ld_x, uint32_t* __restrict__ wq,
                                                       bf16* __restrict__ scales, bf16* __restrict__ biases) {
  const int lane = threadIdx.x & 31;
  const int64_t groups_per_row = cols / 64;
  const int64_t total = rows * groups_per_row;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t g = warp; g < total; g += nwarps) {
    const int64_t r = g / groups_per_row, c = g - r * groups_per_row;
    const T* src = x + r * ld_x + c * 64 + 2 * lane;
    float v0, v1;
    if constexpr (sizeof(T) == 2) {
      uint32_t u = *reinterpret_cast<const uint32_t*>(src);
      v0 = bf16_lo(u);
      v1 = bf16_hi(u);
    } else {
      float2 f = *reinterpret_cast<const float2*>(src);
      v0 = f.x;
      v1 = f.y;
    }
    QParams p = group_params<BITS>(warp_max(fmaxf(v0, v1)), warp_min(fminf(v0, v1)));
    uint32_t q0 = quant_code<BITS>(v0, p), q1 = quant_code<BITS>(v1, p);
    uint32_t word;
    bool writer;
    int widx;
    pack_pair<BITS>(q0, q1, lane, word, writer, widx);
    uint32_t* dst = wq + r * (cols * BITS / 32) + c * (64 * BITS / 32);
    if (writer) dst[widx] = word;
    if (lane == 0) {
      scales[r * groups_per_row + c] = f2bf(p.scale);
      biases[r * groups_per_row + c] = f2bf(p.bias);
    }
  }
}

template <int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ wq, const bf16* __restrict__ scales,
                                                         const bf16* __restrict__ biases, int64_t rows, int64_t cols,
                                                         int group_size, bf16* __restrict__ out) {
  constexpr int PER = 32 / BITS;
  const int64_t words = rows * cols / PER;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < words; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / (cols / PER), cw = i - r * (cols / PER);
    const uint32_t w = wq[i];
    const int64_t col0 = cw * PER;
    const int64_t gi = r * (cols / group_size) + col0 / group_size;
    const float s = bf2f(scales[gi]), b = bf2f(biases[gi]);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const float q = float((w >> (j * BITS)) & ((1u << BITS) - 1));
      out[r * cols + col0 + j] = f2bf(fmaf(q, s, b));
    }
  }
}

}  // namespace m5

using namespace m5;

extern "C" int m5_version(void) { return 100; }

extern "C" size_t m5_last_error(char* buf, size_t n) {
  const std::string& s = g_last_error;
  if (buf && n) {
    size_t k = s.size() < n - 1 ? s.size() : n - 1;
    memcpy(buf, s.data(), k);
    buf[k] = 0;
  }
  return s.size();
}

extern "C" int m5_affine_quantize(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ld_x,
                                  int group_size, int bits, uint32_t* wq, void* scales, void* biases,
                                  void* stream) {
  M5_CHECK_ARG(x && wq && scales && biases, "m5_affine_quantize: null pointer");
  M5_CHECK_ARG(bits == 4 || bits == 8, "m5_affine_quantize: bits must be 4 or 8");
  M5_CHECK_ARG(group_size == 64, "m5_affine_quantize: group_size must be 64");
  M5_CHECK_ARG(rows >= 0 && cols >= 0 && cols % 64 == 0, "m5_affine_quantize: cols must be a multiple of 64");
  M5_CHECK_ARG(ld_x >= cols, "m5_affine_quantize: ld_x < cols");
  M5_CHECK_ARG(x_dtype == M5_DTYPE_BF16 || x_dtype == M5_DTYPE_F32, "m5_affine_quantize: x_dtype");
  if (rows == 0 || cols == 0) return M5_OK;
  M5_CHECK_ARG((x_dtype == M5_DTYPE_BF16 ? (ld_x % 2 == 0) : true), "m5_affine_quantize: ld_x must be even");
  const int64_t groups = rows * (cols / 64);
  const int threads = 256;
  int blocks = (int)std::min<int64_t>((groups + 7) / 8, int64_t(sm_count()) * 16);
  cudaStream_t s = (cudaStream_t)stream;
  bf16* sc = (bf16*)scales;
  bf16* bi = (bf16*)biases;
  if (x_dtype == M5_DTYPE_BF16) {
    if (bits == 8) quantize_kernel<8, bf16><<<blocks, threads, 0, s>>>((const bf16*)x, rows, cols, ld_x, wq, sc, bi);
    else quantize_kernel<4, bf16><<<blocks, threads, 0, s>>>((const bf16*)x, rows, cols, ld_x, wq, sc, bi);
  } else {
    if (bits == 8) quantize_kernel<8, float><<<blocks, threads, 0, s>>>((const float*)x, rows, cols, ld_x, wq, sc, bi);
    else quantize_kernel<4, float><<<blocks, threads, 0, s>>>((const float*)x, rows, cols, ld_x, wq, sc, bi);
  }
  M5_LAUNCH_CHECK("m5_affine_quantize launch");
  return M5_OK;
}

extern "C" int m5_affine_dequantize(const uint32_t* wq, const void* scales, const void* biases, int64_t rows,
                                    int64_t cols, int group_size, int bits, void* out, void* stream) {
  M5_CHECK_ARG(wq && scales && biases && out, "m5_affine_dequantize: null pointer");
  M5_CHECK_ARG(bits == 4 || bits == 8, "m5_affine_dequantize: bits must be 4 or 8");
  M5_CHECK_ARG(group_size == 32 || group_size == 64 || group_size == 128, "m5_affine_dequantize: group_size");
  M5_CHECK_ARG(rows >= 0 && cols % group_size == 0, "m5_affine_dequantize: cols % group_size");
  if (rows == 0 || cols == 0) return M5_OK;
  const int64_t words = rows * cols * bits / 32;
  int blocks = (int)std::min<int64_t>((words + 255) / 256, int64_t(sm_count()) * 32);
  cudaStream_t s = (cudaStream_t)stream;
  if (bits == 8)
    dequantize_kernel<8><<<blocks, 256, 0, s>>>(wq, (const bf16*)scales, (const bf16*)biases, rows, cols, group_size, (bf16*)out);
  else
    dequantize_kernel<4><<<blocks, 256, 0, s>>>(wq, (const bf16*)scales, (const bf16*)biases, rows, cols, group_size, (bf16*)out);
  M5_LAUNCH_CHECK("m5_affine_dequantize launch");
  return M5_OK;
}
