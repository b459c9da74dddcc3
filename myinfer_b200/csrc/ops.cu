// Small fused kernels of the token loop: RMSNorm, QK-norm + RoPE/YaRN + KV
// quantize-on-append, quantized embedding gather, greedy argmax, MoE top-k.
#include <algorithm>
#include <cmath>

#include "ops.cuh"
#include "quant_impl.cuh"
#include "rope_impl.cuh"

namespace m5 {

// ------------------------------------------------------- rope + kv append
template <int BITS>
__global__ void __launch_bounds__(256) rope_append_kernel(const RopeAppendArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int H3 = a.Hq + 2 * a.Hkv;
  if (gw >= a.L * H3) return;
  const int t = gw / H3, h = gw - t * H3;
  rope_append_row<BITS, false>(a, t, h, lane);
}

int rope_append_launch(const RopeAppendArgs& a, cudaStream_t stream) {
  const int warps = a.L * (a.Hq + 2 * a.Hkv);
  const int blocks = ceil_div(warps, 8);
  switch (a.kv.bits) {
    case 0: M5_CUDA(launch_pdl(rope_append_kernel<0>, dim3(blocks), dim3(256), 0, stream, a)); break;
    case 4: M5_CUDA(launch_pdl(rope_append_kernel<4>, dim3(blocks), dim3(256), 0, stream, a)); break;
    case 8: M5_CUDA(launch_pdl(rope_append_kernel<8>, dim3(blocks), dim3(256), 0, stream, a)); break;
    default: return fail(M5_ERR_INVALID, "kv bits must be 0, 4 or 8");
  }
  M5_LAUNCH_CHECK("rope_append launch");
  return M5_OK;
}

// ------------------------------------------------- bf16 cache -> packed cache
template <int BITS>
__global__ void __launch_bounds__(256) kv_convert_kernel(const m5_layer_kv src, const m5_layer_kv dst, int Hkv,
                                                         int len) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int total = 2 * Hkv * len;
  if (gw >= total) return;
  const int which = gw / (Hkv * len);  // 0 = keys, 1 = values
  const int rem = gw - which * Hkv * len;
  const int hk = rem / len, p = rem - hk * len;
  const bf16* s = reinterpret_cast<const bf16*>(which ? src.v : src.k) + (size_t(hk) * src.capacity + p) * 128;
  const uint2 raw = reinterpret_cast<const uint2*>(s)[lane];
  const float x[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  const size_t row = size_t(hk) * dst.capacity + p;
  if (which == 0) store_kv_row<BITS>(x, lane, dst.k, (bf16*)dst.k_scales, (bf16*)dst.k_biases, row);
  else store_kv_row<BITS>(x, lane, dst.v, (bf16*)dst.v_scales, (bf16*)dst.v_biases, row);
}

int kv_quantize_layer_launch(const m5_layer_kv& src, const m5_layer_kv& dst, int Hkv, int D, int len,
                             cudaStream_t stream) {
  if (D != 128) return fail(M5_ERR_UNSUPPORTED, "kv conversion supports head_dim 128");
  if (src.bits != 0) return fail(M5_ERR_INVALID, "kv conversion source must be a bf16 cache");
  if (len <= 0) return M5_OK;
  if (len > src.capacity || len > dst.capacity) return fail(M5_ERR_INVALID, "kv conversion: len exceeds capacity");
  const int blocks = ceil_div(2LL * Hkv * len, 8);
  if (dst.bits == 8) kv_convert_kernel<8><<<blocks, 256, 0, stream>>>(src, dst, Hkv, len);
  else if (dst.bits == 4) kv_convert_kernel<4><<<blocks, 256, 0, stream>>>(src, dst, Hkv, len);
  else return fail(M5_ERR_INVALID, "kv conversion target bits must be 4 or 8");
  M5_LAUNCH_CHECK("kv convert launch");
  return M5_OK;
}

// -------------------------------------------------------------- embedding
__global__ void __launch_bounds__(256) embed_kernel(const int32_t* __restrict__ tokens, int T, const uint32_t* __restrict__ w,
                                                    const bf16* __restrict__ s, const bf16* __restrict__ b, int H, int V,
                                                    bf16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int H8 = H / 8;
  const int64_t total = int64_t(T) * H8;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H8), j = int(i - int64_t(t) * H8);
    const int64_t tok = tokens[t];
    if (tok < 0 || tok >= V) {  // out-of-vocabulary id: zero row, never an out-of-bounds read
      reinterpret_cast<uint4*>(out + size_t(t) * H)[j] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint32_t wd = w[tok * H8 + j];
    const float sc = bf2f(s[tok * (H / 64) + j / 8]), bi = bf2f(b[tok * (H / 64) + j / 8]);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float v0 = fmaf(float((wd >> (8 * k)) & 15u), sc, bi);
      const float v1 = fmaf(float((wd >> (8 * k + 4)) & 15u), sc, bi);
      o[k] = uint32_t(__bfloat16_as_ushort(f2bf(v0))) | (uint32_t(__bfloat16_as_ushort(f2bf(v1))) << 16);
    }
    reinterpret_cast<uint4*>(out + size_t(t) * H)[j] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int embed_launch(const int32_t* tokens, int T, const uint32_t* w, const bf16* s, const bf16* b, int H, int V,
                 bf16* out, cudaStream_t stream) {
  if (H % 64) return fail(M5_ERR_INVALID, "embedding: hidden size must be a multiple of 64");
  const int64_t total = int64_t(T) * (H / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, sm_count() * 8);
  M5_CUDA(launch_pdl(embed_kernel, dim3(blocks), dim3(256), 0, stream, tokens, T, w, s, b, H, V, out));
  M5_LAUNCH_CHECK("embedding launch");
  return M5_OK;
}

// ------------------------------------------------------------------ argmax
constexpr int ARGMAX_BLOCKS = 256;
struct ArgmaxScratch {
  unsigned int counter;
  unsigned int pad[3];
  float val[ARGMAX_BLOCKS];
  int idx[ARGMAX_BLOCKS];
};
size_t argmax_scratch_bytes() { return sizeof(ArgmaxScratch); }

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void block_best(float& v, int& i) {
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) { v = ov; i = oi; }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) { sv[w] = v; si[w] = i; }
  __syncthreads();
  if (w == 0) {
    v = lane < (blockDim.x >> 5) ? sv[lane] : -INFINITY;
    i = lane < (blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
  }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const bf16* __restrict__ x, int64_t n, int32_t* out,
                                                      ArgmaxScratch* sc) {
  pdl_wait();
  pdl_launch_dependents();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float v = bf2f(x[i]);
    if (better(v, int(i), bv, bi)) { bv = v; bi = int(i); }
  }
  block_best(bv, bi);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    sc->val[blockIdx.x] = bv;
    sc->idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned int done = atomicAdd(&sc->counter, 1u);
    last = (done == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int j = threadIdx.x; j < gridDim.x; j += blockDim.x) {
    const float v = ((volatile float*)sc->val)[j];
    const int i = ((volatile int*)sc->idx)[j];
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  __syncthreads();
  block_best(bv, bi);
  if (threadIdx.x == 0) {
    *out = bi;
    sc->counter = 0;  // ready for the next launch (also inside graph replays)
  }
}

__global__ void __launch_bounds__(1024) argmax_rows_kernel(const bf16* __restrict__ x, int64_t n, int32_t* out) {
  pdl_wait();
  pdl_launch_dependents();
  const bf16* xr = x + size_t(blockIdx.x) * n;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf2f(xr[i]);
    if (better(v, int(i), bv, bi)) { bv = v; bi = int(i); }
  }
  block_best(bv, bi);
  if (threadIdx.x == 0) out[blockIdx.x] = bi;
}

int argmax_rows_launch(const bf16* x, int rows, int64_t n, int32_t* out, cudaStream_t stream) {
  if (n <= 0 || rows <= 0) return fail(M5_ERR_INVALID, "argmax: empty input");
  M5_CUDA(launch_pdl(argmax_rows_kernel, dim3(rows), dim3(1024), 0, stream, x, n, out));
  M5_LAUNCH_CHECK("argmax rows launch");
  return M5_OK;
}

int argmax_launch(const bf16* x, int64_t n, int32_t* out, void* scratch, cudaStream_t stream) {
  if (n <= 0) return fail(M5_ERR_INVALID, "argmax: empty input");
  const int blocks = (int)std::min<int64_t>(ARGMAX_BLOCKS, (n + 1023) / 1024);
  M5_CUDA(launch_pdl(argmax_kernel, dim3(blocks), dim3(1024), 0, stream, x, n, out, reinterpret_cast<ArgmaxScratch*>(scratch)));
  M5_LAUNCH_CHECK("argmax launch");
  return M5_OK;
}

// ---------------------------------------------------------------- rms norm
__global__ void __launch_bounds__(256) rms_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                       int dim, float eps, bf16* __restrict__ y) {
  pdl_wait();
  pdl_launch_dependents();
  const bf16* xr = x + size_t(blockIdx.x) * dim;
  bf16* yr = y + size_t(blockIdx.x) * dim;
  __shared__ float red[33];
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = bf2f(xr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[32] = v;
  }
  __syncthreads();
  const float inv = __frsqrt_rn(__fadd_rn(red[32] / float(dim), eps));
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    yr[i] = f2bf(__fmul_rn(bf2f(w[i]), rbf(__fmul_rn(bf2f(xr[i]), inv))));
}

// The same with 16-byte loads and stores: each thread holds up to VPT chunks
// of 8 values of its row in registers between the sum of squares and the
// scaling, so the row is read once and every load is issued up front (the
// strided scalar loop above waits on dim / 256 dependent loads per pass).
template <int VPT>
__global__ void __launch_bounds__(256) rms_norm_vec_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                           int dim, float eps, bf16* __restrict__ y) {
  pdl_wait();
  pdl_launch_dependents();
  const int nv = dim >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + size_t(blockIdx.x) * dim);
  uint4* yr = reinterpret_cast<uint4*>(y + size_t(blockIdx.x) * dim);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  __shared__ float red[33];
  uint4 xv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    const int i = threadIdx.x + 256 * q;
    xv[q] = i < nv ? xr[i] : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    const uint32_t u[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = bf16_lo(u[j]), hi = bf16_hi(u[j]);
      ss += lo * lo;
      ss += hi * hi;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[32] = v;
  }
  __syncthreads();
  const float inv = __frsqrt_rn(__fadd_rn(red[32] / float(dim), eps));
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    const int i = threadIdx.x + 256 * q;
    if (i < nv) {
      const uint4 wv = wr[i];
      const uint32_t xu[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a0 = __fmul_rn(bf16_lo(wu[j]), rbf(__fmul_rn(bf16_lo(xu[j]), inv)));
        const float a1 = __fmul_rn(bf16_hi(wu[j]), rbf(__fmul_rn(bf16_hi(xu[j]), inv)));
        o[j] = uint32_t(__bfloat16_as_ushort(f2bf(a0))) | (uint32_t(__bfloat16_as_ushort(f2bf(a1))) << 16);
      }
      yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

int rms_norm_launch(const bf16* x, const bf16* w, int64_t rows, int dim, float eps, bf16* y, cudaStream_t stream) {
  if (rows <= 0) return M5_OK;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int vpt = (dim / 8 + 255) / 256;
  if (dim % 8 == 0 && al(x) && al(w) && al(y) && vpt >= 1 && vpt <= 4) {
    switch (vpt) {
      case 1: M5_CUDA(launch_pdl(rms_norm_vec_kernel<1>, dim3((unsigned)rows), dim3(256), 0, stream, x, w, dim, eps, y)); break;
      case 2: M5_CUDA(launch_pdl(rms_norm_vec_kernel<2>, dim3((unsigned)rows), dim3(256), 0, stream, x, w, dim, eps, y)); break;
      case 3: M5_CUDA(launch_pdl(rms_norm_vec_kernel<3>, dim3((unsigned)rows), dim3(256), 0, stream, x, w, dim, eps, y)); break;
      default: M5_CUDA(launch_pdl(rms_norm_vec_kernel<4>, dim3((unsigned)rows), dim3(256), 0, stream, x, w, dim, eps, y)); break;
    }
  } else {
    M5_CUDA(launch_pdl(rms_norm_kernel, dim3((unsigned)rows), dim3(256), 0, stream, x, w, dim, eps, y));
  }
  M5_LAUNCH_CHECK("rms_norm launch");
  return M5_OK;
}

// ------------------------------------------------------------- MoE top-k
// One warp per token; E <= 256 router logits, lane j holds logits j, j+32, ...
__global__ void __launch_bounds__(256) moe_topk_kernel(const bf16* __restrict__ logits, int T, int E, int k,
                                                       int norm_topk, int32_t* __restrict__ ids,
                                                       bf16* __restrict__ scores) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  constexpr int PER = 8;
  float v[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? bf2f(logits[size_t(t) * E + e]) : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    v[j] = (lane + 32 * j < E) ? expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
  sum = warp_sum(sum);
#pragma unroll
  for (int j = 0; j < PER; ++j) v[j] = (lane + 32 * j < E) ? rbf(__fdiv_rn(v[j], sum)) : -INFINITY;
  float chosen = 0.f;  // running sum of selected probabilities (fp32, selection order)
  float my_score = 0.f;
  int my_id = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && better(v[j], e, bv, bi)) { bv = v[j]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j == bi) v[j] = -INFINITY;
    chosen += bv;
    if (lane == r) { my_score = bv; my_id = bi; }
  }
  if (lane < k) {
    float s = my_score;
    if (norm_topk) s = rbf(__fdiv_rn(s, rbf(chosen)));
    ids[size_t(t) * k + lane] = my_id;
    scores[size_t(t) * k + lane] = f2bf(s);
  }
}

int moe_topk_launch(const bf16* logits, int T, int E, int k, int norm_topk, int32_t* ids, bf16* scores,
                    cudaStream_t stream) {
  if (E > 256 || k > 32 || k > E || k <= 0) return fail(M5_ERR_INVALID, "moe top-k: E <= 256, 0 < k <= min(32, E)");
  if (T <= 0) return M5_OK;
  M5_CUDA(launch_pdl(moe_topk_kernel, dim3(ceil_div(T, 8)), dim3(256), 0, stream, logits, T, E, k, norm_topk, ids, scores));
  M5_LAUNCH_CHECK("moe top-k launch");
  return M5_OK;
}

// ------------------------------------------------------------ residual add
__global__ void residual_add_f32_kernel(bf16* h, const float* r, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    h[i] = f2bf(bf2f(h[i]) + rbf(r[i]));
}

int residual_add_f32_launch(bf16* h, const float* r, int64_t n, cudaStream_t stream) {
  if (n <= 0) return M5_OK;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, sm_count() * 4);
  M5_CUDA(launch_pdl(residual_add_f32_kernel, dim3(blocks), dim3(256), 0, stream, h, r, n));
  M5_LAUNCH_CHECK("residual add launch");
  return M5_OK;
}

}  // namespace m5
