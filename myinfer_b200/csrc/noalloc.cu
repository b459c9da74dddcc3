// Allocation-free variant of the quantized matmul entry point.
//
// Some callers of this library cannot call cudaMalloc at all: hosts whose
// device memory is handed out by a pool they do not own (an inference server
// that reserved all device memory for its own allocator at start-up), or
// embedders that forbid any allocation once they are running.  The regular
// m5_quantized_matmul lazily grows a per-device cudaMalloc'd scratch for the
// split-tile partial sums of its tensor-core GEMV; this entry point uses a
// fixed array compiled into the library instead.
//
// The scratch is a file-scope __device__ array (every GPU that loads the
// library holds it until the process exits).  Its device address is looked
// up once per device with cudaGetSymbolAddress on the first call made on that
// device, so that first call should come before any stream capture.  The
// rows a call uses ([8][N rounded up to 16] partial sums and N/16 counters)
// are cleared on the stream before the GEMV runs.  All calls share the one
// array and it keeps the last call's contents: calls that overlap on the GPU
// (different streams, no ordering between them) race on it and must not be
// issued.
#include <mutex>

#include "gemv.cuh"

namespace m5 {

// Largest output dimension N (weight rows) the array covers.
constexpr int kNoAllocMaxRows = 1 << 18;  // 262144 rows: every Qwen3 projection and the 151936-row vocabulary
// Split-tile slots of the tensor-map GEMV: 2 x 8 tokens x 16 rows per CTA, for
// up to 8 CTAs on each of up to 256 SMs.
constexpr size_t kNoAllocPartFloats = size_t(2) * 8 * 16 * 8 * 256;
constexpr size_t kNoAllocBytes = size_t(8) * kNoAllocMaxRows * sizeof(float) + size_t(kNoAllocMaxRows / 16) * sizeof(int) +
                                 kNoAllocPartFloats * sizeof(float);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

static int noalloc_scratch(char** out) {
  static std::mutex mu;
  static char* addr[64] = {nullptr};
  int dev = 0;
  M5_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(M5_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    addr[dev] = static_cast<char*>(p);
  }
  *out = addr[dev];
  return M5_OK;
}

}  // namespace m5

using namespace m5;

extern "C" int m5_quantized_matmul_noalloc(const void* x, int64_t M, int64_t K, const uint32_t* wq, const void* scales,
                                           const void* biases, int64_t N, int group_size, int bits, void* y,
                                           void* stream) {
  M5_CHECK_ARG(x && wq && scales && biases && y, "m5_quantized_matmul_noalloc: null pointer");
  M5_CHECK_ARG(bits == 4 && group_size == 64, "m5_quantized_matmul_noalloc: only 4-bit group-64 weights");
  M5_CHECK_ARG(K > 0 && K % 64 == 0 && N > 0 && M >= 0, "m5_quantized_matmul_noalloc: K must be a multiple of 64");
  if (N > kNoAllocMaxRows)
    return fail(M5_ERR_INVALID, "m5_quantized_matmul_noalloc: N = " + std::to_string(N) +
                                    " exceeds the built-in scratch limit of " + std::to_string(kNoAllocMaxRows) +
                                    " rows; use m5_quantized_matmul");
  M5_CHECK_ARG(K < (1LL << 31) && M < (1LL << 31), "m5_quantized_matmul_noalloc: size too large");
  if (M == 0) return M5_OK;
  char* base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int rows16 = int((N + 15) / 16 * 16);
  // This call's layout inside the array: partial sums [8][rows16], then one
  // counter per 16-row tile, then the per-CTA split-tile slots.  The partial
  // sums and the counters must be zero; a finished launch leaves them zeroed,
  // but an earlier call that stopped on an error may not have.  The slots are
  // written before they are read.
  float* acc = reinterpret_cast<float*>(base);
  int* cnt = reinterpret_cast<int*>(base + size_t(8) * kNoAllocMaxRows * sizeof(float));
  M5_CUDA(cudaMemsetAsync(acc, 0, size_t(8) * rows16 * sizeof(float), st));
  M5_CUDA(cudaMemsetAsync(cnt, 0, size_t(rows16 / 16) * sizeof(int), st));
  GemvArgs a{};
  a.x = (const bf16*)x;
  a.ldx = K;
  a.K = (int)K;
  a.nseg = 1;
  a.seg[0].w = wq;
  a.seg[0].s = (const bf16*)scales;
  a.seg[0].b = (const bf16*)biases;
  a.seg[0].rows = (int)N;
  a.seg[0].y = (bf16*)y;
  a.ldy = N;
  a.total_rows = (int)N;
  a.mma_acc = acc;
  a.mma_cnt = cnt;
  a.mma_rows = rows16;
  a.mma_part = reinterpret_cast<float*>(base + size_t(8) * kNoAllocMaxRows * sizeof(float) +
                                        size_t(kNoAllocMaxRows / 16) * sizeof(int));
  a.mma_part_floats = kNoAllocPartFloats;
  const int cap = gemv_max_tokens((int)K);
  for (int64_t t0 = 0; t0 < M;) {
    int mt = (int)std::min<int64_t>(8, M - t0);
    if (!gemv_mma_eligible(a, mt, EPI_STORE) && !gemv_tmap_eligible(a, mt, EPI_STORE)) {
      mt = 1;
      while (mt * 2 <= std::min<int64_t>(cap, M - t0)) mt *= 2;
    }
    GemvArgs c = a;
    c.x = a.x + t0 * K;
    c.seg[0].y = a.seg[0].y + t0 * N;
    rc = gemv_launch(c, mt, EPI_STORE, st);
    if (rc) return rc;
    t0 += mt;
  }
  return M5_OK;
}
