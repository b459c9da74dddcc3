// Routed experts of a Qwen3-MoE layer as two grouped streaming GEMVs.
//
// The router (GEMV + moe_topk) leaves ids/scores [T, k] on the device, so no
// host sync happens inside the layer (the reference's streaming wrapper syncs
// at m5engine/expert_stream.py:384-389).  Then:
//   gate/up - grid.y = (token, slot); a CTA stages RMSNorm(x_t) once and its
//             warps stream rows of expert ids[t, slot]'s gate and up matrices,
//             writing bf16(bf16(g*bf16(sigmoid g)) * u) (mlx-lm SwiGLU);
//   down    - grid.y = token; a CTA stages the k SwiGLU rows of its token and
//             every warp computes one output row for all k experts, then
//             h += bf16(sum_j bf16(bf16(y_j) * score_j)) (the score-weighted
//             sum of mlx-lm Qwen3MoeSparseMoeBlock) in its epilogue.
// Experts outside [e_first, e_first + e_local) are skipped, which is what an
// expert-parallel rank needs; it then writes fp32 partial sums for a reduce.
#include <algorithm>

#include "gemv_impl.cuh"
#include "moe.cuh"

namespace m5 {

constexpr int MOE_WARPS = 4;

__global__ void __launch_bounds__(MOE_WARPS * 32) moe_gate_up_kernel(const MoeArgs a, int rpw) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float smem[];
  const int slot = blockIdx.y;
  const int t = slot / a.k;
  const int e = a.ids[slot] - a.e_first;
  if (e < 0 || e >= a.e_local) return;
  const int H = a.H, I = a.I;
  float* xs = smem;
  float* xsum = xs + H;
  float* red = xsum + (H >> 5);
  stage_rows<1>(a.x + size_t(t) * H, H, H, a.norm_w, a.eps, xs, xsum, red);
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5);
  const size_t H8 = H >> 3, H64 = H >> 6;
  for (int rr = 0; rr < rpw; ++rr) {
    const int row = gw * rpw + rr;
    if (row >= I) break;
    const size_t er = size_t(e) * I + row;
    float g[1] = {0.f}, u[1] = {0.f};
    row_dot<1, 4>(a.gate.w + er * H8, a.gate.s + er * H64, a.gate.b + er * H64, H, xs, xsum, g);
    row_dot<1, 4>(a.up.w + er * H8, a.up.s + er * H64, a.up.b + er * H64, H, xs, xsum, u);
    const float gv = rbf(warp_sum(g[0])), uv = rbf(warp_sum(u[0]));
    if (lane == 0) {
      const float sg = rbf(1.f / (1.f + expf(-gv)));
      a.act[size_t(slot) * I + row] = f2bf(rbf(gv * sg) * uv);
    }
  }
}

__global__ void __launch_bounds__(MOE_WARPS * 32) moe_down_kernel(const MoeArgs a, int rpw) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float smem[];
  const int t = blockIdx.y;
  const int H = a.H, I = a.I, k = a.k;
  float* xs = smem;
  float* xsum = xs + size_t(k) * I;
  float* red = xsum + size_t(k) * (I >> 5);
  for (int j = 0; j < k; ++j) {
    const int e = a.ids[t * k + j] - a.e_first;
    if (e < 0 || e >= a.e_local) continue;  // uniform across the CTA
    stage_rows<1>(a.act + size_t(t * k + j) * I, I, I, nullptr, 0.f, xs + size_t(j) * I, xsum + size_t(j) * (I >> 5),
                  red);
  }
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5);
  const size_t I8 = I >> 3, I64 = I >> 6;
  for (int rr = 0; rr < rpw; ++rr) {
    const int n = gw * rpw + rr;
    if (n >= H) break;
    float sum = 0.f;
    for (int j = 0; j < k; ++j) {
      const int e = a.ids[t * k + j] - a.e_first;
      if (e < 0 || e >= a.e_local) continue;
      const size_t er = size_t(e) * H + n;
      float acc[1] = {0.f};
      row_dot<1, 4>(a.down.w + er * I8, a.down.s + er * I64, a.down.b + er * I64, I, xs + size_t(j) * I,
                    xsum + size_t(j) * (I >> 5), acc);
      const float y = rbf(warp_sum(acc[0]));
      sum += rbf(y * bf2f(a.scores[t * k + j]));
    }
    if (lane == 0) {
      if (a.partial) {
        a.partial[size_t(t) * H + n] = sum;
      } else {
        bf16* p = a.h + size_t(t) * H + n;
        *p = f2bf(bf2f(*p) + rbf(sum));
      }
    }
  }
}

int moe_launch(const MoeArgs& a, cudaStream_t st) {
  if (a.H % 64 || a.I % 64) return fail(M5_ERR_INVALID, "moe: hidden and expert sizes must be multiples of 64");
  if (a.T <= 0) return M5_OK;
  static DeviceOnce once;  // the attributes belong to each device's context
  M5_CUDA(once.run([&] {
    cudaError_t e = cudaFuncSetAttribute(moe_gate_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(moe_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  }));
  const int resident = sm_count() * 48;
  {
    const size_t smem = size_t(a.H) * 4 + size_t(a.H / 32) * 4 + 33 * 4;
    const long long slots = (long long)a.T * a.k;
    const int rpw = std::max(1, (int)((a.I * slots + resident - 1) / resident));
    dim3 grid(ceil_div(a.I, MOE_WARPS * rpw), (unsigned)slots);
    M5_CUDA(launch_pdl(moe_gate_up_kernel, dim3(grid), dim3(MOE_WARPS * 32), smem, st, a, rpw));
    M5_LAUNCH_CHECK("moe gate/up launch");
  }
  {
    const size_t smem = size_t(a.k) * a.I * 4 + size_t(a.k) * (a.I / 32) * 4 + 33 * 4;
    if (smem > 200 * 1024) return fail(M5_ERR_UNSUPPORTED, "moe: k * moe_intermediate_size too large");
    const int rpw = std::max(1, (int)(((long long)a.H * a.T + resident - 1) / resident));
    dim3 grid(ceil_div(a.H, MOE_WARPS * rpw), (unsigned)a.T);
    M5_CUDA(launch_pdl(moe_down_kernel, dim3(grid), dim3(MOE_WARPS * 32), smem, st, a, rpw));
    M5_LAUNCH_CHECK("moe down launch");
  }
  return M5_OK;
}

// ------------------------------------------------ prefill: grouped by expert
// (token, slot) pairs sorted by local expert with a single-CTA counting sort:
// counts, exclusive offsets, and each pair's row in the expert-ordered
// buffers (rows of one expert in any order: a GEMM row does not depend on the
// others).  Pairs of experts on other ranks get -1.
__global__ void __launch_bounds__(1024) moe_sort_kernel(const int32_t* __restrict__ ids, int pairs, int e_first,
                                                        int e_local, int32_t* __restrict__ counts,
                                                        int32_t* __restrict__ offsets, int32_t* __restrict__ pos) {
  extern __shared__ int sh[];  // [e_local] counts, [e_local] fill cursors
  int* cnt = sh;
  int* cur = sh + e_local;
  for (int e = threadIdx.x; e < e_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e_first;
    if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < e_local; ++e) {
      cur[e] = run;
      offsets[e] = run;
      counts[e] = cnt[e];
      run += cnt[e];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e_first;
    pos[i] = (e >= 0 && e < e_local) ? atomicAdd(&cur[e], 1) : -1;
  }
}

// rows_out[pos[t * k + j]] = x[t] (16-byte copies), for pairs with a row
__global__ void __launch_bounds__(256) moe_gather_kernel(const bf16* __restrict__ x, int H, int pairs, int k,
                                                         const int32_t* __restrict__ pos, bf16* __restrict__ out) {
  const int H8 = H >> 3;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < int64_t(pairs) * H8;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int pr = int(i / H8), c = int(i % H8);
    const int r = pos[pr];
    if (r < 0) continue;
    reinterpret_cast<uint4*>(out + size_t(r) * H)[c] = reinterpret_cast<const uint4*>(x + size_t(pr / k) * H)[c];
  }
}

// h[t] += bf16(sum_j bf16(y[pos[t, j]] * score[t, j])) in slot order (mlx-lm
// Qwen3MoeSparseMoeBlock), or partial[t] = the fp32 sum (expert parallel).
__global__ void __launch_bounds__(256) moe_combine_kernel(const bf16* __restrict__ y, int T, int H, int k,
                                                          const int32_t* __restrict__ pos,
                                                          const bf16* __restrict__ scores, bf16* __restrict__ h,
                                                          float* __restrict__ partial) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < int64_t(T) * H;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H), n = int(i % H);
    float sum = 0.f;
    for (int j = 0; j < k; ++j) {
      const int r = pos[t * k + j];
      if (r < 0) continue;
      sum += rbf(bf2f(y[size_t(r) * H + n]) * bf2f(scores[t * k + j]));
    }
    if (partial) partial[i] = sum;
    else h[i] = f2bf(bf2f(h[i]) + rbf(sum));
  }
}

int moe_sort_launch(const int32_t* ids, int pairs, int e_first, int e_local, int32_t* counts, int32_t* offsets,
                    int32_t* pos, cudaStream_t st) {
  moe_sort_kernel<<<1, 1024, size_t(2) * e_local * sizeof(int), st>>>(ids, pairs, e_first, e_local, counts, offsets,
                                                                      pos);
  M5_LAUNCH_CHECK("moe sort launch");
  return M5_OK;
}

int moe_gather_launch(const bf16* x, int H, int pairs, int k, const int32_t* pos, bf16* out, cudaStream_t st) {
  const int64_t n = int64_t(pairs) * (H / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, sm_count() * 8);
  moe_gather_kernel<<<blocks, 256, 0, st>>>(x, H, pairs, k, pos, out);
  M5_LAUNCH_CHECK("moe gather launch");
  return M5_OK;
}

int moe_combine_launch(const bf16* y, int T, int H, int k, const int32_t* pos, const bf16* scores, bf16* h,
                       float* partial, cudaStream_t st) {
  const int64_t n = int64_t(T) * H;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, sm_count() * 8);
  moe_combine_kernel<<<blocks, 256, 0, st>>>(y, T, H, k, pos, scores, h, partial);
  M5_LAUNCH_CHECK("moe combine launch");
  return M5_OK;
}

}  // namespace m5
