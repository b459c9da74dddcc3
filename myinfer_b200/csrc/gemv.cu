// Streaming w4g64 dequant-GEMV (kernel K1 of the decode step).
//
// Decode reads every packed weight once per token, so the kernel is HBM-bound
// and its job is to keep ~44 KB of loads in flight per SM while spending as
// few issue slots per weight as possible:
//   * one warp owns whole rows; a lane loads 16 B (32 codes) per step with
//     ld.global.nc.L1::no_allocate, several steps in flight;
//   * the activation vector is staged once per CTA in shared memory as fp32
//     (with the RMSNorm of the previous residual fused into that staging),
//     swizzled so the 32 lanes' 16-byte reads hit distinct banks;
//   * codes become fp32 without I2F: one PRMT puts a code under the exponent
//     of 128.0f (value 128 + q) and the 128 offset is folded out per half
//     group with the precomputed activation sum:  s*sum(x*q) + b*sum(x)
//     = s*sum(x*(128+q)) + (b - 128*s)*sum(x);
//   * products accumulate in fp32 pairs with the sm_100 fma.rn.f32x2.
#include <algorithm>

#include "gemv.cuh"
#include "gemv_impl.cuh"

namespace m5 {

__device__ __forceinline__ void locate(const GemvArgs& a, int row, int& si, int& r) {
  r = row;
  si = 0;
  while (si < a.nseg - 1 && r >= a.seg[si].rows) {
    r -= a.seg[si].rows;
    ++si;
  }
}

template <int MT, int EPI>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int K = a.K;
  float* xs = smem;
  float* xsum = xs + MT * K;
  float* red = xsum + MT * (K >> 5);
  stage_rows<MT>(a.x, a.ldx, K, a.norm_w, a.eps, xs, xsum, red);

  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int K8 = K >> 3, K64 = K >> 6;
  for (int rr = 0; rr < a.rows_per_warp; ++rr) {
    const int row = gw * a.rows_per_warp + rr;
    if (row >= a.total_rows) break;
    if constexpr (EPI == EPI_SWIGLU) {
      const GemvSeg& g = a.seg[0];
      const GemvSeg& up = a.seg[1];
      float ag[MT], au[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) ag[t] = au[t] = 0.f;
      row_dot<MT, 4>(g.w + size_t(row) * K8, g.s + size_t(row) * K64, g.b + size_t(row) * K64, K, xs, xsum, ag);
      row_dot<MT, 4>(up.w + size_t(row) * K8, up.s + size_t(row) * K64, up.b + size_t(row) * K64, K, xs, xsum, au);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float gv = rbf(warp_sum(ag[t]));
        const float uv = rbf(warp_sum(au[t]));
        if (lane == t) {
          const float sg = rbf(1.f / (1.f + expf(-gv)));
          g.y[t * a.ldy + row] = f2bf(rbf(gv * sg) * uv);
        }
      }
    } else {
      int si, r;
      locate(a, row, si, r);
      const GemvSeg& sg = a.seg[si];
      float acc[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[t] = 0.f;
      row_dot<MT, 8>(sg.w + size_t(r) * K8, sg.s + size_t(r) * K64, sg.b + size_t(r) * K64, K, xs, xsum, acc);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == t) {
          if constexpr (EPI == EPI_STORE) {
            sg.y[t * a.ldy + r] = f2bf(v);
          } else if constexpr (EPI == EPI_RESIDUAL) {
            bf16* p = sg.y + t * a.ldy + r;
            *p = f2bf(bf2f(*p) + rbf(v));
          } else {
            sg.yf[t * a.ldy + r] = v;
          }
        }
      }
    }
  }
}

static size_t gemv_smem(int MT, int K) { return size_t(MT) * K * 4 + size_t(MT) * (K / 32) * 4 + 33 * 4; }

int gemv_max_tokens(int K) {
  for (int mt = 8; mt >= 1; mt >>= 1)
    if (gemv_smem(mt, K) <= 200 * 1024) return mt;
  return 0;
}

template <int MT, int EPI>
static int launch_t(const GemvArgs& a, cudaStream_t stream) {
  const size_t smem = gemv_smem(MT, a.K);
  static bool configured = false;  // per template instance; attribute is per device function
  if (!configured) {
    M5_CUDA(cudaFuncSetAttribute(gemv_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024));
    configured = true;
  }
  const int warps_total = ceil_div(a.total_rows, a.rows_per_warp);
  const int blocks = ceil_div(warps_total, GEMV_WARPS);
  gemv_kernel<MT, EPI><<<blocks, GEMV_WARPS * 32, smem, stream>>>(a);
  M5_LAUNCH_CHECK("gemv launch");
  return M5_OK;
}

template <int MT>
static int launch_epi(const GemvArgs& a, int epi, cudaStream_t stream) {
  switch (epi) {
    case EPI_STORE: return launch_t<MT, EPI_STORE>(a, stream);
    case EPI_RESIDUAL: return launch_t<MT, EPI_RESIDUAL>(a, stream);
    case EPI_SWIGLU: return launch_t<MT, EPI_SWIGLU>(a, stream);
    case EPI_F32: return launch_t<MT, EPI_F32>(a, stream);
  }
  return fail(M5_ERR_INVALID, "gemv: bad epilogue");
}

int gemv_launch(const GemvArgs& a_in, int MT, int epi, cudaStream_t stream) {
  GemvArgs a = a_in;
  if (a.K % 64 != 0 || a.K <= 0) return fail(M5_ERR_INVALID, "gemv: K must be a positive multiple of 64");
  if (gemv_smem(MT, a.K) > 200 * 1024) return fail(M5_ERR_INVALID, "gemv: too many tokens for this K");
  if (a.total_rows <= 0) return M5_OK;
  // Rows per warp: enough warps to fill every SM (about 32 resident warps per
  // SM at this CTA size) in a single wave, whole rows per warp.
  const int resident = sm_count() * 32;
  a.rows_per_warp = std::max(1, ceil_div(a.total_rows, resident));
  switch (MT) {
    case 1: return launch_epi<1>(a, epi, stream);
    case 2: return launch_epi<2>(a, epi, stream);
    case 4: return launch_epi<4>(a, epi, stream);
    case 8: return launch_epi<8>(a, epi, stream);
  }
  return fail(M5_ERR_INVALID, "gemv: MT must be 1, 2, 4 or 8");
}

}  // namespace m5
