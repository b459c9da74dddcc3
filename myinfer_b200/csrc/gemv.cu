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
#include <mutex>

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

constexpr int GW = 8;   // warps per CTA
// Weight rows a warp streams in lockstep (they share the activation loads);
// fewer when several tokens' accumulators compete for registers.
template <int MT, int EPI>
struct Rows {
  static constexpr int value = MT == 1 ? 4 : (MT == 2 || EPI == EPI_SWIGLU ? 2 : 1);
};

// Virtual row v of the launch -> (segment, row).  SWIGLU interleaves gate and
// up rows: v = 2 * row + {0 gate, 1 up}.
template <int EPI>
__device__ __forceinline__ void vrow_locate(const GemvArgs& a, int v, int& si, int& r) {
  if constexpr (EPI == EPI_SWIGLU) {
    si = v & 1;
    r = v >> 1;
  } else {
    locate(a, v, si, r);
  }
}

template <int GR>
struct Slot {
  uint4 w[GR];
  uint32_t sb[GR];  // bf16 scale (low half) and bias (high half)
};

// One item = one 16-byte column block (32 codes per lane) of GR rows.
template <int GR>
__device__ __forceinline__ void issue(const uint4* const (&wrow)[GR], const bf16* const (&srow)[GR],
                                      const bf16* const (&brow)[GR], int i, int K32, Slot<GR>& sl) {
  if (i < K32) {
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      if (wrow[r]) {
        sl.w[r] = ldg_stream(wrow[r] + i);
        sl.sb[r] = uint32_t(__bfloat16_as_ushort(srow[r][i >> 1])) |
                   (uint32_t(__bfloat16_as_ushort(brow[r][i >> 1])) << 16);
      }
    }
  }
}

template <int MT, int GR>
__device__ __forceinline__ void consume(const Slot<GR>& sl, const float* xs, const float* xsum, int K, int K32, int i,
                                        float (&acc)[GR][MT]) {
  if (i >= K32) return;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const float4* xb = reinterpret_cast<const float4*>(xs + t * K + (i << 5));
    const int sw = i & 7;
    float4 xv[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) xv[p] = xb[p ^ sw];
    const float xsm = xsum[t * K32 + i];
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      const uint32_t words[4] = {sl.w[r].x, sl.w[r].y, sl.w[r].z, sl.w[r].w};
      float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t lo = words[k] & 0x0f0f0f0fu;
        const uint32_t hi = (words[k] >> 4) & 0x0f0f0f0fu;
        const float4 xa = xv[2 * k], xc = xv[2 * k + 1];
        a0 = ffma2(make_float2(xa.x, xa.y), make_float2(nib128<0>(lo), nib128<0>(hi)), a0);
        a1 = ffma2(make_float2(xa.z, xa.w), make_float2(nib128<1>(lo), nib128<1>(hi)), a1);
        a0 = ffma2(make_float2(xc.x, xc.y), make_float2(nib128<2>(lo), nib128<2>(hi)), a0);
        a1 = ffma2(make_float2(xc.z, xc.w), make_float2(nib128<3>(lo), nib128<3>(hi)), a1);
      }
      const float A = (a0.x + a0.y) + (a1.x + a1.y);
      const float sc = bf16_lo(sl.sb[r]), bi = bf16_hi(sl.sb[r]);
      acc[r][t] = fmaf(sc, A, fmaf(fmaf(-128.f, sc, bi), xsm, acc[r][t]));
    }
  }
}

// Each warp owns a contiguous run of GR-row groups and streams them as a flat
// sequence of items (group-major, lane-strided 16-byte columns inside a row)
// through a two-slot register ring, so 2 * GR loads per lane stay in flight
// across group boundaries.
template <int MT, int EPI>
__global__ void __launch_bounds__(GW * 32, MT == 1 ? 2 : 1) gemv_kernel(const GemvArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float smem[];
  constexpr int GR = Rows<MT, EPI>::value;
  const int K = a.K;
  float* xs = smem;
  float* xsum = xs + MT * K;
  float* red = xsum + MT * (K >> 5);
  stage_rows<MT>(a.x, a.ldx, K, a.norm_w, a.eps, xs, xsum, red);

  constexpr int VPR = (EPI == EPI_SWIGLU) ? 2 : 1;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * GW + (threadIdx.x >> 5);
  const int K32 = K >> 5, NCL = (K32 + 31) >> 5;
  const int vtotal = a.total_rows * VPR;
  const int gtotal = (vtotal + GR - 1) / GR;
  const int g0 = gw * a.rows_per_warp;  // rows_per_warp counts GR-row groups here
  const int ng = min(a.rows_per_warp, gtotal - g0);
  if (ng <= 0) return;
  const int items = ng * NCL;
  const size_t K8 = K >> 3, K64 = K >> 6;

  // issue-side cursor
  int ig = 0, ic = 0;
  const uint4* wrow[GR];
  const bf16* srow[GR];
  const bf16* brow[GR];
  auto set_rows = [&](int g) {
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      const int v = (g0 + g) * GR + r;
      wrow[r] = nullptr;
      srow[r] = brow[r] = nullptr;
      if (v < vtotal) {
        int si, rr;
        vrow_locate<EPI>(a, v, si, rr);
        const GemvSeg& sg = a.seg[si];
        wrow[r] = reinterpret_cast<const uint4*>(sg.w + size_t(rr) * K8);
        srow[r] = sg.s + size_t(rr) * K64;
        brow[r] = sg.b + size_t(rr) * K64;
      }
    }
  };
  set_rows(0);
  auto advance = [&]() {
    if (++ic == NCL) {
      ic = 0;
      if (++ig < ng) set_rows(ig);
    }
  };
  Slot<GR> s0, s1;
  issue<GR>(wrow, srow, brow, lane, K32, s0);
  advance();
  if (1 < items) issue<GR>(wrow, srow, brow, lane + 32 * ic, K32, s1);
  advance();

  float acc[GR][MT];
#pragma unroll
  for (int r = 0; r < GR; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;
  int cg = 0, cc = 0;
  auto finish = [&]() {
    // a GR-row group is complete: reduce and write
    if constexpr (EPI == EPI_SWIGLU) {
      static_assert(GR % 2 == 0, "SWIGLU pairs gate/up rows inside a group");
#pragma unroll
      for (int r = 0; r < GR; r += 2) {
        const int v = (g0 + cg) * GR + r;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float gv = rbf(warp_sum(acc[r][t]));
          const float uv = rbf(warp_sum(acc[r + 1][t]));
          if (lane == t && v < vtotal) {
            const float sg = rbf(1.f / (1.f + expf(-gv)));
            a.seg[0].y[t * a.ldy + (v >> 1)] = f2bf(rbf(gv * sg) * uv);
          }
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < GR; ++r) {
        const int v = (g0 + cg) * GR + r;
        int si = 0, rr = 0;
        if (v < vtotal) locate(a, v, si, rr);
        const GemvSeg& sg = a.seg[si];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float val = warp_sum(acc[r][t]);
          if (lane == t && v < vtotal) {
            if constexpr (EPI == EPI_STORE) {
              sg.y[t * a.ldy + rr] = f2bf(val);
            } else if constexpr (EPI == EPI_RESIDUAL) {
              bf16* p = sg.y + t * a.ldy + rr;
              *p = f2bf(bf2f(*p) + rbf(val));
            } else {
              sg.yf[t * a.ldy + rr] = val;
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < GR; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;
  };
  for (int j = 0; j < items; j += 2) {
    consume<MT, GR>(s0, xs, xsum, K, K32, lane + 32 * cc, acc);
    if (j + 2 < items) issue<GR>(wrow, srow, brow, lane + 32 * ic, K32, s0);
    advance();
    if (++cc == NCL) { finish(); cc = 0; ++cg; }
    if (j + 1 < items) {
      consume<MT, GR>(s1, xs, xsum, K, K32, lane + 32 * cc, acc);
      if (j + 3 < items) issue<GR>(wrow, srow, brow, lane + 32 * ic, K32, s1);
      advance();
      if (++cc == NCL) { finish(); cc = 0; ++cg; }
    }
  }
}

// Per-device zeroed scratch for tensor-core GEMV calls that bring none
// (standalone m5_quantized_matmul / m5_moe_route).  Grows, never shrinks.
int gemv_default_scratch(int rows, float** acc, int** cnt, int* cap_rows, float** part, size_t* part_floats) {
  static std::mutex mu;
  static char* buf[64] = {nullptr};
  static int cap[64] = {0};
  static float* slots[64] = {nullptr};
  int dev = 0;
  M5_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(M5_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (cap[dev] < rows) {
    const int want = std::max(rows, 1 << 16);
    const int r16 = (want + 15) / 16 * 16;
    char* p = nullptr;
    if (buf[dev]) {
      M5_CUDA(cudaDeviceSynchronize());
      M5_CUDA(cudaFree(buf[dev]));
      buf[dev] = nullptr;
      cap[dev] = 0;
    }
    M5_CUDA(cudaMalloc(&p, gemv_mma_scratch_bytes(r16)));
    M5_CUDA(cudaMemset(p, 0, gemv_mma_scratch_bytes(r16)));
    buf[dev] = p;
    cap[dev] = r16;
  }
  if (!slots[dev]) M5_CUDA(cudaMalloc(&slots[dev], gemv_part_floats() * sizeof(float)));
  *acc = reinterpret_cast<float*>(buf[dev]);
  *cnt = reinterpret_cast<int*>(buf[dev] + size_t(8) * cap[dev] * sizeof(float));
  *cap_rows = cap[dev];
  *part = slots[dev];
  *part_floats = gemv_part_floats();
  return M5_OK;
}

static size_t gemv_smem(int MT, int K) { return size_t(MT) * K * 4 + size_t(MT) * (K / 32) * 4 + 33 * 4; }

int gemv_max_tokens(int K) {
  for (int mt = 8; mt >= 1; mt >>= 1)
    if (gemv_smem(mt, K) <= 200 * 1024) return mt;
  return 0;
}

template <int MT, int EPI>
static int launch_t(const GemvArgs& a_in, cudaStream_t stream) {
  GemvArgs a = a_in;
  const size_t smem = gemv_smem(MT, a.K);
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(gemv_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024); }));
  // One wave: as many warps as fit on the device at this shared-memory size,
  // whole rows per warp.
  int per_sm = 0;
  M5_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kernel<MT, EPI>, GW * 32, smem));
  const long long resident = (long long)std::max(1, per_sm) * sm_count() * GW;
  const int groups = ceil_div((long long)a.total_rows * (EPI == EPI_SWIGLU ? 2 : 1), Rows<MT, EPI>::value);
  a.rows_per_warp = std::max(1, ceil_div(groups, resident));
  const int warps_total = ceil_div(groups, a.rows_per_warp);
  const int blocks = ceil_div(warps_total, GW);
  M5_CUDA(launch_pdl(gemv_kernel<MT, EPI>, dim3(blocks), dim3(GW * 32), smem, stream, a));
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
  if (a.total_rows <= 0) return M5_OK;
  const bool tmap = gemv_tmap_eligible(a, MT, epi);
  if (a.rope_cnt && !(tmap && epi == EPI_STORE && a.rope.L == MT))
    return fail(M5_ERR_INVALID, "gemv: the fused rope epilogue needs the tensor-map GEMV, EPI_STORE and rope.L == MT");
  if (tmap || gemv_mma_eligible(a, MT, epi)) {
    const int vrows = a.total_rows * (epi == EPI_SWIGLU ? 2 : 1);
    float* acc = a.mma_acc;
    int* cnt = a.mma_cnt;
    int rows = a.mma_rows;
    float* part = a.mma_part;
    size_t part_floats = a.mma_part_floats;
    if (!(acc && cnt && rows >= vrows && (!tmap || (part && part_floats >= gemv_part_floats())))) {
      int rc = gemv_default_scratch(vrows, &acc, &cnt, &rows, &part, &part_floats);
      if (rc) return rc;
    }
    if (tmap) return gemv_tmap_launch(a, MT, epi, part, part_floats, cnt, rows, stream);
    return gemv_mma_launch(a, MT, epi, acc, cnt, rows, stream);
  }
  if (gemv_tma_eligible(a.K, MT, epi)) return gemv_tma_launch(a, MT, epi, stream);
  if (gemv_smem(MT, a.K) > 200 * 1024) return fail(M5_ERR_INVALID, "gemv: too many tokens for this K");
  switch (MT) {
    case 1: return launch_epi<1>(a, epi, stream);
    case 2: return launch_epi<2>(a, epi, stream);
    case 4: return launch_epi<4>(a, epi, stream);
    case 8: return launch_epi<8>(a, epi, stream);
  }
  return fail(M5_ERR_INVALID, "gemv: MT must be 1, 2, 4 or 8");
}

}  // namespace m5
