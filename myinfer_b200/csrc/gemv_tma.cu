// TMA-fed streaming w4g64 dequant-GEMV for decode (kernel K1, M <= 2 tokens).
//
// The register-ring GEMV tops out near 2 TB/s because every byte in flight
// costs a register.  Here one producer warp per CTA streams weight tiles with
// 1-D bulk copies (the TMA engine) into a STAGES-deep shared-memory ring guarded
// by mbarriers, so ~36 KB per CTA (several CTAs per SM) are in flight without
// touching registers, and the consumer warps only do the dequant dot products:
//   tile  = TG_CW output rows (x2 rows gate|up for the SwiGLU epilogue), one
//           row per consumer warp;
//   stage = one TG_KC-element chunk of every row of the tile (packed words +
//           bf16 scales + bf16 biases, three bulk copies per row);
//   tiles are dealt to CTAs round-robin (blockIdx.x + i * gridDim.x).
// The activation rows are staged by the consumer warps (fused RMSNorm) while
// the producer's first copies are already in flight.  All mbarrier waits are
// bounded (tma.cuh); a wait that gives up records an error and the warp exits.
// Needs K % 512 == 0 (16-byte aligned scale rows); other K use gemv.cu.
#include <algorithm>

#include "gemv.cuh"
#include "gemv_impl.cuh"
#include "tma.cuh"

namespace m5 {

static __device__ int g_gemv_tma_err = 0;

constexpr int TG_CW = 4;                       // consumer warps = output rows per tile
constexpr int TG_THREADS = (TG_CW + 1) * 32;   // + one producer warp
constexpr int TG_KC = 4096;                    // elements of a row per stage
constexpr int TG_STAGES = 4;

template <int VPR>
struct TgLayout {
  static constexpr int ROWS = TG_CW * VPR;               // weight rows per tile
  static constexpr int W_BYTES = TG_KC / 2;              // packed bytes per row chunk
  static constexpr int S_BYTES = TG_KC / 32;             // bf16 scale bytes per row chunk
  static constexpr int STAGE = ROWS * (W_BYTES + 2 * S_BYTES);
};

// Consumer-only version of stage_rows (named barrier 1 over the consumer warps).
template <int MT>
__device__ __forceinline__ void stage_rows_consumers(const bf16* __restrict__ x, int64_t ldx, int K,
                                                     const bf16* __restrict__ norm_w, float eps, float* xs,
                                                     float* xsum, float* red) {
  constexpr int NT = TG_CW * 32;
  const int tid = threadIdx.x;
  for (int t = 0; t < MT; ++t) {
    const bf16* xr = x + t * ldx;
    float inv = 1.f;
    if (norm_w) {
      float ss = 0.f;
      for (int i = tid; i < K; i += NT) {
        const float v = bf2f(xr[i]);
        ss += v * v;
      }
      ss = warp_sum(ss);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
      named_sync(1, NT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < TG_CW; ++w) tot += red[w];
      inv = __frsqrt_rn(__fadd_rn(tot / float(K), eps));
      named_sync(1, NT);
    }
    float* xrow = xs + t * K;
    for (int i = tid; i < K; i += NT) {
      float v = bf2f(xr[i]);
      if (norm_w) v = rbf(__fmul_rn(bf2f(norm_w[i]), rbf(__fmul_rn(v, inv))));
      xrow[xs_index(i)] = v;
    }
  }
  named_sync(1, NT);
  const int K32 = K >> 5;
  for (int j = tid; j < MT * K32; j += NT) {
    const float4* p = reinterpret_cast<const float4*>(xs + (j / K32) * K + (j % K32) * 32);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 v = p[q];
      s += (v.x + v.y) + (v.z + v.w);
    }
    xsum[j] = s;
  }
  named_sync(1, NT);
}

template <int EPI>
__device__ __forceinline__ bool tg_row(const GemvArgs& a, int tile, int r, int& si, int& rr) {
  // weight row r of a tile -> (segment, row); false past the end
  if constexpr (EPI == EPI_SWIGLU) {
    const int out_row = tile * TG_CW + (r >> 1);
    if (out_row >= a.total_rows) return false;
    si = r & 1;
    rr = out_row;
    return true;
  } else {
    const int v = tile * TG_CW + r;
    if (v >= a.total_rows) return false;
    int s, q;
    // locate segment
    q = v;
    s = 0;
    while (s < a.nseg - 1 && q >= a.seg[s].rows) {
      q -= a.seg[s].rows;
      ++s;
    }
    si = s;
    rr = q;
    return true;
  }
}

template <int MT, int EPI>
__global__ void __launch_bounds__(TG_THREADS) gemv_tma_kernel(const GemvArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int VPR = (EPI == EPI_SWIGLU) ? 2 : 1;
  using LY = TgLayout<VPR>;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TG_STAGES * LY::STAGE);
  uint64_t* empty = full + TG_STAGES;
  float* xs = reinterpret_cast<float*>(empty + TG_STAGES);
  const int K = a.K;
  float* xsum = xs + MT * K;
  float* red = xsum + MT * (K >> 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = (K + TG_KC - 1) / TG_KC;
  const int ntiles = (a.total_rows + TG_CW - 1) / TG_CW;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TG_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], TG_CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == TG_CW) {
    // ---------------- producer: one lane issues every bulk copy
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const size_t K8 = K >> 3, K64 = K >> 6;
      int it = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        for (int c = 0; c < nchunks; ++c, ++it) {
          const int st = it % TG_STAGES;
          const uint32_t par = (it / TG_STAGES) & 1;
          if (!mbar_wait(&empty[st], par ^ 1, &g_gemv_tma_err)) return;
          const int k0 = c * TG_KC;
          const int klen = min(TG_KC, K - k0);
          uint32_t bytes = 0;
          int si[LY::ROWS], rr[LY::ROWS];
          bool ok[LY::ROWS];
#pragma unroll
          for (int r = 0; r < LY::ROWS; ++r) {
            ok[r] = tg_row<EPI>(a, tile, r, si[r], rr[r]);
            if (ok[r]) bytes += klen / 2 + 2 * (klen / 32);
          }
          mbar_arrive_expect_tx(&full[st], bytes);
          unsigned char* sw = stages + st * LY::STAGE;
          unsigned char* ss = sw + LY::ROWS * LY::W_BYTES;
          unsigned char* sb = ss + LY::ROWS * LY::S_BYTES;
#pragma unroll
          for (int r = 0; r < LY::ROWS; ++r) {
            if (!ok[r]) continue;
            const GemvSeg& sg = a.seg[si[r]];
            bulk_g2s_stream(sw + r * LY::W_BYTES, sg.w + rr[r] * K8 + k0 / 8, klen / 2, &full[st], pol);
            bulk_g2s_stream(ss + r * LY::S_BYTES, sg.s + rr[r] * K64 + k0 / 64, klen / 32, &full[st], pol);
            bulk_g2s_stream(sb + r * LY::S_BYTES, sg.b + rr[r] * K64 + k0 / 64, klen / 32, &full[st], pol);
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers: stage x, then one output row per warp per tile
  stage_rows_consumers<MT>(a.x, a.ldx, K, a.norm_w, a.eps, xs, xsum, red);
  const int K32 = K >> 5;
  int it = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float acc[VPR][MT];
#pragma unroll
    for (int v = 0; v < VPR; ++v)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[v][t] = 0.f;
    for (int c = 0; c < nchunks; ++c, ++it) {
      const int st = it % TG_STAGES;
      const uint32_t par = (it / TG_STAGES) & 1;
      if (!mbar_wait(&full[st], par, &g_gemv_tma_err)) return;
      const int k0 = c * TG_KC;
      const int n16 = min(TG_KC, K - k0) >> 5;  // 16-byte blocks per row in this chunk
      const unsigned char* sw = stages + st * LY::STAGE;
      const bf16* ss = reinterpret_cast<const bf16*>(sw + LY::ROWS * LY::W_BYTES);
      const bf16* sb = reinterpret_cast<const bf16*>(sw + LY::ROWS * (LY::W_BYTES + LY::S_BYTES));
#pragma unroll
      for (int v = 0; v < VPR; ++v) {
        const int r = warp * VPR + v;
        const uint4* wr = reinterpret_cast<const uint4*>(sw + r * LY::W_BYTES);
        const bf16* sr = ss + r * (LY::S_BYTES / 2);
        const bf16* br = sb + r * (LY::S_BYTES / 2);
        for (int u = lane; u < n16; u += 32) {
          const uint4 wv = wr[u];
          const float sc = bf2f(sr[u >> 1]), bi = bf2f(br[u >> 1]);
          const float off = fmaf(-128.f, sc, bi);
          const int blk = (k0 >> 5) + u;
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const float A = dot32(wv, xs + t * K, blk);
            acc[v][t] = fmaf(sc, A, fmaf(off, xsum[t * K32 + blk], acc[v][t]));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // epilogue for this warp's output row
    if constexpr (EPI == EPI_SWIGLU) {
      const int row = tile * TG_CW + warp;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float gv = rbf(warp_sum(acc[0][t]));
        const float uv = rbf(warp_sum(acc[1][t]));
        if (lane == t && row < a.total_rows) {
          const float sg = rbf(1.f / (1.f + expf(-gv)));
          a.seg[0].y[t * a.ldy + row] = f2bf(rbf(gv * sg) * uv);
        }
      }
    } else {
      int si = 0, rr = 0;
      const bool ok = tg_row<EPI>(a, tile, warp, si, rr);
      const GemvSeg& sg = a.seg[si];
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float val = warp_sum(acc[0][t]);
        if (lane == t && ok) {
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
}

static size_t tma_smem(int MT, int K, int vpr) {
  const size_t stage = size_t(TG_CW) * vpr * (TG_KC / 2 + 2 * (TG_KC / 32));
  return TG_STAGES * stage + 2 * TG_STAGES * 8 + size_t(MT) * K * 4 + size_t(MT) * (K / 32) * 4 + 33 * 4;
}

bool gemv_tma_eligible(int K, int MT, int epi) {
  if (MT > 2 || K % 512 != 0) return false;
  return tma_smem(MT, K, epi == EPI_SWIGLU ? 2 : 1) <= 200 * 1024;
}

template <int MT, int EPI>
static int tma_launch_t(const GemvArgs& a, cudaStream_t st) {
  const size_t smem = tma_smem(MT, a.K, EPI == EPI_SWIGLU ? 2 : 1);
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(gemv_tma_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024); }));
  int per_sm = 0;
  M5_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_tma_kernel<MT, EPI>, TG_THREADS, smem));
  const int ntiles = (a.total_rows + TG_CW - 1) / TG_CW;
  const int grid = std::max(1, std::min(ntiles, std::max(1, per_sm) * sm_count()));
  M5_CUDA(launch_pdl(gemv_tma_kernel<MT, EPI>, dim3(grid), dim3(TG_THREADS), smem, st, a));
  M5_LAUNCH_CHECK("gemv_tma launch");
  return M5_OK;
}

template <int MT>
static int tma_launch_epi(const GemvArgs& a, int epi, cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: return tma_launch_t<MT, EPI_STORE>(a, st);
    case EPI_RESIDUAL: return tma_launch_t<MT, EPI_RESIDUAL>(a, st);
    case EPI_SWIGLU: return tma_launch_t<MT, EPI_SWIGLU>(a, st);
    case EPI_F32: return tma_launch_t<MT, EPI_F32>(a, st);
  }
  return fail(M5_ERR_INVALID, "gemv_tma: bad epilogue");
}

int gemv_tma_launch(const GemvArgs& a, int MT, int epi, cudaStream_t st) {
  if (MT == 1) return tma_launch_epi<1>(a, epi, st);
  if (MT == 2) return tma_launch_epi<2>(a, epi, st);
  return fail(M5_ERR_INVALID, "gemv_tma: MT must be 1 or 2");
}

int gemv_tma_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_tma_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gemv_tma_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
