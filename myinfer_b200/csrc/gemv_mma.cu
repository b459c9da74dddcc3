// Decode dequant-GEMV on the tensor cores (kernel K1; M <= 8 tokens).
//
// Why: the CUDA-core GEMVs spent ~5 issue slots per 4-bit weight (nibble
// extraction, int->float, fp32 FMA, activation loads) and topped out near
// 2 TB/s with 12-16 warps per SM.  Here the K-reduction runs on mma.sync
// m16n8k16 (bf16 in, fp32 accumulate) and a code becomes an operand with one
// LOP3 per two codes: (word >> 4i) & 0x000F000F | 0x43004300 is the bf16 pair
// (128 + q_i, 128 + q_{i+4}) exactly.  Per 64-element scale group the MMA
// result D = sum x*(128+q) is folded as  s*D + (b - 128*s) * sum(x)  into an
// fp32 accumulator, which equals sum x*(s*q + b) (the MLX dequantized row).
//
// Layout of one warp step (one 64-element group of a 16-row tile):
//   A (weights): lane (g, t) loads words 2t, 2t+1 of the group for rows g and
//     g+8 (two 8-byte loads; a quad covers the row's 32 bytes) -> 8 bf16 pairs
//     per row; MMA m uses pairs 2m, 2m+1.  Every MMA stays inside one group.
//   B (activations): staged once per CTA in shared memory in exactly that
//     permuted order, column n = token (lanes with n >= M read token M-1).
//   D: rows g, g+8 x tokens 2t, 2t+1 per lane.
// Work split: the (tile, group) steps of the whole matrix are dealt out as
// equal contiguous ranges to every warp of the grid (balanced to one step).
// A warp flushes its partial row sums with fp32 atomics into a zeroed scratch
// row and adds its step count to the tile's counter; whoever completes the
// tile runs the epilogue (bf16 store / residual add / SwiGLU) and re-zeroes
// the scratch, so consecutive launches (and graph replays) reuse it.
// Weight loads are prefetched PIPE steps ahead in registers.
#include <algorithm>

#include "frag_stage.cuh"
#include "gemv.cuh"
#include "mma_dq.cuh"

namespace m5 {

constexpr int MW = 8;      // warps per CTA
constexpr int PIPE_S = 12;  // steps prefetched per warp

struct MmaScratch {
  float* acc;      // [8][acc_rows] fp32, zero between launches
  int* cnt;        // [acc_rows / 16] step counters, zero between launches
  int acc_rows;
};

// Virtual row v -> (segment, row in segment).  SWIGLU tiles hold 8 gate rows
// (tile rows 0-7) and the matching 8 up rows (tile rows 8-15).
template <int EPI>
__device__ __forceinline__ void mma_row(const GemvArgs& a, int tile, int r16, int& si, int& rr) {
  if constexpr (EPI == EPI_SWIGLU) {
    si = r16 >> 3;
    rr = tile * 8 + (r16 & 7);
  } else {
    int v = tile * 16 + r16;
    si = 0;
    while (si < a.nseg - 1 && v >= a.seg[si].rows) {
      v -= a.seg[si].rows;
      ++si;
    }
    rr = v;
  }
}

template <int MT, int EPI>
__global__ void __launch_bounds__(MW * 32, 2) gemv_mma_kernel(const GemvArgs a, MmaScratch sc) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int K = a.K, NG = K >> 6;
  uint32_t* xf = reinterpret_cast<uint32_t*>(smem_raw);          // [MT][NG][4 t][8] bf16 pairs
  float* xg = reinterpret_cast<float*>(xf + MT * NG * 32);        // [MT][NG] group sums
  float* red = xg + MT * NG;                                      // [33]

  // ---- stage activations (optionally RMS-normalised) in fragment order
  const int tid = threadIdx.x;
  stage_frag<MT, MW * 32>(a.x, a.ldx, K, a.norm_w, a.eps, xf, xg, red, 0);

  // ---- this warp's range of (tile, group) steps
  const int lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int vrows = a.total_rows * (EPI == EPI_SWIGLU ? 2 : 1);
  const int ntiles = vrows >> 4;
  const long long total = (long long)ntiles * NG;
  const long long nwarps = (long long)gridDim.x * MW;
  const long long wid = (long long)blockIdx.x * MW + (tid >> 5);
  const long long s_begin = total * wid / nwarps, s_end = total * (wid + 1) / nwarps;
  if (s_begin >= s_end) return;
  const int tok = g < MT ? g : MT - 1;   // B column n = g reads this token
  const uint32_t* xfl = xf + tok * NG * 32 + tq * 8;
  const size_t K8 = K >> 3, K64 = K >> 6;

  // issue-side cursor
  long long is = s_begin;
  int it_tile = int(is / NG), it_G = int(is % NG);
  const uint32_t* w_g = nullptr;   // row g words
  const uint32_t* w_g8 = nullptr;  // row g+8 words
  const bf16 *s_g = nullptr, *b_g = nullptr, *s_g8 = nullptr, *b_g8 = nullptr;
  auto set_tile = [&](int tile) {
    int si, rr;
    mma_row<EPI>(a, tile, g, si, rr);
    w_g = a.seg[si].w + rr * K8 + 2 * tq;
    s_g = a.seg[si].s + rr * K64;
    b_g = a.seg[si].b + rr * K64;
    mma_row<EPI>(a, tile, g + 8, si, rr);
    w_g8 = a.seg[si].w + rr * K8 + 2 * tq;
    s_g8 = a.seg[si].s + rr * K64;
    b_g8 = a.seg[si].b + rr * K64;
  };
  set_tile(it_tile);

  uint2 rw[PIPE_S], rw8[PIPE_S];
  uint32_t rsb[PIPE_S], rsb8[PIPE_S];
  auto issue = [&](int slot) {
    if (is < s_end) {
      rw[slot] = ldg_nc_u2(w_g + it_G * 8);
      rw8[slot] = ldg_nc_u2(w_g8 + it_G * 8);
      rsb[slot] = uint32_t(ldg_nc_u16(s_g + it_G)) | (uint32_t(ldg_nc_u16(b_g + it_G)) << 16);
      rsb8[slot] = uint32_t(ldg_nc_u16(s_g8 + it_G)) | (uint32_t(ldg_nc_u16(b_g8 + it_G)) << 16);
      ++is;
      if (++it_G == NG) {
        it_G = 0;
        if (is < s_end) set_tile(++it_tile);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < PIPE_S; ++s) issue(s);

  // consume-side cursor
  long long cs = s_begin;
  int c_tile = int(cs / NG), c_G = int(cs % NG), c_done = 0;
  float tot[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8 x tokens 2tq, 2tq+1: (g,2t) (g,2t+1) (g8,2t) (g8,2t+1)

  auto flush = [&]() {
    // partial sums of tile c_tile -> scratch; last contributor finishes the tile
    const int t0 = 2 * tq, t1 = 2 * tq + 1;
    float* acc = sc.acc;
    const int base = c_tile * 16;
    if (t0 < MT) {
      atomicAdd(&acc[t0 * sc.acc_rows + base + g], tot[0]);
      atomicAdd(&acc[t0 * sc.acc_rows + base + g + 8], tot[2]);
    }
    if (t1 < MT) {
      atomicAdd(&acc[t1 * sc.acc_rows + base + g], tot[1]);
      atomicAdd(&acc[t1 * sc.acc_rows + base + g + 8], tot[3]);
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(&sc.cnt[c_tile], c_done) + c_done == NG);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      // lane handles (token, row) pairs of the tile: 16 rows x MT tokens
      for (int q = lane; q < 16 * MT; q += 32) {
        const int r16 = q & 15, t = q >> 4;
        float* p = &acc[t * sc.acc_rows + base + r16];
        if constexpr (EPI == EPI_SWIGLU) {
          // lane of gate row r16 consumes (and clears) both its gate and up slot
          if (r16 < 8) {
            float* pu = &acc[t * sc.acc_rows + base + r16 + 8];
            const float v = __ldcg(p), u = __ldcg(pu);
            *p = 0.f;
            *pu = 0.f;
            const float gv = rbf(v), uv = rbf(u);
            const float sg = rbf(1.f / (1.f + expf(-gv)));
            a.seg[0].y[t * a.ldy + c_tile * 8 + r16] = f2bf(rbf(gv * sg) * uv);
          }
        } else {
          const float v = __ldcg(p);
          *p = 0.f;
          int si, rr;
          mma_row<EPI>(a, c_tile, r16, si, rr);
          const GemvSeg& sg = a.seg[si];
          if constexpr (EPI == EPI_STORE) {
            sg.y[t * a.ldy + rr] = f2bf(v);
          } else if constexpr (EPI == EPI_RESIDUAL) {
            bf16* o = sg.y + t * a.ldy + rr;
            *o = f2bf(bf2f(*o) + rbf(v));
          } else {
            sg.yf[t * a.ldy + rr] = v;
          }
        }
      }
      __syncwarp();
      if (lane == 0) sc.cnt[c_tile] = 0;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[i] = 0.f;
    c_done = 0;
  };

  const float* xgl0 = xg + (2 * tq < MT ? 2 * tq : MT - 1) * NG;
  const float* xgl1 = xg + (2 * tq + 1 < MT ? 2 * tq + 1 : MT - 1) * NG;
  for (long long s0 = s_begin; s0 < s_end; s0 += PIPE_S) {
#pragma unroll
    for (int slot = 0; slot < PIPE_S; ++slot) {
      if (s0 + slot < s_end) {
        // B fragments of this group: 8 bf16 pairs (2 x 16-byte shared loads)
        const uint4 xa = *reinterpret_cast<const uint4*>(xfl + c_G * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xfl + c_G * 32 + 4);
        const uint32_t wg[2] = {rw[slot].x, rw[slot].y}, wg8[2] = {rw8[slot].x, rw8[slot].y};
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        {
          uint32_t A[4] = {nib_pair(wg[0], 0), nib_pair(wg8[0], 0), nib_pair(wg[0], 1), nib_pair(wg8[0], 1)};
          mma_bf16(d, A, xa.x, xa.y);
        }
        {
          uint32_t A[4] = {nib_pair(wg[0], 2), nib_pair(wg8[0], 2), nib_pair(wg[0], 3), nib_pair(wg8[0], 3)};
          mma_bf16(d, A, xa.z, xa.w);
        }
        {
          uint32_t A[4] = {nib_pair(wg[1], 0), nib_pair(wg8[1], 0), nib_pair(wg[1], 1), nib_pair(wg8[1], 1)};
          mma_bf16(d, A, xb.x, xb.y);
        }
        {
          uint32_t A[4] = {nib_pair(wg[1], 2), nib_pair(wg8[1], 2), nib_pair(wg[1], 3), nib_pair(wg8[1], 3)};
          mma_bf16(d, A, xb.z, xb.w);
        }
        const float sA = bf16_lo(rsb[slot]), bA = bf16_hi(rsb[slot]);
        const float sB = bf16_lo(rsb8[slot]), bB = bf16_hi(rsb8[slot]);
        const float X0 = xgl0[c_G], X1 = xgl1[c_G];
        const float oA = fmaf(-128.f, sA, bA), oB = fmaf(-128.f, sB, bB);
        tot[0] = fmaf(sA, d[0], fmaf(oA, X0, tot[0]));
        tot[1] = fmaf(sA, d[1], fmaf(oA, X1, tot[1]));
        tot[2] = fmaf(sB, d[2], fmaf(oB, X0, tot[2]));
        tot[3] = fmaf(sB, d[3], fmaf(oB, X1, tot[3]));
        issue(slot);
        ++c_done;
        if (++c_G == NG) {
          flush();
          c_G = 0;
          ++c_tile;
        }
      }
    }
  }
  if (c_done) flush();
}

static size_t mma_smem(int MT, int K) { return size_t(MT) * (K / 64) * 32 * 4 + size_t(MT) * (K / 64) * 4 + 33 * 4; }

size_t gemv_mma_scratch_bytes(int rows) {
  rows = (rows + 15) / 16 * 16;
  return size_t(8) * rows * sizeof(float) + size_t(rows / 16) * sizeof(int);
}

bool gemv_mma_eligible(const GemvArgs& a, int MT, int epi) {
  if (MT < 1 || MT > 8 || a.K % 64) return false;
  if (mma_smem(MT, a.K) > 200 * 1024) return false;
  if (epi == EPI_SWIGLU) return a.total_rows % 8 == 0;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].rows % 16) return false;
  return true;
}

template <int MT, int EPI>
static int mma_launch_t(const GemvArgs& a, const MmaScratch& sc, cudaStream_t st) {
  const size_t smem = mma_smem(MT, a.K);
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(gemv_mma_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024); }));
  int per_sm = 0;
  M5_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_mma_kernel<MT, EPI>, MW * 32, smem));
  const int vrows = a.total_rows * (EPI == EPI_SWIGLU ? 2 : 1);
  const long long steps = (long long)(vrows / 16) * (a.K / 64);
  const long long max_ctas = (long long)std::max(1, per_sm) * sm_count();
  const int grid = (int)std::max(1LL, std::min(max_ctas, (steps + MW - 1) / MW));
  M5_CUDA(launch_pdl(gemv_mma_kernel<MT, EPI>, dim3(grid), dim3(MW * 32), smem, st, a, sc));
  M5_LAUNCH_CHECK("gemv_mma launch");
  return M5_OK;
}

template <int MT>
static int mma_launch_epi(const GemvArgs& a, int epi, const MmaScratch& sc, cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: return mma_launch_t<MT, EPI_STORE>(a, sc, st);
    case EPI_RESIDUAL: return mma_launch_t<MT, EPI_RESIDUAL>(a, sc, st);
    case EPI_SWIGLU: return mma_launch_t<MT, EPI_SWIGLU>(a, sc, st);
    case EPI_F32: return mma_launch_t<MT, EPI_F32>(a, sc, st);
  }
  return fail(M5_ERR_INVALID, "gemv_mma: bad epilogue");
}

int gemv_mma_launch(const GemvArgs& a, int MT, int epi, float* acc, int* cnt, int acc_rows, cudaStream_t st) {
  const int vrows = a.total_rows * (epi == EPI_SWIGLU ? 2 : 1);
  if (vrows > acc_rows) return fail(M5_ERR_INVALID, "gemv_mma: scratch too small for this matrix");
  MmaScratch sc{acc, cnt, acc_rows};
  switch (MT) {
    case 1: return mma_launch_epi<1>(a, epi, sc, st);
    case 2: return mma_launch_epi<2>(a, epi, sc, st);
    case 3: return mma_launch_epi<3>(a, epi, sc, st);
    case 4: return mma_launch_epi<4>(a, epi, sc, st);
    case 5: return mma_launch_epi<5>(a, epi, sc, st);
    case 6: return mma_launch_epi<6>(a, epi, sc, st);
    case 7: return mma_launch_epi<7>(a, epi, sc, st);
    case 8: return mma_launch_epi<8>(a, epi, sc, st);
  }
  return fail(M5_ERR_INVALID, "gemv_mma: MT must be 1..8");
}

}  // namespace m5
