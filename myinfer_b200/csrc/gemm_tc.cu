// Prefill dequant-GEMM on the fifth-generation tensor cores (kernel K2):
// Y[M, N] = epi(X[M, K] @ dequant(W)^T) for M >= 16 tokens, w4 g64 weights.
//
// Exactness.  MLX computes with w = q * s + b held in fp32.  Rounding w to
// bf16 for the tensor core would add a 2^-9 relative error to every weight, so
// the product is split into exactly representable bf16 parts instead:
//     q * s = hi + lo,  hi = bf16(q * s),  lo = q * s - hi
// (q has 4 significant bits and s 8, so q * s has at most 12 and the remainder
// lo at most 5: both are exact bf16 values, computed with one bf16x2 multiply
// and one bf16x2 FMA per pair), and
//     sum_k w[n,k] x[m,k] = sum_k hi x + sum_k lo x + sum_g b[n,g] xs[m,g],
//     xs[m,g] = sum_{k in g} x[m,k]  (fp32, split into bf16 hi + lo).
// Per 64-column group the tensor core runs eight 128 x 128 x 16 MMAs (hi and lo
// against the same X slice) and, after the last group, 4 MMAs per 32 groups of
// A = [b | b] against B = [xs_hi | xs_lo].  The tensor core's fp32 accumulation
// is not IEEE round-to-nearest over long chains, and the bias term cancels much
// of the main term, so partial sums are promoted every NG groups: the MMAs of a
// unit of NG groups (or of all bias blocks) accumulate in one of two TMEM
// buffers, which promoter warps add into IEEE fp32 registers.
//
// Pipeline (one persistent CTA per SM, tiles of 128 weight rows x 128 tokens):
//   warp 16     TMA producer: X tile (128 x 64 bf16, 128-byte swizzle) and the
//               packed weight tile (128 rows x 32 B) per group; xs and bias
//               tiles for the bias blocks; 8-stage ring;
//   warp 17     MMA issuer: tcgen05.mma kind::f16, A from tensor memory, B = X
//               tile from shared memory, D = one of two TMEM partial buffers;
//   warps 8-15  dequant: two sets of four warps take alternate blocks; thread =
//               weight row (its TMEM lane); writes hi | lo (64 columns) into a
//               4-slot A ring in tensor memory;
//   warps 0-7   promote + epilogue: thread = weight row, 64 of the 128 tokens;
//               adds each partial buffer into fp32 registers, then applies the
//               epilogue while the MMA already runs the next tile.
// Every mbarrier wait is bounded in time; a timeout sets a CTA-wide failure
// flag that ends all roles, records a device error and still frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "gemv.cuh"
#include "tcgen05.cuh"

namespace m5 {

static __device__ int g_gemm_tc_err = 0;

namespace gtc {

constexpr int BR = 128;          // weight rows per tile (MMA M)
constexpr int BT = 128;          // tokens per tile (MMA N)
constexpr int NS = 8;            // shared-memory stages (covers ~5 us of loaded L2 latency)
constexpr int NA = 4;            // A slots in tensor memory (64 columns each: hi | lo)
constexpr int X_BYTES = BT * 128;            // 64 bf16 per token row
constexpr int W_BYTES = 8192;                // 128 rows x 32 B (codes) or 128 rows x 64 B (biases)
constexpr int STAGE = X_BYTES + W_BYTES;     // multiple of 1024
constexpr int NG = 4;            // groups per promoted partial sum
constexpr int THREADS = 18 * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t P_COL = 0;                // partial buffers at columns 0 and 128
constexpr uint32_t A_COL = 256;              // A slots at 256 + 64 a
constexpr size_t SMEM = 1024 + size_t(NS) * STAGE + 256;

struct Seg {
  const bf16* s;   // scales [rows, G]
  int rows;
  bf16* y;         // output column base
  float* yf;
};

struct Params {
  int M, K, G, C;      // tokens, reduction length, scale groups, bias blocks (ceil(G / 32))
  int gld;             // scale / bias row stride in groups (G, or more for a K slice)
  int vec_sb;          // G % 8 == 0: 16-byte scale loads and TMA bias tiles (else scalar global loads)
  const bf16* bias[3]; // per segment, for the scalar bias path
  int nseg;
  Seg seg[3];
  int64_t ldy;
  int n_tiles, m_tiles;
  uint32_t hint_ns;    // suspend-time hint of the mbarrier waits (0 = poll)
};

struct Maps {
  CUtensorMap x, xs, w[3], b[3];
};

__device__ __forceinline__ void tile_rows(const Params& p, int epi, int nt, int& si, int& row0) {
  if (epi == EPI_SWIGLU) {
    si = 0;
    row0 = nt * (BR / 2);
    return;
  }
  int v = nt * BR;
  si = 0;
  while (si < p.nseg - 1 && v >= p.seg[si].rows) {
    v -= p.seg[si].rows;
    ++si;
  }
  row0 = v;
}

// Segment and row of tile row r (SwiGLU tiles interleave 16 gate rows and the
// same 16 up rows per 32-row lane quadrant).
template <int EPI>
__device__ __forceinline__ void row_of(const Params& p, int si, int row0, int r, int& seg, int& grow) {
  if (EPI == EPI_SWIGLU) {
    seg = (r & 16) ? 1 : 0;
    grow = row0 + 16 * (r >> 5) + (r & 15);
  } else {
    seg = si;
    grow = row0 + r;
  }
}

// Bounded wait by one thread, ~2 s of wall time.  hint_ns = 0 polls; otherwise
// each try_wait may suspend the thread until the phase completes (or the hint
// runs out), so a waiting role does not take issue slots from working warps.
__device__ __forceinline__ uint64_t gtc_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool gtc_try_wait_hint(uint64_t* bar, uint32_t par, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(par), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait1(uint64_t* bar, uint32_t par, volatile int* fail, uint32_t hint_ns) {
  if (mbar_try_wait_fast(bar, par)) return true;
  const uint64_t t0 = gtc_now_ns();
  for (uint32_t i = 1;; ++i) {
    if (hint_ns ? gtc_try_wait_hint(bar, par, hint_ns) : mbar_try_wait_fast(bar, par)) return true;
    if (*fail) return false;
    if ((hint_ns || (i & 255) == 0) && gtc_now_ns() - t0 > 2000000000ull) break;
  }
  *fail = 1;
  atomicExch(&g_gemm_tc_err, M5_DEV_ERR_WAIT_TIMEOUT);
  return false;
}

// Bounded wait by a whole warp with a warp-uniform result.
__device__ __forceinline__ bool waitw(uint64_t* bar, uint32_t par, volatile int* fail, int lane, uint32_t hint_ns) {
  bool ok = true;
  if (lane == 0) ok = wait1(bar, par, fail, hint_ns);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_try_wait_fast(bar, par);  // acquire for every lane (the phase is complete)
  return ok;
}

// Wait of a group of warps that share one named barrier: a single poller warp
// waits (bounded), then the group meets at the barrier and every thread reads
// the poller's verdict from a double-buffered flag (so a slow reader never sees
// the next call's value) and takes its own acquire on the completed phase.
struct GroupWait {
  int id, threads;
  volatile int* flag;  // [2]
  int calls;
  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t par, volatile int* fail, bool poller, int lane,
                                       uint32_t hint_ns) {
    const int slot = calls++ & 1;
    if (poller) {
      bool ok = true;
      if (lane == 0) ok = wait1(bar, par, fail, hint_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane == 0) flag[slot] = ok ? 1 : 0;
    }
    named_sync(id, threads);
    if (!flag[slot]) return false;
    (void)mbar_try_wait_fast(bar, par);
    return true;
  }
};

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t sub128(uint32_t v) {
  return bfma2(v, 0x3F803F80u, 0xC300C300u);  // v * 1 - 128 (exact)
}

// 8 codes (low bits first) of one word times the scale pair s2 ->
// hi[0..3] and nlo[0..3] = -lo: bf16 pairs for k = (0,1) (2,3) (4,5) (6,7)
// (s2n = -s2; the MMA of the lo part negates A through its descriptor).
__device__ __forceinline__ void codes_hi_lo(uint32_t w, uint32_t s2, uint32_t s2n, uint32_t* hi, uint32_t* nlo) {
  const uint32_t t0 = (w & 0x000F000Fu) | 0x43004300u;          // (128+q0, 128+q4)
  const uint32_t t1 = ((w >> 4) & 0x000F000Fu) | 0x43004300u;   // (q1, q5)
  const uint32_t t2 = ((w >> 8) & 0x000F000Fu) | 0x43004300u;   // (q2, q6)
  const uint32_t t3 = ((w >> 12) & 0x000F000Fu) | 0x43004300u;  // (q3, q7)
  const uint32_t q[4] = {sub128(__byte_perm(t0, t1, 0x5410)), sub128(__byte_perm(t2, t3, 0x5410)),
                         sub128(__byte_perm(t0, t1, 0x7632)), sub128(__byte_perm(t2, t3, 0x7632))};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    hi[i] = bmul2(q[i], s2);
    nlo[i] = bfma2(q[i], s2n, hi[i]);  // hi - q*s, exact
  }
}

__device__ __forceinline__ uint32_t pick_bf16_pair(const uint4& v, int j) {
  const uint32_t w = (j < 4) ? ((j < 2) ? v.x : v.y) : ((j < 6) ? v.z : v.w);
  const uint32_t h = (j & 1) ? (w >> 16) : (w & 0xFFFFu);
  return h | (h << 16);
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ Params p,
                                                             const __grid_constant__ Maps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + size_t(NS) * STAGE);
  uint64_t* full = bars;
  uint64_t* empty = full + NS;
  uint64_t* a_full = empty + NS;
  uint64_t* a_empty = a_full + NA;
  uint64_t* p_full = a_empty + NA;
  uint64_t* p_empty = p_full + 2;
  uint64_t* done = p_empty + 2;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ int s_flags[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.G + p.C;
  const int total_tiles = p.n_tiles * p.m_tiles;
  const int my_tiles = blockIdx.x < total_tiles ? (total_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int my_blocks = my_tiles * nblk;
  volatile int* fail = &s_fail;

  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], 8);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&s_tmem, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int idx = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const int nt = t / p.m_tiles, mt = t % p.m_tiles;
        int si, row0;
        tile_rows(p, EPI, nt, si, row0);
        const int m0 = mt * BT;
        for (int b = 0; b < nblk; ++b, ++idx) {
          const int s = idx % NS;
          const uint32_t ph = (idx / NS) & 1;
          if (!wait1(&empty[s], ph ^ 1, fail, p.hint_ns)) {
            ok = false;
            break;
          }
          uint8_t* x_dst = stages + size_t(s) * STAGE;
          uint8_t* w_dst = x_dst + X_BYTES;
          if (b < p.G) {
            mbar_arrive_expect_tx(&full[s], X_BYTES + BR * 32);
            tma_load_2d(x_dst, &maps.x, b * 64, m0, &full[s]);
            if (EPI == EPI_SWIGLU) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                tma_load_2d(w_dst + (32 * qq) * 32, &maps.w[0], b * 8, row0 + 16 * qq, &full[s]);
                tma_load_2d(w_dst + (32 * qq + 16) * 32, &maps.w[1], b * 8, row0 + 16 * qq, &full[s]);
              }
            } else {
              tma_load_2d(w_dst, &maps.w[si], b * 8, row0, &full[s]);
            }
          } else {
            const int c = b - p.G;
            mbar_arrive_expect_tx(&full[s], X_BYTES + (p.vec_sb ? BR * 64 : 0));
            tma_load_2d(x_dst, &maps.xs, c * 64, m0, &full[s]);
            if (!p.vec_sb) {
              // biases are read by the dequant warps straight from global memory
            } else if (EPI == EPI_SWIGLU) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                tma_load_2d(w_dst + (32 * qq) * 64, &maps.b[0], c * 32, row0 + 16 * qq, &full[s]);
                tma_load_2d(w_dst + (32 * qq + 16) * 64, &maps.b[1], c * 32, row0 + 16 * qq, &full[s]);
              }
            } else {
              tma_load_2d(w_dst, &maps.b[si], c * 32, row0, &full[s]);
            }
          }
        }
      }
      // every issued copy lands before the CTA may exit
      const int issued = idx;
      for (int k = std::max(0, issued - NS); k < issued; ++k) (void)wait1(&full[k % NS], (k / NS) & 1, fail, p.hint_ns);
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc_bf16(BR, BT);
      constexpr uint32_t idesc_neg = idesc | (1u << 13);  // negate A (the lo part is stored as -lo)
      int idx = 0, unit = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        for (int b = 0; b < nblk; ++b, ++idx) {
          const bool first = (b < p.G) ? (b % NG == 0) : (b == p.G);
          const bool last = (b < p.G) ? (b % NG == NG - 1 || b == p.G - 1) : (b == nblk - 1);
          const int pb = unit & 1;
          const int s = idx % NS, a = idx % NA;
          if ((first && !wait1(&p_empty[pb], ((unit >> 1) & 1) ^ 1, fail, p.hint_ns)) ||
              !wait1(&full[s], (idx / NS) & 1, fail, p.hint_ns) || !wait1(&a_full[a], (idx / NA) & 1, fail, p.hint_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + P_COL + 128u * pb;
          const uint32_t aaddr = tmem + A_COL + 64u * a;
          const uint64_t bdesc = tc_sdesc_sw128(smem_addr(stages + size_t(s) * STAGE));
          if (b < p.G) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              tc_mma_ts(d, aaddr + 8u * k, bdesc + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
              tc_mma_ts(d, aaddr + 32u + 8u * k, bdesc + 2u * k, idesc_neg, 1u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) tc_mma_ts(d, aaddr + 8u * k, bdesc + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
          }
          tc_commit(&empty[s]);
          tc_commit(&a_empty[a]);
          if (last) {
            tc_commit(&p_full[pb]);
            ++unit;
          }
        }
      }
      tc_commit(done);
      (void)wait1(done, 0, fail, p.hint_ns);
    }
  } else if (warp >= 8) {
    // ----------------------------------------------------------------- dequant
    // Both sets work on every block: set 0 converts codes 0-31 of each row, set 1
    // codes 32-63 (A columns: hi 0-15 | 16-31, -lo 32-47 | 48-63).
    const int q = warp & 3, set = (warp - 8) >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    int cur_tile = -1, si = 0, row0 = 0;
    const uint4* srow = nullptr;
    const bf16* srow16 = nullptr;  // scalar path (G % 8 != 0)
    const bf16* brow16 = nullptr;
    int cur_w = -2;
    uint4 s_cur = make_uint4(0, 0, 0, 0), s_nxt = s_cur;
    // 8 scales of window w (16-byte load when rows are 16-byte aligned)
    auto load_win = [&](int w) -> uint4 {
      if (p.vec_sb) return srow[w];
      uint32_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = (8 * w + j < p.G) ? __bfloat16_as_ushort(srow16[8 * w + j]) : 0u;
      return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    };
    for (int idx = 0; idx < my_blocks; ++idx) {
      const int tl = idx / nblk, b = idx % nblk;
      if (tl != cur_tile) {
        cur_tile = tl;
        tile_rows(p, EPI, (blockIdx.x + tl * gridDim.x) / p.m_tiles, si, row0);
        int sg, grow;
        row_of<EPI>(p, si, row0, r, sg, grow);
        srow = reinterpret_cast<const uint4*>(p.seg[sg].s + size_t(grow) * p.gld);
        srow16 = p.seg[sg].s + size_t(grow) * p.gld;
        brow16 = p.bias[sg] + size_t(grow) * p.gld;
        cur_w = -2;
      }
      uint32_t s2 = 0;
      if (b < p.G) {
        const int w = b >> 3;
        if (w != cur_w) {
          s_cur = (w == cur_w + 1) ? s_nxt : load_win(w);
          cur_w = w;
          if (8 * (w + 1) < p.G) s_nxt = load_win(w + 1);
        }
        s2 = pick_bf16_pair(s_cur, b & 7);
      }
      const int s = idx % NS, a = idx % NA;
      if (!waitw(&full[s], (idx / NS) & 1, fail, lane, p.hint_ns) || !waitw(&a_empty[a], ((idx / NA) & 1) ^ 1, fail, lane, p.hint_ns))
        break;
      tc_fence_after();
      const uint8_t* w_src = stages + size_t(s) * STAGE + X_BYTES;
      const uint32_t col = A_COL + 64u * a + 16u * set;
      if (b < p.G) {
        const uint4 c = *reinterpret_cast<const uint4*>(w_src + r * 32 + 16 * set);
        const uint32_t s2n = s2 ^ 0x80008000u;
        uint32_t hi[16], nlo[16];
        codes_hi_lo(c.x, s2, s2n, hi + 0, nlo + 0);
        codes_hi_lo(c.y, s2, s2n, hi + 4, nlo + 4);
        codes_hi_lo(c.z, s2, s2n, hi + 8, nlo + 8);
        codes_hi_lo(c.w, s2, s2n, hi + 12, nlo + 12);
        tmem_st16(lane_base + col, hi);
        tmem_st16(lane_base + col + 32u, nlo);
      } else {
        uint32_t v[16];
        if (p.vec_sb) {
          const uint4* bsrc = reinterpret_cast<const uint4*>(w_src + r * 64);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 c = bsrc[i];
            v[4 * i + 0] = c.x;
            v[4 * i + 1] = c.y;
            v[4 * i + 2] = c.z;
            v[4 * i + 3] = c.w;
          }
        } else {
          const int g0 = 32 * (b - p.G);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t lo = (g0 + 2 * i < p.G) ? __bfloat16_as_ushort(brow16[g0 + 2 * i]) : 0u;
            const uint32_t hi = (g0 + 2 * i + 1 < p.G) ? __bfloat16_as_ushort(brow16[g0 + 2 * i + 1]) : 0u;
            v[i] = lo | (hi << 16);
          }
        }
        tmem_st16(lane_base + col, v);  // A = [b | b] against B = [xs_hi | xs_lo]
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[a]);
    }
  } else {
    // ------------------------------------------------------ promote + epilogue
    const int q = warp & 3, h = warp >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    const int units = (p.G + NG - 1) / NG + 1;
    float acc[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    int unit = 0;
    bool ok = true;
    GroupWait gw{1, 256, s_flags, 0};
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      for (int u = 0; u < units; ++u, ++unit) {
        const int pb = unit & 1;
        if (!(ok = gw.wait(&p_full[pb], (unit >> 1) & 1, fail, warp == 0, lane, p.hint_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          float v[16];
          tmem_ld16(lane_base + P_COL + 128u * pb + 64u * h + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c + j] += v[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_empty[pb]);
      }
      if (!ok) break;
      const int nt = t / p.m_tiles, mt = t % p.m_tiles;
      int si, row0, sg, grow;
      tile_rows(p, EPI, nt, si, row0);
      row_of<EPI>(p, si, row0, r, sg, grow);
      const int m0 = mt * BT + 64 * h;
      if (EPI == EPI_SWIGLU) {
        bf16* y = p.seg[0].y + grow;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float u = __shfl_down_sync(0xffffffffu, rbf(acc[j]), 16);  // up row of the same column
          const int m = m0 + j;
          if (!(r & 16) && m < p.M) {
            const float g = rbf(acc[j]);
            const float sgm = rbf(1.f / (1.f + expf(-g)));
            y[size_t(m) * p.ldy] = f2bf(rbf(g * sgm) * u);
          }
        }
      } else if (EPI == EPI_F32) {
        float* y = p.seg[sg].yf + grow;
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (m0 + j < p.M) y[size_t(m0 + j) * p.ldy] = acc[j];
      } else {
        bf16* y = p.seg[sg].y + grow;
#pragma unroll
        for (int j0 = 0; j0 < 64; j0 += 8) {
          float res[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            res[j] = (EPI == EPI_RESIDUAL && m0 + j0 + j < p.M) ? bf2f(y[size_t(m0 + j0 + j) * p.ldy]) : 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (m0 + j0 + j < p.M)
              y[size_t(m0 + j0 + j) * p.ldy] = (EPI == EPI_RESIDUAL) ? f2bf(res[j] + rbf(acc[j0 + j])) : f2bf(acc[j0 + j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// xs[m, 64c + t] = bf16 hi of sum_{k in group 32c+t} x[m, k]; xs[m, 64c + 32 + t] = lo.
__global__ void gemm_tc_xs_kernel(const bf16* __restrict__ x, int64_t ldx, int M, int G, int C, bf16* __restrict__ xs) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= M * C) return;
  const int m = wid / C, c = wid % C, g = 32 * c + lane;
  float sum = 0.f;
  if (g < G) {
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(m) * ldx + size_t(g) * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 v = src[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) sum += __uint_as_float(w[k] << 16) + __uint_as_float(w[k] & 0xFFFF0000u);
    }
  }
  const bf16 hi = f2bf(sum);
  const bf16 lo = f2bf(sum - bf2f(hi));
  bf16* dst = xs + size_t(m) * (64 * C) + 64 * c;
  dst[lane] = hi;
  dst[32 + lane] = lo;
}

}  // namespace gtc

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 gtc_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static int gtc_map(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
                   uint64_t stride_bytes, uint32_t box_in, uint32_t box_out, CUtensorMapSwizzle sw, const char* what) {
  auto enc = gtc_encode();
  if (!enc) return fail(M5_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_in, box_out}, es[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M5_ERR_CUDA, std::string("gemm_tc: tensor map encode failed (") + what + ")");
  return M5_OK;
}

size_t gemm_tc_xs_bytes(int M, int K) {
  const int G = K / 64, C = (G + 31) / 32;
  return size_t(M) * 64 * C * sizeof(bf16);
}

bool gemm_tc_eligible(const GemvArgs& a, int M, int epi) {
  if (M < 1 || a.K % 64 || a.norm_w || a.ldx % 8 || a.nseg < 1 || a.nseg > 3) return false;
  if (a.ldk && (a.ldk % 512 || a.ldk < a.K)) return false;  // slice rows stay 16-byte aligned
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.x)) return false;
  for (int i = 0; i < a.nseg; ++i) {
    if (!al(a.seg[i].w) || !al(a.seg[i].s) || !al(a.seg[i].b)) return false;
    if (a.seg[i].rows % (epi == EPI_SWIGLU ? 64 : 128)) return false;
  }
  if (epi == EPI_SWIGLU && (a.nseg != 2 || a.seg[0].rows != a.total_rows || a.seg[1].rows != a.total_rows))
    return false;
  return gtc_encode() != nullptr;
}

// M5_GEMM_TC_HINT_NS: suspend-time hint of the kernel's mbarrier waits (0 =
// poll; the default 1 ms measured 0.7 % faster than polling).
static uint32_t gtc_hint_ns() {
  static const uint32_t v = [] {
    const char* e = getenv("M5_GEMM_TC_HINT_NS");
    return e ? uint32_t(strtoul(e, nullptr, 10)) : 1000000u;
  }();
  return v;
}

template <int EPI>
static int gtc_launch_t(const gtc::Params& p_in, const gtc::Maps& m, cudaStream_t st) {
  gtc::Params p = p_in;
  p.hint_ns = gtc_hint_ns();
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(gtc::gemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)gtc::SMEM); }));
  const int tiles = p.n_tiles * p.m_tiles;
  const int grid = std::max(1, std::min(tiles, sm_count()));
  gtc::gemm_tc_kernel<EPI><<<grid, gtc::THREADS, gtc::SMEM, st>>>(p, m);
  M5_LAUNCH_CHECK("gemm_tc launch");
  return M5_OK;
}

int gemm_tc_launch(const GemvArgs& a, int M, int epi, bf16* xs, size_t xs_bytes, cudaStream_t st) {
  if (!gemm_tc_eligible(a, M, epi)) return fail(M5_ERR_INVALID, "gemm_tc: unsupported shape or alignment");
  if (xs_bytes < gemm_tc_xs_bytes(M, a.K) || (reinterpret_cast<uintptr_t>(xs) & 15))
    return fail(M5_ERR_INVALID, "gemm_tc: xs scratch too small or misaligned");
  gtc::Params p{};
  p.M = M;
  p.K = a.K;
  p.G = a.K / 64;
  p.C = (p.G + 31) / 32;
  const int64_t kst = a.ldk ? a.ldk : a.K;  // full row length of the weights (K slices)
  p.gld = (int)(kst / 64);
  p.vec_sb = (p.G % 8) == 0;
  p.nseg = a.nseg;
  p.ldy = a.ldy;
  int rows = 0;
  for (int i = 0; i < a.nseg; ++i) {
    p.seg[i].s = a.seg[i].s;
    p.bias[i] = a.seg[i].b;
    p.seg[i].rows = a.seg[i].rows;
    p.seg[i].y = a.seg[i].y;
    p.seg[i].yf = a.seg[i].yf;
    rows += a.seg[i].rows;
  }
  p.n_tiles = epi == EPI_SWIGLU ? a.total_rows / (gtc::BR / 2) : rows / gtc::BR;
  p.m_tiles = (M + gtc::BT - 1) / gtc::BT;
  gtc::Maps m;
  memset(&m, 0, sizeof(m));
  const int KB = 64 * p.C;
  int rc = gtc_map(&m.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.K, M, a.ldx * 2, 64, gtc::BT,
                   CU_TENSOR_MAP_SWIZZLE_128B, "x");
  if (!rc)
    rc = gtc_map(&m.xs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xs, KB, M, size_t(KB) * 2, 64, gtc::BT,
                 CU_TENSOR_MAP_SWIZZLE_128B, "xs");
  const uint32_t box_rows = epi == EPI_SWIGLU ? 16 : gtc::BR;
  for (int i = 0; i < a.nseg && !rc; ++i) {
    rc = gtc_map(&m.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, a.seg[i].w, a.K / 8, a.seg[i].rows, size_t(kst) / 2, 8,
                 box_rows, CU_TENSOR_MAP_SWIZZLE_NONE, "weights");
    if (!rc && p.vec_sb)
      rc = gtc_map(&m.b[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.seg[i].b, p.G, a.seg[i].rows, size_t(p.gld) * 2, 32,
                   box_rows, CU_TENSOR_MAP_SWIZZLE_NONE, "biases");
  }
  if (rc) return rc;
  {
    const int warps = M * p.C;
    const int threads = 256;
    const int blocks = (warps * 32 + threads - 1) / threads;
    gtc::gemm_tc_xs_kernel<<<blocks, threads, 0, st>>>(a.x, a.ldx, M, p.G, p.C, xs);
    M5_LAUNCH_CHECK("gemm_tc xs launch");
  }
  switch (epi) {
    case EPI_STORE: return gtc_launch_t<EPI_STORE>(p, m, st);
    case EPI_RESIDUAL: return gtc_launch_t<EPI_RESIDUAL>(p, m, st);
    case EPI_SWIGLU: return gtc_launch_t<EPI_SWIGLU>(p, m, st);
    case EPI_F32: return gtc_launch_t<EPI_F32>(p, m, st);
  }
  return fail(M5_ERR_INVALID, "gemm_tc: bad epilogue");
}

// y[m, n] = epi(sum over the S slices of part[s][m][n]), slices added in
// order, with the GEMM's own epilogues: EPI_STORE y = bf16(sum), EPI_RESIDUAL
// y += bf16(sum), EPI_F32 yf = sum.
__global__ void gemm_splitk_reduce_kernel(const float* __restrict__ part, int S, int M, int N, int epi, bf16* y,
                                          float* yf, int64_t ldy) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < S; ++s) v += part[size_t(s) * total + i];
    const int64_t m = i / N, n = i % N;
    if (epi == EPI_RESIDUAL) {
      bf16* o = y + m * ldy + n;
      *o = f2bf(bf2f(*o) + rbf(v));
    } else if (epi == EPI_STORE) {
      y[m * ldy + n] = f2bf(v);
    } else {
      yf[m * ldy + n] = v;
    }
  }
}

int gemm_splitk_reduce_launch(const float* part, int S, int M, int N, int epi, bf16* y, float* yf, int64_t ldy,
                              cudaStream_t st) {
  if (epi != EPI_RESIDUAL && epi != EPI_F32 && epi != EPI_STORE) return fail(M5_ERR_INVALID, "split-K reduce: epilogue");
  const int64_t total = int64_t(M) * N;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sm_count());
  gemm_splitk_reduce_kernel<<<blocks, 256, 0, st>>>(part, S, M, N, epi, y, yf, ldy);
  M5_LAUNCH_CHECK("split-K reduce launch");
  return M5_OK;
}

int gemm_tc_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_tc_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gemm_tc_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
