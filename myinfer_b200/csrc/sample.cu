// Token sampler over bf16 logits: the logits processors and the sampler that
// the reference builds for every request (m5engine/engine.py:384-392 calls
// mlx-lm 0.31.3 sample_utils.make_sampler / make_logits_processors), as one
// kernel with one 1024-thread CTA per logits row.
//
// Per row, in order:
//  1. Penalties on the distinct tokens of the row's history window, written
//     back into the logits in place, rounded to bf16 after each rule (mlx-lm
//     returns the processed bf16 logits): repetition v<0 ? v*r : v/r, then
//     presence v - p (once per distinct token), then frequency v - f*count.
//  2. The kept set.  top-p, min-p and top-k are all thresholds on the logit
//     value, so mlx-lm's order (top-p on the full distribution, min-p, then
//     top-k on what is left) keeps exactly the values at or above the largest
//     of three thresholds, each computed on the full row:
//       theta_p  smallest value whose strictly larger values hold less than
//                top_p of the probability mass,
//       theta_m  max + log(min_p),
//       theta_k  the k-th largest value (ties at it are all kept).
//     theta_p and theta_k come from a two-level radix select over the 16-bit
//     order-preserving key of the bf16 value (high byte, then low byte) with
//     per-warp histograms in shared memory: counts, and probability mass
//     exp(v - max) in 2^-40 fixed point, so every sum is exact and independent
//     of the order the atomics land in.  One atomic-free pass first counts the
//     entries and mass within 1, 2, 4, 8 and 16 of the max; when the narrowest
//     band that contains both crossings holds at most 8192 entries (a peaked
//     row) those are compacted into shared memory and the select runs there,
//     otherwise (a flat row) it runs over the whole row.
//  3. An inverse-CDF draw at the temperature: u = SplitMix64(seed, counter)
//     in [0, 1), target u * sum over the kept set of exp((v - max) / T),
//     found in index order tile by tile (one pass for the tile sums, then one
//     tile re-read and scanned).
// Temperature <= 0 is greedy: the first index of the largest (penalised)
// value.  The row is read from L2 once per pass (a 151936-entry row is 297 KB),
// each thread keeping four 16-byte loads in flight.
//
// Row r uses counter offset + state[0] + r.  With a device state the last CTA
// to finish adds the row count to state[0] (CTAs count themselves in
// state[1]), and with the append flag each row's history window rolls left
// by one and takes the drawn token: a decode loop replayed from a CUDA graph
// then draws fresh numbers and sees its own tokens every step.
#include <climits>

#include "common.cuh"

namespace m5 {
namespace {

constexpr int kSmpThreads = 1024;
constexpr int kSmpWarps = kSmpThreads / 32;
constexpr int kSmpPer = 8;                         // consecutive entries per thread per tile (one 16-byte load)
constexpr int kSmpTile = kSmpThreads * kSmpPer;    // 8192 entries
constexpr int kSmpMaxTiles = 64;
constexpr int kSmpMaxHist = 1024;
constexpr float kSmpMassScale = 1099511627776.f;   // 2^40
constexpr int kSmpAhead = 4;                       // tiles whose loads a thread keeps in flight
constexpr int kSmpCap = 8192;                      // candidate entries compacted into shared memory
constexpr int kSmpLevels = 5;                      // candidate bands: within 1, 2, 4, 8, 16 of the max
constexpr size_t kSmpSmem = size_t(kSmpWarps) * 256 * (sizeof(uint32_t) + sizeof(unsigned long long)) +
                            size_t(kSmpCap) * sizeof(unsigned short);

__device__ __forceinline__ float smp_band(int i) { return (float)(1 << i); }

struct SampleArgs {
  bf16* logits;
  int64_t ld;
  int vocab;
  const int32_t* hist;
  int hist_len;
  int64_t hist_ld;
  float temp, top_p, min_p;
  int top_k;
  float rep, pres, freq;
  unsigned long long seed, offset;
  int32_t* out;
  unsigned long long* state;  // optional {counter, CTAs done}: base counter and its advance on the device
  int append;                 // roll each history row left and append the drawn token
  int vec;                    // row base and stride allow 16-byte loads
};

// Order-preserving 16-bit key of a bf16 bit pattern (larger value, larger key).
__device__ __forceinline__ uint32_t smp_key(uint32_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }
__device__ __forceinline__ float smp_val(uint32_t b) { return __uint_as_float(b << 16); }

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) of counter `ctr` under `seed`; top 24 bits as a
// float in [0, 1).
__device__ __forceinline__ float smp_uniform(unsigned long long seed, unsigned long long ctr) {
  unsigned long long z = seed + (ctr + 1ull) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.f / 16777216.f);
}

// One thread's 8 consecutive entries of a tile as raw bf16 bits (entry j in
// half j & 1 of word j >> 1); returns how many lie inside the row.  Plain
// loads: the penalties may have just rewritten them.
__device__ __forceinline__ int smp_load(const bf16* row, int vocab, int i0, int vec, uint4& u) {
  u = make_uint4(0u, 0u, 0u, 0u);
  if (i0 >= vocab) return 0;
  if (vec && i0 + kSmpPer <= vocab) {
    u = *reinterpret_cast<const uint4*>(row + i0);
    return kSmpPer;
  }
  const unsigned short* r = reinterpret_cast<const unsigned short*>(row);
  const int n = min(kSmpPer, vocab - i0);
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < kSmpPer; ++j)
    if (j < n) w[j >> 1] |= (uint32_t)r[i0 + j] << (16 * (j & 1));
  u = make_uint4(w[0], w[1], w[2], w[3]);
  return n;
}
__device__ __forceinline__ uint32_t smp_bits(const uint4& u, int j) {
  const uint32_t w = j < 2 ? u.x : j < 4 ? u.y : j < 6 ? u.z : u.w;
  return (j & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Calls f(i0, n, u) for this thread's slot of every tile, with the loads of
// kSmpAhead tiles issued before the first of them is used.
template <class F>
__device__ __forceinline__ void smp_tiles(const bf16* row, int vocab, int vec, int ntile, F&& f) {
  const int off = threadIdx.x * kSmpPer;
  for (int t0 = 0; t0 < ntile; t0 += kSmpAhead) {
    uint4 u[kSmpAhead];
    int n[kSmpAhead];
#pragma unroll
    for (int q = 0; q < kSmpAhead; ++q) n[q] = smp_load(row, vocab, (t0 + q) * kSmpTile + off, vec, u[q]);
#pragma unroll
    for (int q = 0; q < kSmpAhead; ++q) f(t0 + q, (t0 + q) * kSmpTile + off, n[q], u[q]);
  }
}

// Block-wide max / min with a fixed combination order (every thread gets
// the same bits back).
__device__ float smp_block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kSmpWarps; ++w) r = fmaxf(r, red[w]);
  return r;
}
__device__ int smp_block_min(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = red[0];
  for (int w = 1; w < kSmpWarps; ++w) r = min(r, red[w]);
  return r;
}

// One full warp: the first bin, scanning 255 down to 0, at which the running
// sum reaches `target` (>= 1), or -1 when the total stays below it; *before
// receives the sum of the bins above that bin.
template <typename T>
__device__ int smp_cross(const T* bins, unsigned long long target, unsigned long long* before) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = (unsigned long long)bins[255 - 8 * lane - j];
    s += v[j];
  }
  unsigned long long incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const unsigned long long excl = incl - s;
  const unsigned m = __ballot_sync(0xffffffffu, excl < target && incl >= target);
  if (!m) {
    *before = 0;
    return -1;
  }
  const int src = __ffs(m) - 1;
  int bin = -1;
  unsigned long long bef = 0;
  if (lane == src) {
    unsigned long long c = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (bin < 0 && c + v[j] >= target) {
        bin = 255 - 8 * lane - j;
        bef = c;
      }
      c += v[j];
    }
  }
  bin = __shfl_sync(0xffffffffu, bin, src);
  bef = __shfl_sync(0xffffffffu, bef, src);
  *before = bef;
  return bin;
}

__device__ __forceinline__ unsigned long long smp_fixed_mass(float v, float vmax) {
  return __float2ull_rn(expf(v - vmax) * kSmpMassScale);
}

// Shared scratch of one row's selection.
struct SmpShared {
  uint32_t* wcnt;              // [warps][256] per-warp counts
  unsigned long long* wmass;   // [warps][256] per-warp fixed-point mass
  uint32_t* cnt1;              // [256] merged counts
  unsigned long long* mass1;   // [256] merged mass
  int* s_int;
  unsigned long long* s_u;
};

// Exact 16-bit key thresholds of top-k (k entries) and top-p (fixed-point
// mass P) over the entries visit() yields to each thread: a round of per-warp
// 256-bin histograms over the high key byte, the crossing bins, then a round
// over the low byte of the entries inside them.  Returns the larger key (0
// when the filters keep everything).  Counts and masses are integers, so the
// result does not depend on the order the atomics land in.
template <class Visit>
__device__ uint32_t smp_select(Visit&& visit, bool do_k, bool do_p, unsigned long long k, unsigned long long P,
                               float vmax, const SmpShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* my_cnt = sh.wcnt + warp * 256;
  unsigned long long* my_mass = sh.wmass + warp * 256;
  for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) {
    sh.wcnt[i] = 0u;
    sh.wmass[i] = 0ull;
  }
  __syncthreads();
  {  // round 1: high byte, equal consecutive bins of a thread merged before the atomic
    uint32_t ccur = 0xFFFFFFFFu, crun = 0, mcur = 0xFFFFFFFFu;
    unsigned long long mrun = 0;
    visit([&](uint32_t bits) {
      const uint32_t bin = smp_key(bits) >> 8;
      if (do_k) {
        if (bin != ccur) {
          if (crun) atomicAdd(my_cnt + ccur, crun);
          ccur = bin;
          crun = 0;
        }
        ++crun;
      }
      if (do_p) {
        if (bin != mcur) {
          if (mrun) atomicAdd(my_mass + mcur, mrun);
          mcur = bin;
          mrun = 0;
        }
        mrun += smp_fixed_mass(smp_val(bits), vmax);
      }
    });
    if (crun) atomicAdd(my_cnt + ccur, crun);
    if (mrun) atomicAdd(my_mass + mcur, mrun);
  }
  __syncthreads();
  if (tid < 256) {
    uint32_t c = 0;
    unsigned long long m = 0;
    for (int w = 0; w < kSmpWarps; ++w) {
      c += sh.wcnt[w * 256 + tid];
      m += sh.wmass[w * 256 + tid];
    }
    sh.cnt1[tid] = c;
    sh.mass1[tid] = m;
  }
  __syncthreads();
  if (warp == 0) {
    unsigned long long bk_bef = 0, bp_bef = 0;
    const int bk = do_k ? smp_cross(sh.cnt1, k, &bk_bef) : -1;
    const int bp = do_p ? smp_cross(sh.mass1, P, &bp_bef) : -1;
    if (lane == 0) {
      sh.s_int[0] = bk;
      sh.s_int[1] = bp;
      sh.s_u[0] = bk_bef;
      sh.s_u[1] = bp_bef;
    }
  }
  __syncthreads();
  const int bk = sh.s_int[0], bp = sh.s_int[1];
  const unsigned long long bk_bef = sh.s_u[0], bp_bef = sh.s_u[1];
  if (bk < 0 && bp < 0) return 0u;
  for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) {
    sh.wcnt[i] = 0u;
    sh.wmass[i] = 0ull;
  }
  __syncthreads();
  visit([&](uint32_t bits) {  // round 2: low byte inside the crossing bins
    const uint32_t key = smp_key(bits);
    const int hb = (int)(key >> 8);
    if (hb == bk) atomicAdd(my_cnt + (key & 255u), 1u);
    if (hb == bp) atomicAdd(my_mass + (key & 255u), smp_fixed_mass(smp_val(bits), vmax));
  });
  __syncthreads();
  if (tid < 256) {
    uint32_t c = 0;
    unsigned long long m = 0;
    for (int w = 0; w < kSmpWarps; ++w) {
      c += sh.wcnt[w * 256 + tid];
      m += sh.wmass[w * 256 + tid];
    }
    sh.cnt1[tid] = c;
    sh.mass1[tid] = m;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t kk = 0, kp = 0;
    unsigned long long unused;
    if (bk >= 0) kk = ((uint32_t)bk << 8) | (uint32_t)max(smp_cross(sh.cnt1, k - bk_bef, &unused), 0);
    if (bp >= 0) kp = ((uint32_t)bp << 8) | (uint32_t)max(smp_cross(sh.mass1, P - bp_bef, &unused), 0);
    if (lane == 0) sh.s_int[2] = (int)max(kk, kp);
  }
  __syncthreads();
  return (uint32_t)sh.s_int[2];
}

// Draws the token of one row into *pick_out (left untouched when nothing has weight).
__device__ __forceinline__ void sample_row(const SampleArgs& a, int row, unsigned long long base, int* pick_out) {
  extern __shared__ __align__(16) unsigned char smp_smem[];
  uint32_t* wcnt = reinterpret_cast<uint32_t*>(smp_smem);  // [warps][256] counts
  unsigned long long* wmass =
      reinterpret_cast<unsigned long long*>(smp_smem + size_t(kSmpWarps) * 256 * sizeof(uint32_t));  // [warps][256]
  unsigned short* cand = reinterpret_cast<unsigned short*>(wmass + kSmpWarps * 256);  // [kSmpCap] raw bits
  __shared__ float red[kSmpWarps];
  __shared__ float red4[kSmpAhead][kSmpWarps];
  __shared__ int red_i[kSmpWarps];
  __shared__ uint32_t cnt1[256];
  __shared__ unsigned long long mass1[256];
  __shared__ unsigned long long lvl_part[kSmpWarps][2 * kSmpLevels + 1];
  __shared__ unsigned long long lvl[2 * kSmpLevels + 1];
  __shared__ float tile_sum[kSmpMaxTiles];
  __shared__ int s_int[5];
  __shared__ unsigned long long s_u[4];
  __shared__ float s_f[1];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bf16* lg = a.logits + (int64_t)row * a.ld;
  const int V = a.vocab;
  const int ntile = (V + kSmpTile - 1) / kSmpTile;

  // ---- 1. penalties on the history window
  const bool rep_on = a.rep != 1.f, pres_on = a.pres != 0.f, freq_on = a.freq != 0.f;
  if ((rep_on || pres_on || freq_on) && a.hist_len > 0) {
    int* h = reinterpret_cast<int*>(wcnt);
    const int32_t* hg = a.hist + (int64_t)row * a.hist_ld;
    for (int j = tid; j < a.hist_len; j += kSmpThreads) h[j] = hg[j];
    __syncthreads();
    for (int j = tid; j < a.hist_len; j += kSmpThreads) {
      const int t = h[j];
      if (t < 0 || t >= V) continue;
      int cnt = 0;
      bool first = true;
      for (int q = 0; q < a.hist_len; ++q) {
        if (h[q] == t) {
          ++cnt;
          if (q < j) first = false;
        }
      }
      if (!first) continue;
      float v = bf2f(lg[t]);
      if (rep_on) v = rbf(v < 0.f ? v * a.rep : v / a.rep);
      if (pres_on) v = rbf(v - a.pres);
      if (freq_on) v = rbf(v - a.freq * (float)cnt);
      lg[t] = f2bf(v);
    }
    __syncthreads();
  }

  const bool greedy = !(a.temp > 0.f);
  const bool do_k = !greedy && a.top_k > 0 && a.top_k < V;
  const bool do_p = !greedy && a.top_p > 0.f && a.top_p < 1.f;

  // ---- 2a. max
  float vmax = -INFINITY;
  smp_tiles(lg, V, a.vec, ntile, [&](int, int, int n, const uint4& u) {
#pragma unroll
    for (int j = 0; j < kSmpPer; ++j)
      if (j < n) vmax = fmaxf(vmax, smp_val(smp_bits(u, j)));
  });
  vmax = smp_block_max(vmax, red);

  if (greedy) {  // first index of the max
    int best = INT_MAX;
    smp_tiles(lg, V, a.vec, ntile, [&](int, int i0, int n, const uint4& u) {
#pragma unroll
      for (int j = 0; j < kSmpPer; ++j)  // tiles and entries in index order: the first hit is the lowest
        if (j < n && best == INT_MAX && smp_val(smp_bits(u, j)) == vmax) best = i0 + j;
    });
    best = smp_block_min(best, red_i);
    if (tid == 0 && best != INT_MAX) *pick_out = best;
    return;
  }
  // reference point of the exponentials (a row of -inf keeps every weight 0 and draws index 0)
  if (vmax == -INFINITY) vmax = 0.f;

  // ---- 2b. thresholds of top-k / top-p
  uint32_t key_th = 0;
  if (do_k || do_p) {
    // Bands [max - 2^i, max]: entries and fixed-point mass in each, and the
    // row's total mass, in one pass without atomics.
    uint32_t lc[kSmpLevels];
    unsigned long long lm[kSmpLevels], ztot = 0;
#pragma unroll
    for (int i = 0; i < kSmpLevels; ++i) {
      lc[i] = 0u;
      lm[i] = 0ull;
    }
    smp_tiles(lg, V, a.vec, ntile, [&](int, int, int n, const uint4& u) {
#pragma unroll
      for (int j = 0; j < kSmpPer; ++j) {
        if (j < n) {
          const float v = smp_val(smp_bits(u, j));
          const unsigned long long w = smp_fixed_mass(v, vmax);
          ztot += w;
#pragma unroll
          for (int i = 0; i < kSmpLevels; ++i)
            if (v >= vmax - smp_band(i)) {
              ++lc[i];
              lm[i] += w;
            }
        }
      }
    });
#pragma unroll
    for (int i = 0; i < 2 * kSmpLevels + 1; ++i) {
      unsigned long long x = i < kSmpLevels ? (unsigned long long)lc[i] : i < 2 * kSmpLevels ? lm[i - kSmpLevels] : ztot;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) lvl_part[warp][i] = x;
    }
    __syncthreads();
    if (tid < 2 * kSmpLevels + 1) {
      unsigned long long x = 0;
      for (int w = 0; w < kSmpWarps; ++w) x += lvl_part[w][tid];
      lvl[tid] = x;
    }
    __syncthreads();
    // keep a value while the mass strictly above it is below top_p * total
    unsigned long long P = 0;
    if (do_p) {
      P = (unsigned long long)ceil((double)a.top_p * (double)lvl[2 * kSmpLevels]);
      if (P < 1ull) P = 1ull;
    }
    const unsigned long long K = do_k ? (unsigned long long)a.top_k : 0ull;
    // the narrowest band that holds both crossings, if it fits the candidate store
    int band = -1;
    for (int i = 0; i < kSmpLevels; ++i) {
      if ((!do_k || lvl[i] >= K) && (!do_p || lvl[kSmpLevels + i] >= P)) {
        band = i;
        break;
      }
    }
    if (band >= 0 && lvl[band] > (unsigned long long)kSmpCap) band = -1;
    SmpShared sh{wcnt, wmass, cnt1, mass1, s_int, s_u};
    if (band >= 0) {
      if (tid == 0) s_int[4] = 0;
      __syncthreads();
      const float thr = vmax - smp_band(band);
      smp_tiles(lg, V, a.vec, ntile, [&](int, int, int n, const uint4& u) {
#pragma unroll
        for (int j = 0; j < kSmpPer; ++j) {
          const uint32_t bits = smp_bits(u, j);
          const bool take = j < n && smp_val(bits) >= thr;
          const unsigned m = __ballot_sync(0xffffffffu, take);
          if (m) {
            const int leader = __ffs(m) - 1;
            int pos = 0;
            if (lane == leader) pos = atomicAdd(&s_int[4], __popc(m));
            pos = __shfl_sync(0xffffffffu, pos, leader) + __popc(m & ((1u << lane) - 1u));
            if (take && pos < kSmpCap) cand[pos] = (unsigned short)bits;
          }
        }
      });
      __syncthreads();
      const int ncand = min(s_int[4], kSmpCap);
      key_th = smp_select(
          [&](auto&& g) {
            for (int i = tid; i < ncand; i += kSmpThreads) g((uint32_t)cand[i]);
          },
          do_k, do_p, K, P, vmax, sh);
    } else {  // flat rows: the crossing lies deep in the bulk, select over the whole row
      key_th = smp_select(
          [&](auto&& g) {
            smp_tiles(lg, V, a.vec, ntile, [&](int, int, int n, const uint4& u) {
#pragma unroll
              for (int j = 0; j < kSmpPer; ++j)
                if (j < n) g(smp_bits(u, j));
            });
          },
          do_k, do_p, K, P, vmax, sh);
    }
  }
  const float thr_m = a.min_p > 0.f ? vmax + logf(a.min_p) : -INFINITY;
  const float inv_t = 1.f / a.temp;

  // ---- 3. inverse-CDF draw over the kept set at the temperature
  for (int t0 = 0; t0 < ntile; t0 += kSmpAhead) {
    uint4 u[kSmpAhead];
    int n[kSmpAhead];
#pragma unroll
    for (int q = 0; q < kSmpAhead; ++q) n[q] = smp_load(lg, V, (t0 + q) * kSmpTile + tid * kSmpPer, a.vec, u[q]);
#pragma unroll
    for (int q = 0; q < kSmpAhead; ++q) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kSmpPer; ++j) {
        const uint32_t bits = smp_bits(u[q], j);
        const float v = smp_val(bits);
        if (j < n[q] && smp_key(bits) >= key_th && v >= thr_m) s += expf((v - vmax) * inv_t);
      }
      s = warp_sum(s);
      if (lane == 0) red4[q][warp] = s;
    }
    __syncthreads();
    if (tid < kSmpAhead && t0 + tid < ntile) {
      float s = 0.f;
      for (int w = 0; w < kSmpWarps; ++w) s += red4[tid][w];
      tile_sum[t0 + tid] = s;
    }
    __syncthreads();
  }
  if (tid == 0) {
    float z = 0.f;
    for (int t = 0; t < ntile; ++t) z += tile_sum[t];
    float target = smp_uniform(a.seed, base + (unsigned long long)row) * z;
    if (!(target < z)) target = nextafterf(z, 0.f);
    float cum = 0.f;
    int ti = -1, last = 0;
    float cum_last = 0.f;
    for (int t = 0; t < ntile; ++t) {
      if (tile_sum[t] > 0.f) {
        if (cum + tile_sum[t] > target) {
          ti = t;
          break;
        }
        last = t;
        cum_last = cum;
        cum += tile_sum[t];
      }
    }
    if (ti < 0) {  // rounding left the target past the last tile
      ti = last;
      cum = cum_last;
    }
    s_int[3] = ti;
    s_f[0] = fmaxf(target - cum, 0.f);
  }
  __syncthreads();
  const int ti = s_int[3];
  float rem = s_f[0];
  uint4 u;
  const int i0 = ti * kSmpTile + tid * kSmpPer;
  const int n = smp_load(lg, V, i0, a.vec, u);
  float w[kSmpPer];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kSmpPer; ++j) {
    const uint32_t bits = smp_bits(u, j);
    const float v = smp_val(bits);
    w[j] = (j < n && smp_key(bits) >= key_th && v >= thr_m) ? expf((v - vmax) * inv_t) : 0.f;
    s += w[j];
  }
  // block-wide scan: the exclusive prefix of thread i is bit-identical to the
  // inclusive prefix of thread i - 1, so exactly one thread holds the target
  float wincl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, wincl, o);
    if (lane >= o) wincl += y;
  }
  float wexcl = __shfl_up_sync(0xffffffffu, wincl, 1);
  if (lane == 0) wexcl = 0.f;
  if (lane == 31) red[warp] = wincl;
  __syncthreads();
  float woff = 0.f;
  for (int q = 0; q < warp; ++q) woff += red[q];
  float tot = 0.f;
  for (int q = 0; q < kSmpWarps; ++q) tot += red[q];
  if (!(rem < tot)) rem = nextafterf(tot, 0.f);
  const float excl = woff + wexcl, incl = woff + wincl;
  if (s > 0.f && excl <= rem && rem < incl) {
    float c = excl;
    int pick = -1, lastj = -1;
#pragma unroll
    for (int j = 0; j < kSmpPer; ++j) {
      if (w[j] > 0.f) {
        lastj = j;
        if (pick < 0 && rem < c + w[j]) pick = j;
        c += w[j];
      }
    }
    if (pick < 0) pick = lastj;
    *pick_out = i0 + pick;
  }
}

__global__ void __launch_bounds__(kSmpThreads, 1) sample_rows_kernel(SampleArgs a) {
  __shared__ int s_pick;
  __shared__ unsigned long long s_base;
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  int32_t* hg = a.hist ? const_cast<int32_t*>(a.hist) + (int64_t)row * a.hist_ld : nullptr;
  // the entry each thread moves one place left when the window rolls
  const int hnext = (a.append && hg && tid + 1 < a.hist_len) ? hg[tid + 1] : 0;
  if (tid == 0) {
    s_pick = 0;
    s_base = a.offset + (a.state ? a.state[0] : 0ull);
  }
  __syncthreads();
  sample_row(a, row, s_base, &s_pick);
  __syncthreads();
  if (tid == 0) a.out[row] = s_pick;
  if (a.append && hg && a.hist_len > 0) {
    if (tid + 1 < a.hist_len) hg[tid] = hnext;
    if (tid == a.hist_len - 1) hg[tid] = s_pick;
  }
  if (a.state && tid == 0) {  // the last CTA to finish advances the counter for the next call
    __threadfence();
    const unsigned long long done = atomicAdd(a.state + 1, 1ull);
    if (done == (unsigned long long)gridDim.x - 1ull) {
      a.state[0] += (unsigned long long)gridDim.x;
      a.state[1] = 0ull;
      __threadfence();
    }
  }
}

}  // namespace
}  // namespace m5

extern "C" int m5_sample_bf16(void* logits, int rows, int64_t vocab, int64_t ld, int32_t* history, int hist_len,
                              int64_t hist_ld, const m5_sample_params* p, uint64_t* state, int32_t* out,
                              void* stream) {
  using namespace m5;
  M5_CHECK_ARG(logits && out && p, "m5_sample_bf16: null pointer");
  M5_CHECK_ARG(rows > 0 && rows <= (1 << 20), "m5_sample_bf16: rows must be in [1, 2^20]");
  M5_CHECK_ARG(vocab > 0 && vocab <= int64_t(kSmpTile) * kSmpMaxTiles, "m5_sample_bf16: vocab must be in [1, 524288]");
  M5_CHECK_ARG(ld >= vocab, "m5_sample_bf16: row stride below vocab");
  M5_CHECK_ARG(hist_len >= 0 && hist_len <= kSmpMaxHist, "m5_sample_bf16: history window must be in [0, 1024]");
  M5_CHECK_ARG(hist_len == 0 || (history && hist_ld >= hist_len), "m5_sample_bf16: history pointer / stride");
  M5_CHECK_ARG(p->temperature == p->temperature && p->temperature < INFINITY, "m5_sample_bf16: temperature");
  M5_CHECK_ARG(p->top_p == p->top_p && p->min_p == p->min_p, "m5_sample_bf16: top_p / min_p must not be NaN");
  M5_CHECK_ARG(p->min_p <= 1.f, "m5_sample_bf16: min_p must be <= 1");
  M5_CHECK_ARG(!(p->repetition_penalty < 0.f), "m5_sample_bf16: repetition_penalty must be >= 0");
  M5_CHECK_ARG((p->flags & ~M5_SAMPLE_APPEND_HISTORY) == 0, "m5_sample_bf16: unknown flags");
  M5_CHECK_ARG(!(p->flags & M5_SAMPLE_APPEND_HISTORY) || hist_len > 0, "m5_sample_bf16: append needs a history");
  SampleArgs a;
  a.logits = static_cast<bf16*>(logits);
  a.ld = ld;
  a.vocab = (int)vocab;
  a.hist = history;
  a.hist_len = hist_len;
  a.hist_ld = hist_ld;
  a.temp = p->temperature;
  a.top_p = p->top_p;
  a.min_p = p->min_p;
  a.top_k = p->top_k;
  // a zero or NaN repetition penalty is "off" (mlx-lm builds no processor for it)
  a.rep = p->repetition_penalty > 0.f ? p->repetition_penalty : 1.f;
  a.pres = p->presence_penalty == p->presence_penalty ? p->presence_penalty : 0.f;
  a.freq = p->frequency_penalty == p->frequency_penalty ? p->frequency_penalty : 0.f;
  a.seed = p->seed;
  a.offset = p->offset;
  a.out = out;
  a.state = reinterpret_cast<unsigned long long*>(state);
  a.append = (p->flags & M5_SAMPLE_APPEND_HISTORY) ? 1 : 0;
  a.vec = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && (ld % 8 == 0);
  static DeviceOnce once;  // once per device, normally before any graph capture
  M5_CUDA(once.run(
      [&] { return cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmpSmem); }));
  sample_rows_kernel<<<rows, kSmpThreads, kSmpSmem, static_cast<cudaStream_t>(stream)>>>(a);
  M5_LAUNCH_CHECK("sample_rows_kernel");
  return M5_OK;
}
