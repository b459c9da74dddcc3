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
//     of the order the atomics land in.
//  3. An inverse-CDF draw at the temperature: u = SplitMix64(seed, counter)
//     in [0, 1), target u * sum over the kept set of exp((v - max) / T),
//     found in index order tile by tile (one pass for the tile sums, then one
//     tile re-read and scanned).
// Temperature <= 0 is greedy: the first index of the largest (penalised)
// value.  The row is read from L2 once per pass (a 151936-entry row is 297 KB).
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
constexpr size_t kSmpSmem = size_t(kSmpWarps) * 256 * (sizeof(uint32_t) + sizeof(unsigned long long));

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

// The raw bf16 bits of one thread's 8 entries of a tile; returns how many lie
// inside the row.  Plain loads: the penalties may have just rewritten them.
__device__ __forceinline__ int smp_load8(const bf16* row, int vocab, int i0, int vec, uint32_t (&b)[kSmpPer]) {
  if (i0 >= vocab) return 0;
  if (vec && i0 + kSmpPer <= vocab) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + i0);
    b[0] = u.x & 0xFFFFu; b[1] = u.x >> 16; b[2] = u.y & 0xFFFFu; b[3] = u.y >> 16;
    b[4] = u.z & 0xFFFFu; b[5] = u.z >> 16; b[6] = u.w & 0xFFFFu; b[7] = u.w >> 16;
    return kSmpPer;
  }
  const unsigned short* r = reinterpret_cast<const unsigned short*>(row);
  const int n = min(kSmpPer, vocab - i0);
#pragma unroll
  for (int j = 0; j < kSmpPer; ++j) b[j] = j < n ? (uint32_t)r[i0 + j] : 0u;
  return n;
}

// Block-wide max / sum / min with a fixed combination order (every thread gets
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
__device__ float smp_block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < kSmpWarps; ++w) r += red[w];
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

// Draws the token of one row into *pick_out (left untouched when nothing has weight).
__device__ __forceinline__ void sample_row(const SampleArgs& a, int row, unsigned long long base, int* pick_out) {
  extern __shared__ __align__(16) unsigned char smp_smem[];
  uint32_t* wcnt = reinterpret_cast<uint32_t*>(smp_smem);  // [warps][256] counts
  unsigned long long* wmass =
      reinterpret_cast<unsigned long long*>(smp_smem + size_t(kSmpWarps) * 256 * sizeof(uint32_t));  // [warps][256]
  __shared__ float red[kSmpWarps];
  __shared__ int red_i[kSmpWarps];
  __shared__ uint32_t cnt1[256];
  __shared__ unsigned long long mass1[256];
  __shared__ float tile_sum[kSmpMaxTiles];
  __shared__ int s_int[4];
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

  // ---- 2a. max (+ level-1 counts for top-k)
  if (do_k) {
    for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) wcnt[i] = 0u;
    __syncthreads();
  }
  uint32_t* my_cnt = wcnt + warp * 256;
  unsigned long long* my_mass = wmass + warp * 256;
  float vmax = -INFINITY;
  for (int t = 0; t < ntile; ++t) {
    uint32_t b[kSmpPer];
    const int i0 = t * kSmpTile + tid * kSmpPer;
    const int n = smp_load8(lg, V, i0, a.vec, b);
    uint32_t cur = 0xFFFFFFFFu, run = 0;
#pragma unroll
    for (int j = 0; j < kSmpPer; ++j) {
      if (j < n) {
        vmax = fmaxf(vmax, smp_val(b[j]));
        if (do_k) {
          const uint32_t bin = smp_key(b[j]) >> 8;
          if (bin != cur) {
            if (run) atomicAdd(my_cnt + cur, run);
            cur = bin;
            run = 0;
          }
          ++run;
        }
      }
    }
    if (do_k && run) atomicAdd(my_cnt + cur, run);
  }
  vmax = smp_block_max(vmax, red);

  if (greedy) {  // first index of the max
    int best = INT_MAX;
    for (int t = 0; t < ntile; ++t) {
      uint32_t b[kSmpPer];
      const int i0 = t * kSmpTile + tid * kSmpPer;
      const int n = smp_load8(lg, V, i0, a.vec, b);
#pragma unroll
      for (int j = kSmpPer - 1; j >= 0; --j)
        if (j < n && smp_val(b[j]) == vmax) best = i0 + j;
      if (best != INT_MAX) break;
    }
    best = smp_block_min(best, red_i);
    if (tid == 0 && best != INT_MAX) *pick_out = best;
    return;
  }
  // reference point of the exponentials (a row of -inf keeps every weight 0 and draws index 0)
  if (vmax == -INFINITY) vmax = 0.f;

  // ---- 2b. level-1 crossing for top-k
  int bk = -1, bp = -1;
  unsigned long long bef_k = 0, bef_p = 0, ptarget = 0;
  if (do_k) {
    if (tid < 256) {
      uint32_t s = 0;
      for (int w = 0; w < kSmpWarps; ++w) s += wcnt[w * 256 + tid];
      cnt1[tid] = s;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned long long bef;
      const int bin = smp_cross(cnt1, (unsigned long long)a.top_k, &bef);
      if (lane == 0) {
        s_int[0] = bin;
        s_u[0] = bef;
      }
    }
    __syncthreads();
    bk = s_int[0];
    bef_k = s_u[0];
  }

  // ---- 2c. level-1 mass and crossing for top-p
  if (do_p) {
    for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) wmass[i] = 0ull;
    __syncthreads();
    for (int t = 0; t < ntile; ++t) {
      uint32_t b[kSmpPer];
      const int i0 = t * kSmpTile + tid * kSmpPer;
      const int n = smp_load8(lg, V, i0, a.vec, b);
      uint32_t cur = 0xFFFFFFFFu;
      unsigned long long run = 0;
#pragma unroll
      for (int j = 0; j < kSmpPer; ++j) {
        if (j < n) {
          const uint32_t bin = smp_key(b[j]) >> 8;
          if (bin != cur) {
            if (run) atomicAdd(my_mass + cur, run);
            cur = bin;
            run = 0;
          }
          run += smp_fixed_mass(smp_val(b[j]), vmax);
        }
      }
      if (run) atomicAdd(my_mass + cur, run);
    }
    __syncthreads();
    if (tid < 256) {
      unsigned long long s = 0;
      for (int w = 0; w < kSmpWarps; ++w) s += wmass[w * 256 + tid];
      mass1[tid] = s;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned long long tot = 0;
      for (int j = lane; j < 256; j += 32) tot += mass1[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
      // keep a value while the mass strictly above it is below top_p * total
      unsigned long long P = (unsigned long long)ceil((double)a.top_p * (double)tot);
      if (P < 1ull) P = 1ull;
      unsigned long long bef;
      const int bin = smp_cross(mass1, P, &bef);
      if (lane == 0) {
        s_int[1] = bin;
        s_u[1] = bef;
        s_u[2] = P;
      }
    }
    __syncthreads();
    bp = s_int[1];
    bef_p = s_u[1];
    ptarget = s_u[2];
  }

  // ---- 2d. level 2 inside the crossing bins: exact 16-bit keys
  uint32_t key_th = 0;
  if (bk >= 0 || bp >= 0) {
    for (int i = tid; i < kSmpWarps * 256; i += kSmpThreads) {
      wcnt[i] = 0u;
      wmass[i] = 0ull;
    }
    __syncthreads();
    for (int t = 0; t < ntile; ++t) {
      uint32_t b[kSmpPer];
      const int i0 = t * kSmpTile + tid * kSmpPer;
      const int n = smp_load8(lg, V, i0, a.vec, b);
#pragma unroll
      for (int j = 0; j < kSmpPer; ++j) {
        if (j < n) {
          const uint32_t key = smp_key(b[j]);
          const int hb = (int)(key >> 8);
          if (hb == bk) atomicAdd(my_cnt + (key & 255u), 1u);
          if (hb == bp) atomicAdd(my_mass + (key & 255u), smp_fixed_mass(smp_val(b[j]), vmax));
        }
      }
    }
    __syncthreads();
    if (tid < 256) {
      uint32_t c = 0;
      unsigned long long m = 0;
      for (int w = 0; w < kSmpWarps; ++w) {
        c += wcnt[w * 256 + tid];
        m += wmass[w * 256 + tid];
      }
      cnt1[tid] = c;
      mass1[tid] = m;
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t kk = 0, kp = 0;
      unsigned long long unused;
      if (bk >= 0) {
        const int low = smp_cross(cnt1, (unsigned long long)a.top_k - bef_k, &unused);
        kk = ((uint32_t)bk << 8) | (uint32_t)max(low, 0);
      }
      if (bp >= 0) {
        const int low = smp_cross(mass1, ptarget - bef_p, &unused);
        kp = ((uint32_t)bp << 8) | (uint32_t)max(low, 0);
      }
      if (lane == 0) s_int[2] = (int)max(kk, kp);
    }
    __syncthreads();
    key_th = (uint32_t)s_int[2];
  }
  const float thr_m = a.min_p > 0.f ? vmax + logf(a.min_p) : -INFINITY;
  const float inv_t = 1.f / a.temp;

  // ---- 3. inverse-CDF draw over the kept set at the temperature
  for (int t = 0; t < ntile; ++t) {
    uint32_t b[kSmpPer];
    const int i0 = t * kSmpTile + tid * kSmpPer;
    const int n = smp_load8(lg, V, i0, a.vec, b);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kSmpPer; ++j) {
      const float v = smp_val(b[j]);
      if (j < n && smp_key(b[j]) >= key_th && v >= thr_m) s += expf((v - vmax) * inv_t);
    }
    s = smp_block_sum(s, red);
    if (tid == 0) tile_sum[t] = s;
  }
  __syncthreads();
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
  uint32_t b[kSmpPer];
  const int i0 = ti * kSmpTile + tid * kSmpPer;
  const int n = smp_load8(lg, V, i0, a.vec, b);
  float w[kSmpPer];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kSmpPer; ++j) {
    const float v = smp_val(b[j]);
    w[j] = (j < n && smp_key(b[j]) >= key_th && v >= thr_m) ? expf((v - vmax) * inv_t) : 0.f;
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
  int dev = 0;
  M5_CUDA(cudaGetDevice(&dev));
  static bool configured[64] = {false};  // once per device, normally before any graph capture
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    M5_CUDA(cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmpSmem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  sample_rows_kernel<<<rows, kSmpThreads, kSmpSmem, static_cast<cudaStream_t>(stream)>>>(a);
  M5_LAUNCH_CHECK("sample_rows_kernel");
  return M5_OK;
}
