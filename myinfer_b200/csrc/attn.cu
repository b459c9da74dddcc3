// Attention over an 8/4-bit (or bf16) KV cache, split-KV flash decoding.
//
// Restates m5engine/attention.py:29-103 (and the mlx-lm dense SDPA it falls
// back to for L == 1) as one online-softmax pass per key split:
//   * q is multiplied by `scale` and rounded to bf16 (attention.py:49);
//   * each score is rounded to bf16 before the fp32 softmax (attention.py:66-69);
//   * masked keys get probability 0 (attention.py:80-86);
//   * p is rounded to bf16 for the PV product, the denominator sums fp32 p
//     (attention.py:87-96); output = acc / max(denom, 1e-30) (attention.py:100).
// A CTA owns one kv head, a block of queries times the GQA group of q heads
// (R <= 16 rows), and one contiguous range of keys.  Key tiles of 128:
//   QK  - one thread per key walks its packed row; codes become exact floats
//         (PRMT under a power-of-two exponent, then subtract it) and scale/bias
//         are applied per 64-group: s*sum(q*code) + b*sum(q);
//   PV  - one lane per D/32 dims, one warp per 32 keys of the tile; each value
//         is dequantized as fma(code, scale, bias) exactly like the CPU oracle.
// Partial (O, max, sum) per split go to scratch; a second kernel combines.
#include <algorithm>
#include <cmath>

#include "attn.cuh"

namespace m5 {

constexpr int ATT_THREADS = 128;
constexpr int ATT_TK = 128;  // keys per tile
constexpr int ATT_RMAX = 16;

template <int BITS, int D>
struct KRow {
  static constexpr int WORDS = BITS ? D * BITS / 32 : D / 2;
};

// Exact float value of the codes of elements (2j, 2j+1) of one 32-bit word.
template <int BITS, int J>
__device__ __forceinline__ float2 code_pair(uint32_t w) {
  if constexpr (BITS == 8) {
    const float2 m = make_float2(byte32768<2 * J>(w), byte32768<2 * J + 1>(w));
    return ffma2(m, make_float2(1.f, 1.f), make_float2(-32768.f, -32768.f));
  } else if constexpr (BITS == 4) {
    const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;
    const float2 m = make_float2(nib128<J>(lo), nib128<J>(hi));
    return ffma2(m, make_float2(1.f, 1.f), make_float2(-128.f, -128.f));
  } else {
    return make_float2(bf16_lo(w), bf16_hi(w));
  }
}

template <int BITS, int D, int R>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnArgs a) {
  constexpr int DPL = D / 32;  // dims per lane in PV
  constexpr int G = D / 64;    // scale groups per row (D is 64 or 128)
  constexpr int WORDS = KRow<BITS, D>::WORDS;
  constexpr int EPW = BITS ? 32 / BITS : 2;  // elements per word
  __shared__ __align__(16) float q_s[R][D];
  __shared__ float qsum[R][G];
  __shared__ float sc[R][ATT_TK];
  __shared__ float m_s[R], l_s[R], corr_s[R];
  __shared__ int qpos_s[R];
  __shared__ __align__(16) float red[R][D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int qb = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / a.Hkv, hk = bh - b * a.Hkv;
  const int rep = a.Hq / a.Hkv;
  const int S = a.d_S ? (*a.d_S + a.S_add) : a.S_host;
  const int q0 = qb * a.QB;
  const int nq = min(a.QB, a.L - q0);
  const int rows = nq * rep;  // row r -> query q0 + r / rep, head hk*rep + r % rep

  // ---- stage scaled q (bf16-rounded) and per-group sums
  for (int i = tid; i < R * D; i += ATT_THREADS) {
    const int r = i / D, d = i - r * D;
    float v = 0.f;
    if (r < rows) {
      const int qi = q0 + r / rep, h = hk * rep + r % rep;
      v = rbf(bf2f(a.q[((size_t(b) * a.Hq + h) * a.L + qi) * D + d]) * a.scale);
    }
    q_s[r][d] = v;
  }
  if (tid < R) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
    qpos_s[tid] = S - a.L + q0 + (tid < rows ? tid / rep : 0);
  }
  __syncthreads();
  if (tid < R * G) {
    const int r = tid / G, g = tid - r * G;
    float s = 0.f;
    for (int d = 0; d < 64; ++d) s += q_s[r][g * 64 + d];
    qsum[r][g] = s;
  }

  // ---- key range of this split
  int chunk = a.chunk;
  if (chunk <= 0) chunk = ((S + a.nsplit - 1) / a.nsplit + ATT_TK - 1) / ATT_TK * ATT_TK;
  const int k_begin = split * chunk;
  int k_end = min(S, k_begin + chunk);
  if (a.mask_kind == M5_MASK_CAUSAL) k_end = min(k_end, S - a.L + q0 + nq);  // last query's position + 1

  const size_t krow_base = size_t(b) * a.k.batch_stride + size_t(hk) * a.k.head_stride;
  const size_t vrow_base = size_t(b) * a.v.batch_stride + size_t(hk) * a.v.head_stride;
  const uint32_t* kw = reinterpret_cast<const uint32_t*>(a.k.data);
  const uint32_t* vw = reinterpret_cast<const uint32_t*>(a.v.data);
  const bf16* ks = reinterpret_cast<const bf16*>(a.k.scales);
  const bf16* kb = reinterpret_cast<const bf16*>(a.k.biases);
  const bf16* vs = reinterpret_cast<const bf16*>(a.v.scales);
  const bf16* vb = reinterpret_cast<const bf16*>(a.v.biases);

  float acc[R][DPL];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[r][j] = 0.f;
  __syncthreads();

  for (int t0 = k_begin; t0 < k_end; t0 += ATT_TK) {
    // ---- QK: thread per key
    {
      const int kk = t0 + tid;
      float2 s2[G][R];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int r = 0; r < R; ++r) s2[g][r] = make_float2(0.f, 0.f);
      if (kk < k_end) {
        const uint32_t* row = kw + (krow_base + kk) * WORDS;
#pragma unroll
        for (int w4 = 0; w4 < WORDS; w4 += 4) {
          const uint4 wv = *reinterpret_cast<const uint4*>(row + w4);
          const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const int e0 = (w4 + wi) * EPW;  // first element of this word
            constexpr int g_per = 64;
            const int g = e0 / g_per;
#pragma unroll
            for (int j = 0; j < EPW / 2; ++j) {
              float2 kf;
              if (j == 0) kf = code_pair<BITS, 0>(ws[wi]);
              else if (j == 1) kf = code_pair<BITS, 1>(ws[wi]);
              else if (j == 2) kf = code_pair<BITS, 2>(ws[wi]);
              else kf = code_pair<BITS, 3>(ws[wi]);
              // code_pair<4, J> returns elements (2J, 2J+1) of the word, in
              // element order e0 + 2j, e0 + 2j + 1 for every BITS.
              const int e = e0 + 2 * j;
#pragma unroll
              for (int r = 0; r < R; ++r) {
                const float2 qv = *reinterpret_cast<const float2*>(&q_s[r][e]);
                s2[g][r] = ffma2(qv, kf, s2[g][r]);
              }
            }
          }
        }
      }
      float sk[G], bk[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sk[g] = 1.f;
        bk[g] = 0.f;
        if (BITS && kk < k_end) {
          sk[g] = bf2f(ks[(krow_base + kk) * G + g]);
          bk[g] = bf2f(kb[(krow_base + kk) * G + g]);
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float s = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float dot = s2[g][r].x + s2[g][r].y;
          s += BITS ? fmaf(sk[g], dot, bk[g] * qsum[r][g]) : dot;
        }
        s = rbf(s);
        bool valid = kk < k_end && r < rows;
        if (valid) {
          if (a.mask_kind == M5_MASK_CAUSAL) {
            valid = kk <= qpos_s[r];
          } else if (a.mask_kind == M5_MASK_BOOL || a.mask_kind == M5_MASK_ADDITIVE) {
            const int qi = q0 + r / rep, h = hk * rep + r % rep;
            const int64_t mi = b * a.ms_b + h * a.ms_h + qi * a.ms_l + kk;
            if (a.mask_kind == M5_MASK_BOOL) valid = reinterpret_cast<const uint8_t*>(a.mask)[mi] != 0;
            else s += reinterpret_cast<const float*>(a.mask)[mi];
          }
        }
        sc[r][tid] = valid ? s : -INFINITY;
      }
    }
    __syncthreads();
    // ---- online softmax per row
    for (int r = warp; r < R; r += ATT_THREADS / 32) {
      float v[ATT_TK / 32];
      float tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < ATT_TK / 32; ++i) {
        v[i] = sc[r][lane + 32 * i];
        tmax = fmaxf(tmax, v[i]);
      }
      tmax = warp_max(tmax);
      const float m_old = m_s[r];
      const float m_new = fmaxf(m_old, tmax);
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < ATT_TK / 32; ++i) {
        const float p = (v[i] == -INFINITY) ? 0.f : expf(v[i] - m_new);
        sc[r][lane + 32 * i] = p;
        psum += p;
      }
      psum = warp_sum(psum);
      if (lane == 0) {
        const float corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        corr_s[r] = corr;
        l_s[r] = l_s[r] * corr + psum;
        m_s[r] = m_new;
      }
    }
    __syncthreads();
    // ---- PV: warp takes 32 keys of the tile, lane owns DPL dims
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float c = corr_s[r];
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[r][j] *= c;
    }
    {
      const int e0 = lane * DPL;
      const int g = e0 / 64;
      const int kbeg = t0 + warp * 32;
      const int kn = max(0, min(32, k_end - kbeg));
#pragma unroll 4
      for (int j = 0; j < kn; ++j) {
        const int kk = kbeg + j;
        float vv[DPL];
        if constexpr (BITS == 0) {
          const bf16* vr = reinterpret_cast<const bf16*>(a.v.data) + (vrow_base + kk) * D + e0;
#pragma unroll
          for (int i = 0; i < DPL; ++i) vv[i] = bf2f(vr[i]);
        } else {
          const uint32_t wd = vw[(vrow_base + kk) * WORDS + e0 * BITS / 32];
          const int sh0 = (e0 * BITS) & 31;
          const float s = bf2f(vs[(vrow_base + kk) * G + g]);
          const float bb = bf2f(vb[(vrow_base + kk) * G + g]);
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const float code = float((wd >> (sh0 + i * BITS)) & ((1u << BITS) - 1));
            vv[i] = fmaf(code, s, bb);
          }
        }
        const int col = warp * 32 + j;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float p = rbf(sc[r][col]);
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[r][i] = fmaf(p, vv[i], acc[r][i]);
        }
      }
    }
    __syncthreads();
  }

  // ---- reduce the warps' partial accumulators and emit
  for (int i = tid; i < R * D; i += ATT_THREADS) (&red[0][0])[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int i = 0; i < DPL; ++i) atomicAdd(&red[r][lane * DPL + i], acc[r][i]);
  __syncthreads();
  for (int i = tid; i < rows * D; i += ATT_THREADS) {
    const int r = i / D, d = i - r * D;
    const float o = red[r][d];
    const int qi = q0 + r / rep, h = hk * rep + r % rep;
    const size_t orow = (size_t(b) * a.Hq + h) * a.L + qi;
    if (a.nsplit == 1) {
      const size_t od = a.out_tokens_major ? ((size_t(b) * a.L + qi) * a.Hq + h) : orow;
      a.out[od * D + d] = f2bf(o / fmaxf(l_s[r], 1e-30f));
    } else {
      a.part_o[(orow * a.nsplit + split) * D + d] = o;
      if (d == 0) {
        a.part_ml[(orow * a.nsplit + split) * 2 + 0] = m_s[r];
        a.part_ml[(orow * a.nsplit + split) * 2 + 1] = l_s[r];
      }
    }
  }
}

// Merge of the split-KV partials of one output row (b, h, qi): weights
// exp(m_s - M) over the splits, out = sum_s w_s o_s / sum_s w_s l_s.  One CTA
// per (row, 32 output dims): its 8 warps take every 8th split with coalesced
// 128-byte loads of the partial rows, the split weights are computed once per
// CTA, and the 8 warp sums are added in shared memory.
constexpr int CMB_WARPS = 8;
__global__ void __launch_bounds__(CMB_WARPS * 32) attn_combine_kernel(const float* __restrict__ part_o,
                                                                       const float* __restrict__ part_ml,
                                                                       int nsplit, int D, int Hq, int L,
                                                                       int tokens_major, bf16* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t row = blockIdx.x;  // (b * Hq + h) * L + qi
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = blockIdx.y * 32 + lane;
  __shared__ float w_s[1024];
  __shared__ float red[CMB_WARPS][33];
  const float* ml = part_ml + row * nsplit * 2;
  float m = -INFINITY;
  for (int s = tid; s < nsplit; s += CMB_WARPS * 32) m = fmaxf(m, ml[2 * s]);
  m = warp_max(m);
  if (lane == 0) red[warp][32] = m;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < CMB_WARPS; ++w) M = fmaxf(M, red[w][32]);
  float den = 0.f;
  for (int s = tid; s < nsplit; s += CMB_WARPS * 32) {
    const float ms = ml[2 * s];
    const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
    w_s[s] = w;
    den = fmaf(w, ml[2 * s + 1], den);
  }
  den = warp_sum(den);
  __syncthreads();  // every warp has read red[.][32]; w_s complete
  if (lane == 0) red[warp][32] = den;
  float num = 0.f;
  if (d < D) {
    const float* po = part_o + row * nsplit * D + d;
#pragma unroll 4
    for (int s = warp; s < nsplit; s += CMB_WARPS) num = fmaf(w_s[s], po[size_t(s) * D], num);
  }
  red[warp][lane] = num;
  __syncthreads();
  if (warp == 0 && d < D) {
    float tot = 0.f, dsum = 0.f;
#pragma unroll
    for (int w = 0; w < CMB_WARPS; ++w) {
      tot += red[w][lane];
      dsum += red[w][32];
    }
    size_t od = row;
    if (tokens_major) {
      const size_t qi = row % L, bh = row / L, h = bh % Hq, b = bh / Hq;
      od = (b * L + qi) * Hq + h;
    }
    out[od * D + d] = f2bf(tot / fmaxf(dsum, 1e-30f));
  }
}

size_t attn_scratch_bytes(int B, int Hq, int L, int D, int nsplit) {
  if (nsplit <= 1) return 0;
  const size_t rows = size_t(B) * Hq * L;
  return rows * nsplit * (size_t(D) + 2) * sizeof(float);
}

void attn_plan(int B, int Hq, int Hkv, int L, int S_max, int& QB, int& nsplit) {
  const int rep = Hq / Hkv;
  QB = std::max(1, ATT_RMAX / rep);
  if (QB > L) QB = L;
  const long long ctas = (long long)B * Hkv * ((L + QB - 1) / QB);
  const int tiles = std::max(1, (S_max + ATT_TK - 1) / ATT_TK);
  // Enough CTAs to fill the SMs once at the tensor-core kernel's occupancy
  // (3 per SM for one 8-row query block, else 2), each with at least one key
  // tile; more, shorter splits than resident slots only add per-CTA prologue
  // and merge work.
  const long long per_sm = attn_mma_ctas_per_sm(std::min(QB, L) * rep);
  long long want = (per_sm * sm_count() + ctas - 1) / ctas;
  nsplit = (int)std::max(1LL, std::min<long long>(std::min<long long>(want, tiles), 1024));
}

template <int BITS, int D, int R>
static int launch_kernel(const AttnArgs& a, cudaStream_t stream) {
  dim3 grid(a.nsplit, (a.L + a.QB - 1) / a.QB, a.B * a.Hkv);
  attn_kernel<BITS, D, R><<<grid, ATT_THREADS, 0, stream>>>(a);
  M5_LAUNCH_CHECK("attention launch");
  return M5_OK;
}

template <int BITS, int D>
static int launch_r(const AttnArgs& a, int R, cudaStream_t stream) {
  if (R <= 2) return launch_kernel<BITS, D, 2>(a, stream);
  if (R <= 4) return launch_kernel<BITS, D, 4>(a, stream);
  if (R <= 8) return launch_kernel<BITS, D, 8>(a, stream);
  return launch_kernel<BITS, D, 16>(a, stream);
}

int attn_launch(const AttnArgs& a, cudaStream_t stream) {
  const int rep = a.Hq / a.Hkv;
  const int R = a.QB * rep;
  if (R > ATT_RMAX) return fail(M5_ERR_INVALID, "attention: queries-per-CTA x GQA group exceeds 16");
  int rc;
  if (attn_pf_eligible(a)) {
    // prefill: 128 rows per CTA; the caller's scratch holds a.nsplit partials per row
    AttnArgs p = a;
    const int S_max = a.d_S ? a.k.head_stride : a.S_host;
    if (attn_tc_eligible(a)) {
      attn_tc_plan(a, (int)std::min<int64_t>(S_max, 1 << 30), std::max(1, a.nsplit), p.QB, p.nsplit);
      if ((rc = attn_tc_launch(p, stream))) return rc;
    } else {
      attn_pf_plan(a, (int)std::min<int64_t>(S_max, 1 << 30), std::max(1, a.nsplit), p.QB, p.nsplit);
      if ((rc = attn_pf_launch(p, stream))) return rc;
    }
    if (p.nsplit > 1) {
      const int rows = a.B * a.Hq * a.L;
      M5_CUDA(launch_pdl(attn_combine_kernel, dim3(rows, 4), dim3(CMB_WARPS * 32), 0, stream, p.part_o, p.part_ml,
                         p.nsplit, 128, a.Hq, a.L, a.out_tokens_major, a.out));
      M5_LAUNCH_CHECK("attention combine launch");
    }
    return M5_OK;
  }
  if (attn_mma_eligible(a)) {
    rc = attn_mma_launch(a, stream);
  } else if (a.D == 128) {
    if (a.bits == 8) rc = launch_r<8, 128>(a, R, stream);
    else if (a.bits == 4) rc = launch_r<4, 128>(a, R, stream);
    else rc = launch_r<0, 128>(a, R, stream);
  } else {
    if (a.bits == 8) rc = launch_r<8, 64>(a, R, stream);
    else if (a.bits == 4) rc = launch_r<4, 64>(a, R, stream);
    else rc = launch_r<0, 64>(a, R, stream);
  }
  if (rc) return rc;
  if (a.nsplit > 1) {
    const int rows = a.B * a.Hq * a.L;
    M5_CUDA(launch_pdl(attn_combine_kernel, dim3(rows, (a.D + 31) / 32), dim3(CMB_WARPS * 32), 0, stream, a.part_o,
                       a.part_ml, a.nsplit, a.D, a.Hq, a.L, a.out_tokens_major, a.out));
    M5_LAUNCH_CHECK("attention combine launch");
  }
  return M5_OK;
}

}  // namespace m5
