// Prefill flash attention over an 8/4-bit KV cache on the tensor cores
// (kernel K4p: chunks of L queries, rows = GQA group x queries up to 128).
//
// Work of one CTA: one kv head, QB = 128 / rep query tokens (all rep heads of
// the group: 128 rows), one key range.  A producer warp streams 64-key tiles of
// K, V and their bf16 scales/biases with 1-D bulk copies into a 4-stage ring
// (bounded mbarrier waits).  Eight consumer warps each own 16 rows and run
// every key of every tile, so each warp keeps a complete online-softmax state
// for its rows and no cross-warp merge is needed.
//
// Arithmetic per 64-key tile and warp is the decode kernel's (attn_mma.cu),
// scaled up: S = Q K^T with q in fp16 (exact: bf16-rounded q * scale) against
// exact fp16 codes, one MMA chain per 64-dim scale group, folded as
// scale_g * (q . code_g) + bias_g * sum(q_g); scores rounded to bf16
// (attention.py:66-69), fp32 online softmax, p rounded to bf16 for PV
// (attention.py:87-90) with the per-key value scale folded into A = p * vscale
// * 2^6 (fp16) and the value bias accumulated as p * vbias in fp32.
// 8 + 8 mma.sync m16n8k16 per 16 x 8 block of S / of O per 16 keys.
#include <algorithm>
#include <cmath>

#include "attn.cuh"
#include "tma.cuh"

namespace m5 {

static __device__ int g_attn_pf_err = 0;

namespace apf {

constexpr int TK = 64;          // keys per stage
constexpr int STAGES = 4;
constexpr int CW = 8;           // consumer warps, 16 rows each
constexpr int ROWS = 16 * CW;   // rows per CTA
constexpr int THREADS = (CW + 1) * 32;
constexpr float PSCALE = 64.f;  // p * vscale is kept in fp16 scaled by 2^6

template <int BITS>
struct Layout {
  static constexpr int KROW = 128 * BITS / 8;          // packed bytes per key row (D = 128)
  static constexpr int K_OFF = 0;
  static constexpr int KS_OFF = K_OFF + TK * KROW;     // bf16 [TK][2]
  static constexpr int KB_OFF = KS_OFF + TK * 4;
  static constexpr int V_OFF = KB_OFF + TK * 4;
  static constexpr int VS_OFF = V_OFF + TK * KROW;
  static constexpr int VB_OFF = VS_OFF + TK * 4;
  static constexpr int STAGE = VB_OFF + TK * 4;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t hsub1024(uint32_t x) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(0x64006400u));
  return r;
}

template <int SEL>
__device__ __forceinline__ uint32_t code8_pair(uint32_t w) {
  return hsub1024(__byte_perm(w, 0x64u, SEL));
}
__device__ __forceinline__ uint32_t code4_pair(uint32_t w, int i) {
  return hsub1024(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u);
}

// Physical dim of contraction slot (slice j, logical k) of lane quad index t
// (the same permutation as the decode kernel: a lane reads 16 contiguous code
// bytes per 64-dim group and every MMA stays inside one scale group).
template <int BITS>
__device__ __forceinline__ int qk_dim(int j, int t, int k) {
  const int G = j >> 2, sub = j & 3;
  const int hi = k >= 8, e = k & 1;
  if constexpr (BITS == 8) {
    return 64 * G + 16 * t + 4 * sub + 2 * hi + e;
  } else {
    const int w = sub >> 1, i0 = 2 * (sub & 1);
    const int n = i0 + hi + 4 * e;
    return 64 * G + 16 * t + 8 * w + n;
  }
}

template <int BITS>
__global__ void __launch_bounds__(THREADS, 1) attn_pf_kernel(const AttnArgs a) {
  using LY = Layout<BITS>;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * LY::STAGE);
  uint64_t* empty = full + STAGES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x;
  const int b = blockIdx.z / a.Hkv, hk = blockIdx.z % a.Hkv;
  const int rep = a.Hq / a.Hkv;
  const int S = a.d_S ? (*a.d_S + a.S_add) : a.S_host;
  const int q0 = blockIdx.y * a.QB;
  const int nq = min(a.QB, a.L - q0);
  const int rows = nq * rep;

  int chunk = a.chunk;
  if (chunk <= 0) chunk = ((S + a.nsplit - 1) / a.nsplit + TK - 1) / TK * TK;
  const int k_begin = split * chunk;
  int k_end = min(S, k_begin + chunk);
  if (a.mask_kind == M5_MASK_CAUSAL) k_end = min(k_end, S - a.L + q0 + nq);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + TK - 1) / TK : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      const size_t kbase = size_t(b) * a.k.batch_stride + size_t(hk) * a.k.head_stride;
      const size_t vbase = size_t(b) * a.v.batch_stride + size_t(hk) * a.v.head_stride;
      const unsigned char* kd = reinterpret_cast<const unsigned char*>(a.k.data);
      const unsigned char* vd = reinterpret_cast<const unsigned char*>(a.v.data);
      const unsigned char* ksd = reinterpret_cast<const unsigned char*>(a.k.scales);
      const unsigned char* kbd = reinterpret_cast<const unsigned char*>(a.k.biases);
      const unsigned char* vsd = reinterpret_cast<const unsigned char*>(a.v.scales);
      const unsigned char* vbd = reinterpret_cast<const unsigned char*>(a.v.biases);
      int issued = 0;
      for (int it = 0; it < ntiles; ++it) {
        const int st = it % STAGES;
        if (!mbar_wait(&empty[st], ((it / STAGES) & 1) ^ 1, &g_attn_pf_err)) break;
        const int key0 = k_begin + it * TK;
        const int nk = (min(TK, k_end - key0) + 3) & ~3;  // whole 16-byte scale rows
        unsigned char* sb = smem + st * LY::STAGE;
        const uint32_t rowb = nk * LY::KROW, sclb = nk * 4;
        mbar_arrive_expect_tx(&full[st], 2 * rowb + 4 * sclb);
        bulk_g2s(sb + LY::K_OFF, kd + (kbase + key0) * LY::KROW, rowb, &full[st]);
        bulk_g2s(sb + LY::KS_OFF, ksd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::KB_OFF, kbd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::V_OFF, vd + (vbase + key0) * LY::KROW, rowb, &full[st]);
        bulk_g2s(sb + LY::VS_OFF, vsd + (vbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::VB_OFF, vbd + (vbase + key0) * 4, sclb, &full[st]);
        issued = it + 1;
      }
      // the copies in flight land before the CTA may exit
      for (int it = std::max(0, issued - STAGES); it < issued; ++it)
        (void)mbar_wait(&full[it % STAGES], (it / STAGES) & 1, &g_attn_pf_err);
    }
    return;
  }

  // ----------------------------------------------------------- consumers
  // rows of this warp: 16 * warp + (g, g + 8); row r -> token q0 + r / rep, head hk * rep + r % rep
  const int r0 = 16 * warp + g, r8 = r0 + 8;
  // q fragments, scaled and bf16-rounded (attention.py:49), permuted dims
  uint32_t qa[8][4];
  float qsum[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [row g / g+8][group]
  {
    const bf16* qr[2] = {nullptr, nullptr};
    const int rr[2] = {r0, r8};
#pragma unroll
    for (int hr = 0; hr < 2; ++hr)
      if (rr[hr] < rows) {
        const int qi = q0 + rr[hr] / rep, h = hk * rep + rr[hr] % rep;
        qr[hr] = a.q + ((size_t(b) * a.Hq + h) * a.L + qi) * 128;
      }
    auto qv = [&](int hr, int d) -> float {
      return qr[hr] ? rbf(bf2f(qr[hr][d]) * a.scale) : 0.f;
    };
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d0 = qk_dim<BITS>(j, t, 2 * t), d1 = qk_dim<BITS>(j, t, 2 * t + 1);
      const int d8 = qk_dim<BITS>(j, t, 2 * t + 8), d9 = qk_dim<BITS>(j, t, 2 * t + 9);
      const float x0 = qv(0, d0), x1 = qv(0, d1), x8 = qv(0, d8), x9 = qv(0, d9);
      const float y0 = qv(1, d0), y1 = qv(1, d1), y8 = qv(1, d8), y9 = qv(1, d9);
      qa[j][0] = pack_h2(x0, x1);
      qa[j][1] = pack_h2(y0, y1);
      qa[j][2] = pack_h2(x8, x9);
      qa[j][3] = pack_h2(y8, y9);
      qsum[0][j >> 2] += (x0 + x1) + (x8 + x9);
      qsum[1][j >> 2] += (y0 + y1) + (y8 + y9);
    }
    // the quad's four lanes hold disjoint dims of the same rows
#pragma unroll
    for (int hr = 0; hr < 2; ++hr)
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        qsum[hr][G] += __shfl_xor_sync(0xffffffffu, qsum[hr][G], 1);
        qsum[hr][G] += __shfl_xor_sync(0xffffffffu, qsum[hr][G], 2);
      }
  }
  const int qp0 = S - a.L + q0 + min(r0, max(rows - 1, 0)) / rep;
  const int qp8 = S - a.L + q0 + min(r8, max(rows - 1, 0)) / rep;
  const bool causal = a.mask_kind == M5_MASK_CAUSAL;

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float vb_acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int it = 0; it < ntiles; ++it) {
    const int st = it % STAGES;
    if (!mbar_wait(&full[st], (it / STAGES) & 1, &g_attn_pf_err)) break;
    const unsigned char* sb = smem + st * LY::STAGE;
    const int tile_key0 = k_begin + it * TK;

    // ---------------- S = Q K^T, 8 blocks of 8 keys
    float sc[8][4];
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
      const int kl = 8 * kb + g;
      float dG[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        if constexpr (BITS == 8) {
          const uint4 c = *reinterpret_cast<const uint4*>(sb + LY::K_OFF + kl * 128 + 64 * G + 16 * t);
          const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
          for (int sub = 0; sub < 4; ++sub)
            mma_f16(dG[G], qa[4 * G + sub], code8_pair<0x4140>(w4[sub]), code8_pair<0x4342>(w4[sub]));
        } else {
          const uint2 c = *reinterpret_cast<const uint2*>(sb + LY::K_OFF + kl * 64 + 32 * G + 8 * t);
          const uint32_t w2[2] = {c.x, c.y};
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) {
            const uint32_t w = w2[sub >> 1];
            const int i0 = 2 * (sub & 1);
            mma_f16(dG[G], qa[4 * G + sub], code4_pair(w, i0), code4_pair(w, i0 + 1));
          }
        }
      }
      const int kk = 8 * kb + 2 * t;
      const uint2 ks2 = *reinterpret_cast<const uint2*>(sb + LY::KS_OFF + kk * 4);
      const uint2 kb2 = *reinterpret_cast<const uint2*>(sb + LY::KB_OFF + kk * 4);
      const float s00 = bf16_lo(ks2.x), s01 = bf16_hi(ks2.x), s10 = bf16_lo(ks2.y), s11 = bf16_hi(ks2.y);
      const float b00 = bf16_lo(kb2.x), b01 = bf16_hi(kb2.x), b10 = bf16_lo(kb2.y), b11 = bf16_hi(kb2.y);
      float s[4];
      s[0] = fmaf(s00, dG[0][0], b00 * qsum[0][0]) + fmaf(s01, dG[1][0], b01 * qsum[0][1]);
      s[1] = fmaf(s10, dG[0][1], b10 * qsum[0][0]) + fmaf(s11, dG[1][1], b11 * qsum[0][1]);
      s[2] = fmaf(s00, dG[0][2], b00 * qsum[1][0]) + fmaf(s01, dG[1][2], b01 * qsum[1][1]);
      s[3] = fmaf(s10, dG[0][3], b10 * qsum[1][0]) + fmaf(s11, dG[1][3], b11 * qsum[1][1]);
      const int key0 = tile_key0 + kk;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = key0 + (i & 1);
        const int qp = (i < 2) ? qp0 : qp8;
        const bool valid = key < k_end && (!causal || key <= qp);
        sc[kb][i] = valid ? rbf(s[i]) : -INFINITY;
      }
    }

    // ---------------- online softmax (rows g, g+8; a quad shares a row)
    float pm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
      pm[0] = fmaxf(pm[0], fmaxf(sc[kb][0], sc[kb][1]));
      pm[1] = fmaxf(pm[1], fmaxf(sc[kb][2], sc[kb][3]));
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      pm[hr] = fmaxf(pm[hr], __shfl_xor_sync(0xffffffffu, pm[hr], 1));
      pm[hr] = fmaxf(pm[hr], __shfl_xor_sync(0xffffffffu, pm[hr], 2));
    }
    float corr[2];
    bool changed = false;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const float mn = fmaxf(m_run[hr], pm[hr]);
      corr[hr] = (m_run[hr] == mn) ? 1.f : (m_run[hr] == -INFINITY ? 0.f : expf(m_run[hr] - mn));
      changed |= corr[hr] != 1.f;
      m_run[hr] = mn;
    }
    if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[0];
        o[i][2] *= corr[1];
        o[i][3] *= corr[1];
      }
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        vb_acc[0][G] *= corr[0];
        vb_acc[1][G] *= corr[1];
      }
      l_run[0] *= corr[0];
      l_run[1] *= corr[1];
    }
    // p in place of the scores (fp32); l accumulates fp32 p
#pragma unroll
    for (int kb = 0; kb < 8; ++kb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float mm = m_run[i >> 1];
        const float pv = (sc[kb][i] == -INFINITY) ? 0.f : expf(sc[kb][i] - mm);
        l_run[i >> 1] += pv;
        sc[kb][i] = pv;
      }

    // ---------------- O += P V, 4 slices of 16 keys (key blocks 2ks, 2ks+1)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int vk0 = 16 * ks + 2 * t, vk1 = 16 * ks + 8 + 2 * t;
      const uint2 vs0 = *reinterpret_cast<const uint2*>(sb + LY::VS_OFF + vk0 * 4);
      const uint2 vs1 = *reinterpret_cast<const uint2*>(sb + LY::VS_OFF + vk1 * 4);
      const uint2 vb0 = *reinterpret_cast<const uint2*>(sb + LY::VB_OFF + vk0 * 4);
      const uint2 vb1 = *reinterpret_cast<const uint2*>(sb + LY::VB_OFF + vk1 * 4);
      const float* pA = sc[2 * ks];
      const float* pB = sc[2 * ks + 1];
      const float r00 = rbf(pA[0]), r01 = rbf(pA[1]), r02 = rbf(pA[2]), r03 = rbf(pA[3]);
      const float r10 = rbf(pB[0]), r11 = rbf(pB[1]), r12 = rbf(pB[2]), r13 = rbf(pB[3]);
      // masked keys have p == 0; their stage bytes may be stale, so never multiply them
      auto mul = [](float r, float x) { return r == 0.f ? 0.f : r * x; };
      uint32_t pa[2][4];
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        const float sA0 = G ? bf16_hi(vs0.x) : bf16_lo(vs0.x), sA1 = G ? bf16_hi(vs0.y) : bf16_lo(vs0.y);
        const float sB0 = G ? bf16_hi(vs1.x) : bf16_lo(vs1.x), sB1 = G ? bf16_hi(vs1.y) : bf16_lo(vs1.y);
        const float bA0 = G ? bf16_hi(vb0.x) : bf16_lo(vb0.x), bA1 = G ? bf16_hi(vb0.y) : bf16_lo(vb0.y);
        const float bB0 = G ? bf16_hi(vb1.x) : bf16_lo(vb1.x), bB1 = G ? bf16_hi(vb1.y) : bf16_lo(vb1.y);
        pa[G][0] = pack_h2(mul(r00, sA0 * PSCALE), mul(r01, sA1 * PSCALE));
        pa[G][1] = pack_h2(mul(r02, sA0 * PSCALE), mul(r03, sA1 * PSCALE));
        pa[G][2] = pack_h2(mul(r10, sB0 * PSCALE), mul(r11, sB1 * PSCALE));
        pa[G][3] = pack_h2(mul(r12, sB0 * PSCALE), mul(r13, sB1 * PSCALE));
        vb_acc[0][G] += mul(r00, bA0) + mul(r01, bA1) + mul(r10, bB0) + mul(r11, bB1);
        vb_acc[1][G] += mul(r02, bA0) + mul(r03, bA1) + mul(r12, bB0) + mul(r13, bB1);
      }
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        uint32_t vw[2][4];
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const int kl = 16 * ks + 8 * kb + g;
          if constexpr (BITS == 8) {
            const uint4 c = *reinterpret_cast<const uint4*>(sb + LY::V_OFF + kl * 128 + 64 * G + 16 * t);
            vw[kb][0] = c.x; vw[kb][1] = c.y; vw[kb][2] = c.z; vw[kb][3] = c.w;
          } else {
            const uint2 c = *reinterpret_cast<const uint2*>(sb + LY::V_OFF + kl * 64 + 32 * G + 8 * t);
            vw[kb][0] = c.x; vw[kb][1] = c.y; vw[kb][2] = 0; vw[kb][3] = 0;
          }
        }
#pragma unroll
        for (int dbl = 0; dbl < 8; ++dbl) {
          uint32_t bb[2];
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            uint32_t pr;
            if constexpr (BITS == 8) {
              const uint32_t w = vw[kb][dbl >> 1];
              pr = (dbl & 1) ? code8_pair<0x4342>(w) : code8_pair<0x4140>(w);
            } else {
              const uint32_t w = vw[kb][dbl >> 2];
              const int n0 = (2 * dbl) & 7;
              const uint32_t lo = (w >> (4 * n0)) & 0xFu, hi = (w >> (4 * n0 + 4)) & 0xFu;
              pr = hsub1024(0x64006400u | lo | (hi << 16));
            }
            bb[kb] = movmatrix_t(pr);
          }
          mma_f16(o[8 * G + dbl], pa[G], bb[0], bb[1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ---------------- finish: quad reductions, then each lane writes its dims
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      vb_acc[hr][G] += __shfl_xor_sync(0xffffffffu, vb_acc[hr][G], 1);
      vb_acc[hr][G] += __shfl_xor_sync(0xffffffffu, vb_acc[hr][G], 2);
    }
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = hr ? r8 : r0;
    if (r >= rows) continue;
    const int qi = q0 + r / rep, h = hk * rep + r % rep;
    const size_t orow = (size_t(b) * a.Hq + h) * a.L + qi;
    const float inv = 1.f / fmaxf(l_run[hr], 1e-30f);
#pragma unroll
    for (int db = 0; db < 16; ++db) {
      const int G = db >> 3, dbl = db & 7;
      const int d0 = 64 * G + 16 * t + 2 * dbl;
      const float n0 = o[db][2 * hr] / PSCALE + vb_acc[hr][G];
      const float n1 = o[db][2 * hr + 1] / PSCALE + vb_acc[hr][G];
      if (a.nsplit == 1) {
        const size_t od = a.out_tokens_major ? ((size_t(b) * a.L + qi) * a.Hq + h) : orow;
        __nv_bfloat162 v2 = __floats2bfloat162_rn(n0 * inv, n1 * inv);
        *reinterpret_cast<__nv_bfloat162*>(a.out + od * 128 + d0) = v2;
      } else {
        float* po = a.part_o + (orow * a.nsplit + split) * 128;
        po[d0] = n0;
        po[d0 + 1] = n1;
      }
    }
    if (a.nsplit > 1 && t == 0) {
      a.part_ml[(orow * a.nsplit + split) * 2 + 0] = m_run[hr];
      a.part_ml[(orow * a.nsplit + split) * 2 + 1] = l_run[hr];
    }
  }
}

}  // namespace apf

static size_t apf_smem(int bits) {
  const size_t stage = bits == 8 ? apf::Layout<8>::STAGE : apf::Layout<4>::STAGE;
  return apf::STAGES * stage + 2 * apf::STAGES * 8;
}

bool attn_pf_eligible(const AttnArgs& a) {
  if (a.D != 128 || (a.bits != 8 && a.bits != 4)) return false;
  if (a.mask_kind != M5_MASK_NONE && a.mask_kind != M5_MASK_CAUSAL) return false;
  const int rep = a.Hq / a.Hkv;
  if (rep < 1 || rep > apf::ROWS || apf::ROWS % rep) return false;
  if (a.L * rep <= 16) return false;  // the decode kernel covers these
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.k.data) || !al(a.v.data) || !al(a.k.scales) || !al(a.k.biases) || !al(a.v.scales) || !al(a.v.biases))
    return false;
  if ((a.k.head_stride % 4) || (a.v.head_stride % 4) || (a.k.batch_stride % 4) || (a.v.batch_stride % 4))
    return false;
  if (!a.d_S) {
    const long long s4 = (a.S_host + 3LL) / 4 * 4;
    if (s4 > a.k.head_stride || s4 > a.v.head_stride) return false;
  }
  return true;
}

// Queries per CTA for the prefill kernel and a split count (<= max_split) that
// gives about two CTAs per SM.
void attn_pf_plan(const AttnArgs& a, int S_max, int max_split, int& QB, int& nsplit) {
  const int rep = a.Hq / a.Hkv;
  QB = std::max(1, std::min(a.L, apf::ROWS / rep));
  const long long ctas = (long long)a.B * a.Hkv * ((a.L + QB - 1) / QB);
  const int tiles = std::max(1, (S_max + apf::TK - 1) / apf::TK);
  const long long want = (2LL * sm_count() + ctas - 1) / ctas;
  nsplit = (int)std::max(1LL, std::min<long long>(std::min<long long>(want, tiles), max_split));
}

int attn_pf_launch(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = apf_smem(a.bits);
  static DeviceOnce once8, once4;  // the attribute belongs to each device's context
  dim3 grid(a.nsplit, (a.L + a.QB - 1) / a.QB, a.B * a.Hkv);
  if (a.bits == 8) {
    M5_CUDA(once8.run(
        [&] { return cudaFuncSetAttribute(apf::attn_pf_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); }));
    apf::attn_pf_kernel<8><<<grid, apf::THREADS, smem, stream>>>(a);
  } else {
    M5_CUDA(once4.run(
        [&] { return cudaFuncSetAttribute(apf::attn_pf_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); }));
    apf::attn_pf_kernel<4><<<grid, apf::THREADS, smem, stream>>>(a);
  }
  M5_LAUNCH_CHECK("prefill attention launch");
  return M5_OK;
}

int attn_pf_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_pf_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_pf_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
