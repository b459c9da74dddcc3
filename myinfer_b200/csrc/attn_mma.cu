// Split-KV flash decoding over an 8/4-bit KV cache on the tensor cores
// (kernel K4, rows = GQA group x queries <= 16).
//
// Work of one CTA: one kv head, one contiguous key range (a split).  A
// producer warp streams 64-key tiles of K, V and their bf16 scales/biases
// with 1-D bulk copies (each head's rows are contiguous) into a 4-stage
// shared-memory ring guarded by mbarriers (bounded waits).  Four consumer
// warps take 16 keys of every tile each and keep their own online-softmax
// state; the states are merged at the end of the split.
//
// Per 16-key step of a consumer warp (mma.sync m16n8k16, fp16 in, fp32 acc):
//   S = Q K^T : A = q (rows = heads of the group, scaled by `scale` and rounded
//               to bf16 like attention.py:49; exact in fp16), B = K codes.  A
//               code becomes an fp16 operand with one PRMT per two codes
//               (byte | 0x6400 = 1024 + code) and one HSUB2 (exact code);
//               contraction dims are permuted so a lane reads 16 contiguous
//               code bytes per 64-dim group, and every MMA stays inside one
//               scale group, so  s = sum_g scale_g * (q . code_g) + bias_g * sum(q_g)
//               is the reference's dequantized dot product.
//   scores rounded to bf16 (attention.py:66-69), fp32 online softmax; p rounded
//   to bf16 for PV (attention.py:87-90), fp32 p in the denominator.
//   O += P V  : the per-key value scale is folded into A = p * vscale_g * 2^6
//               (one A per scale group; fp16), B = V codes transposed in
//               registers with movmatrix; the per-key value bias adds
//               p * vbias_g to an fp32 side sum.
#include <algorithm>
#include <cmath>

#include "attn.cuh"
#include "tma.cuh"

namespace m5 {

static __device__ int g_attn_mma_err = 0;

constexpr int AM_TK = 64;       // keys per stage
constexpr int AM_STAGES = 4;
constexpr int AM_CW = 4;        // consumer warps (16 keys of each stage each)
constexpr int AM_THREADS = (AM_CW + 1) * 32;
constexpr float AM_PSCALE = 64.f;  // p * vscale is kept in fp16 scaled by 2^6

template <int BITS>
struct AmLayout {
  static constexpr int KROW = 128 * BITS / 8;           // packed bytes per key row (D = 128)
  static constexpr int K_OFF = 0;
  static constexpr int KS_OFF = K_OFF + AM_TK * KROW;   // bf16 [TK][2]
  static constexpr int KB_OFF = KS_OFF + AM_TK * 4;
  static constexpr int V_OFF = KB_OFF + AM_TK * 4;
  static constexpr int VS_OFF = V_OFF + AM_TK * KROW;
  static constexpr int VB_OFF = VS_OFF + AM_TK * 4;
  static constexpr int STAGE = VB_OFF + AM_TK * 4;
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

// fp16 pair (code_a, code_b) exactly, from 8-bit codes at bytes ia, ib of w.
template <int SEL>
__device__ __forceinline__ uint32_t code8_pair(uint32_t w) {
  return hsub1024(__byte_perm(w, 0x64u, SEL));
}
// fp16 pair (nibble i, nibble i+4) of w exactly.
__device__ __forceinline__ uint32_t code4_pair(uint32_t w, int i) {
  return hsub1024(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u);
}

// Physical dim of contraction slot (slice j, logical k) of lane quad index t.
template <int BITS>
__device__ __forceinline__ int qk_dim(int j, int t, int k) {
  const int G = j >> 2, sub = j & 3;
  const int hi = k >= 8, e = k & 1;  // k in {2t, 2t+1, 2t+8, 2t+9}
  if constexpr (BITS == 8) {
    return 64 * G + 16 * t + 4 * sub + 2 * hi + e;
  } else {
    const int w = sub >> 1, i0 = 2 * (sub & 1);
    const int n = i0 + hi + 4 * e;
    return 64 * G + 16 * t + 8 * w + n;
  }
}

template <int BITS>
__global__ void __launch_bounds__(AM_THREADS) attn_mma_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  using LY = AmLayout<BITS>;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + AM_STAGES * LY::STAGE);
  uint64_t* empty = full + AM_STAGES;
  float* q_s = reinterpret_cast<float*>(empty + AM_STAGES);  // [16][128] scaled, bf16-rounded q
  int* qpos = reinterpret_cast<int*>(q_s + 16 * 128);        // [16]

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
  if (chunk <= 0) chunk = ((S + a.nsplit - 1) / a.nsplit + AM_TK - 1) / AM_TK * AM_TK;
  const int k_begin = split * chunk;
  int k_end = min(S, k_begin + chunk);
  if (a.mask_kind == M5_MASK_CAUSAL) k_end = min(k_end, S - a.L + q0 + nq);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + AM_TK - 1) / AM_TK : 0;

  if (tid == 0) {
    for (int s = 0; s < AM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], AM_CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == AM_CW) {
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
      for (int it = 0; it < ntiles; ++it) {
        const int st = it % AM_STAGES;
        const uint32_t par = (it / AM_STAGES) & 1;
        if (!mbar_wait(&empty[st], par ^ 1, &g_attn_mma_err)) return;
        const int key0 = k_begin + it * AM_TK;
        const int nk = (min(AM_TK, k_end - key0) + 3) & ~3;  // whole 16-byte scale rows
        unsigned char* sb = smem + st * LY::STAGE;
        const uint32_t rowb = nk * LY::KROW, sclb = nk * 4;
        mbar_arrive_expect_tx(&full[st], 2 * rowb + 4 * sclb);
        bulk_g2s(sb + LY::K_OFF, kd + (kbase + key0) * LY::KROW, rowb, &full[st]);
        bulk_g2s(sb + LY::KS_OFF, ksd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::KB_OFF, kbd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::V_OFF, vd + (vbase + key0) * LY::KROW, rowb, &full[st]);
        bulk_g2s(sb + LY::VS_OFF, vsd + (vbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + LY::VB_OFF, vbd + (vbase + key0) * 4, sclb, &full[st]);
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers
  // stage scaled q (bf16-rounded) for the 16 MMA rows; padding rows are zero.
  // 16 rows x 16 blocks of 8 bf16 = 256 16-byte loads, two per thread, both
  // issued before use.
  {
    uint4 v[2];
    int rr[2], cc[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * AM_CW * 32;  // 0..255
      rr[k] = i >> 4;
      cc[k] = i & 15;
      v[k] = make_uint4(0, 0, 0, 0);
      if (rr[k] < rows) {
        const int qi = q0 + rr[k] / rep, h = hk * rep + rr[k] % rep;
        v[k] = *reinterpret_cast<const uint4*>(a.q + ((size_t(b) * a.Hq + h) * a.L + qi) * 128 + cc[k] * 8);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      float* dst = q_s + rr[k] * 128 + cc[k] * 8;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        dst[2 * q] = rbf(bf16_lo(w[q]) * a.scale);
        dst[2 * q + 1] = rbf(bf16_hi(w[q]) * a.scale);
      }
    }
  }
  if (tid < 16) qpos[tid] = S - a.L + q0 + (tid < rows ? tid / rep : 0);
  named_sync(1, AM_CW * 32);

  // A fragments of q for the 8 contraction slices, and per-group sums of q
  uint32_t qa[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float* r0 = q_s + g * 128;
    const float* r8 = q_s + (g + 8) * 128;
    const int d0 = qk_dim<BITS>(j, t, 2 * t), d1 = qk_dim<BITS>(j, t, 2 * t + 1);
    const int d8 = qk_dim<BITS>(j, t, 2 * t + 8), d9 = qk_dim<BITS>(j, t, 2 * t + 9);
    qa[j][0] = pack_h2(r0[d0], r0[d1]);
    qa[j][1] = pack_h2(r8[d0], r8[d1]);
    qa[j][2] = pack_h2(r0[d8], r0[d9]);
    qa[j][3] = pack_h2(r8[d8], r8[d9]);
  }
  // per-(row, group) sums of q: 4 threads x 16 elements per (row, group)
  float* qsum_s = reinterpret_cast<float*>(qpos + 16);  // [16][2]
  {
    const int pair = tid >> 2, part = tid & 3;  // 32 (row, group) pairs
    const float4* src = reinterpret_cast<const float4*>(q_s + (pair >> 1) * 128 + (pair & 1) * 64 + part * 16);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 f = src[k];
      sum += (f.x + f.y) + (f.z + f.w);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (part == 0) qsum_s[pair] = sum;
  }
  named_sync(1, AM_CW * 32);
  float qsum[2][2];  // [row g / g+8][group]
#pragma unroll
  for (int hr = 0; hr < 2; ++hr)
#pragma unroll
    for (int G = 0; G < 2; ++G) qsum[hr][G] = qsum_s[(g + 8 * hr) * 2 + G];
  const int qp0 = qpos[g], qp8 = qpos[g + 8];
  const bool causal = a.mask_kind == M5_MASK_CAUSAL;

  float o[16][4];  // PV accumulators, dim-block db: rows g, g+8 x dims pv_dim(db, 2t / 2t+1)
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float vb_acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [row][group] sum p * vbias
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  // A timed-out wait ends this warp's key loop (its state stays as is) but the
  // warp still joins the merge barriers below.
  for (int it = 0; it < ntiles; ++it) {
    const int st = it % AM_STAGES;
    const uint32_t par = (it / AM_STAGES) & 1;
    if (!mbar_wait(&full[st], par, &g_attn_mma_err)) break;
    const unsigned char* sb = smem + st * LY::STAGE;
    const int kw0 = warp * 16;  // this warp's first key within the tile
    const int key_base = k_begin + it * AM_TK + kw0;

    // ---------------- S = Q K^T for two blocks of 8 keys
    float sc[2][4];
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      const int kl = kw0 + 8 * kb + g;  // key row this lane feeds as B column g
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
      // scale/bias per (key, group): keys 2t, 2t+1 of this block
      const int kk = kw0 + 8 * kb + 2 * t;
      const uint2 ks2 = *reinterpret_cast<const uint2*>(sb + LY::KS_OFF + kk * 4);  // [k][g0,g1],[k+1][g0,g1]
      const uint2 kb2 = *reinterpret_cast<const uint2*>(sb + LY::KB_OFF + kk * 4);
      const float s00 = bf16_lo(ks2.x), s01 = bf16_hi(ks2.x), s10 = bf16_lo(ks2.y), s11 = bf16_hi(ks2.y);
      const float b00 = bf16_lo(kb2.x), b01 = bf16_hi(kb2.x), b10 = bf16_lo(kb2.y), b11 = bf16_hi(kb2.y);
      // d[0]: (row g, key 2t) d[1]: (row g, key 2t+1) d[2]: (row g+8, 2t) d[3]: (row g+8, 2t+1)
      float s[4];
      s[0] = fmaf(s00, dG[0][0], b00 * qsum[0][0]) + fmaf(s01, dG[1][0], b01 * qsum[0][1]);
      s[1] = fmaf(s10, dG[0][1], b10 * qsum[0][0]) + fmaf(s11, dG[1][1], b11 * qsum[0][1]);
      s[2] = fmaf(s00, dG[0][2], b00 * qsum[1][0]) + fmaf(s01, dG[1][2], b01 * qsum[1][1]);
      s[3] = fmaf(s10, dG[0][3], b10 * qsum[1][0]) + fmaf(s11, dG[1][3], b11 * qsum[1][1]);
      const int key0 = key_base + 8 * kb + 2 * t;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = key0 + (i & 1);
        const int qp = (i < 2) ? qp0 : qp8;
        const bool valid = key < k_end && (!causal || key <= qp);
        sc[kb][i] = valid ? rbf(s[i]) : -INFINITY;
      }
    }

    // ---------------- online softmax (rows g and g+8; quads share a row)
    float pm[2];
    pm[0] = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    pm[1] = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
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
    float p[2][4];  // fp32 p, same layout as sc
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float mm = m_run[i >> 1];
        p[kb][i] = (sc[kb][i] == -INFINITY) ? 0.f : expf(sc[kb][i] - mm);
        l_run[i >> 1] += p[kb][i];
      }

    // ---------------- O += P V
    // value scale / bias of keys 2t, 2t+1 (block 0) and 8+2t, 8+2t+1 (block 1)
    const int vk0 = kw0 + 2 * t, vk1 = kw0 + 8 + 2 * t;
    const uint2 vs0 = *reinterpret_cast<const uint2*>(sb + LY::VS_OFF + vk0 * 4);
    const uint2 vs1 = *reinterpret_cast<const uint2*>(sb + LY::VS_OFF + vk1 * 4);
    const uint2 vb0 = *reinterpret_cast<const uint2*>(sb + LY::VB_OFF + vk0 * 4);
    const uint2 vb1 = *reinterpret_cast<const uint2*>(sb + LY::VB_OFF + vk1 * 4);
    uint32_t pa[2][4];  // A fragments per value group
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      // scales of keys (2t, 2t+1) for block 0 and block 1 in group G
      const float sA0 = G ? bf16_hi(vs0.x) : bf16_lo(vs0.x), sA1 = G ? bf16_hi(vs0.y) : bf16_lo(vs0.y);
      const float sB0 = G ? bf16_hi(vs1.x) : bf16_lo(vs1.x), sB1 = G ? bf16_hi(vs1.y) : bf16_lo(vs1.y);
      const float bA0 = G ? bf16_hi(vb0.x) : bf16_lo(vb0.x), bA1 = G ? bf16_hi(vb0.y) : bf16_lo(vb0.y);
      const float bB0 = G ? bf16_hi(vb1.x) : bf16_lo(vb1.x), bB1 = G ? bf16_hi(vb1.y) : bf16_lo(vb1.y);
      const float r00 = rbf(p[0][0]), r01 = rbf(p[0][1]), r02 = rbf(p[0][2]), r03 = rbf(p[0][3]);
      const float r10 = rbf(p[1][0]), r11 = rbf(p[1][1]), r12 = rbf(p[1][2]), r13 = rbf(p[1][3]);
      // masked keys have p == 0; their stage bytes may be stale, so never multiply them
      auto mul = [](float r, float x) { return r == 0.f ? 0.f : r * x; };
      pa[G][0] = pack_h2(mul(r00, sA0 * AM_PSCALE), mul(r01, sA1 * AM_PSCALE));  // row g, keys 2t, 2t+1
      pa[G][1] = pack_h2(mul(r02, sA0 * AM_PSCALE), mul(r03, sA1 * AM_PSCALE));  // row g+8
      pa[G][2] = pack_h2(mul(r10, sB0 * AM_PSCALE), mul(r11, sB1 * AM_PSCALE));  // row g, keys 8+2t, 8+2t+1
      pa[G][3] = pack_h2(mul(r12, sB0 * AM_PSCALE), mul(r13, sB1 * AM_PSCALE));  // row g+8
      vb_acc[0][G] += mul(r00, bA0) + mul(r01, bA1) + mul(r10, bB0) + mul(r11, bB1);
      vb_acc[1][G] += mul(r02, bA0) + mul(r03, bA1) + mul(r12, bB0) + mul(r13, bB1);
    }
    // V rows this lane feeds to movmatrix: key g of block 0 and of block 1,
    // 16 (8-bit) / 8 (4-bit) bytes per value group at offset 16t (8t).
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      uint32_t vw[2][4];
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        const int kl = kw0 + 8 * kb + g;
        if constexpr (BITS == 8) {
          const uint4 c = *reinterpret_cast<const uint4*>(sb + LY::V_OFF + kl * 128 + 64 * G + 16 * t);
          vw[kb][0] = c.x; vw[kb][1] = c.y; vw[kb][2] = c.z; vw[kb][3] = c.w;
        } else {
          const uint2 c = *reinterpret_cast<const uint2*>(sb + LY::V_OFF + kl * 64 + 32 * G + 8 * t);
          vw[kb][0] = c.x; vw[kb][1] = c.y; vw[kb][2] = 0; vw[kb][3] = 0;
        }
      }
#pragma unroll
      for (int dbl = 0; dbl < 8; ++dbl) {  // dim-block within the group
        uint32_t bb[2];
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint32_t pr;  // fp16 pair: this key, dims pv_dim(db, 2t), pv_dim(db, 2t+1)
          if constexpr (BITS == 8) {
            const uint32_t w = vw[kb][dbl >> 1];
            pr = (dbl & 1) ? code8_pair<0x4342>(w) : code8_pair<0x4140>(w);
          } else {
            // 4-bit: dims 16t + 2*dbl + {0,1} -> word dbl >> 2, nibbles (2*dbl) & 7, +1
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ---------------- reduce quad partials, merge the four warps
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
  named_sync(1, AM_CW * 32);  // all consumers are done with the stages: reuse them
  float* wm = reinterpret_cast<float*>(smem);       // [CW][16]
  float* wl = wm + AM_CW * 16;                      // [CW][16]
  float* wo = wl + AM_CW * 16;                      // [CW][16][128]
  if (t == 0) {
    wm[warp * 16 + g] = m_run[0];
    wm[warp * 16 + g + 8] = m_run[1];
    wl[warp * 16 + g] = l_run[0];
    wl[warp * 16 + g + 8] = l_run[1];
  }
#pragma unroll
  for (int db = 0; db < 16; ++db) {
    const int G = db >> 3, dbl = db & 7;
    // dims of columns 2t, 2t+1 of dim-block db (value permutation: 16t + 2 dbl + e within the group)
    const int d0 = 64 * G + 16 * t + 2 * dbl;
    wo[(warp * 16 + g) * 128 + d0] = o[db][0] / AM_PSCALE;
    wo[(warp * 16 + g) * 128 + d0 + 1] = o[db][1] / AM_PSCALE;
    wo[(warp * 16 + g + 8) * 128 + d0] = o[db][2] / AM_PSCALE;
    wo[(warp * 16 + g + 8) * 128 + d0 + 1] = o[db][3] / AM_PSCALE;
  }
  float* wvb = wo + AM_CW * 16 * 128;               // [CW][16][2]
  if (t == 0) {
    wvb[(warp * 16 + g) * 2 + 0] = vb_acc[0][0];
    wvb[(warp * 16 + g) * 2 + 1] = vb_acc[0][1];
    wvb[(warp * 16 + g + 8) * 2 + 0] = vb_acc[1][0];
    wvb[(warp * 16 + g + 8) * 2 + 1] = vb_acc[1][1];
  }
  named_sync(1, AM_CW * 32);
  for (int i = tid; i < rows * 128; i += AM_CW * 32) {
    const int r = i >> 7, d = i & 127;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AM_CW; ++w) M = fmaxf(M, wm[w * 16 + r]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < AM_CW; ++w) {
      const float mw = wm[w * 16 + r];
      if (mw == -INFINITY) continue;
      const float f = expf(mw - M);
      num = fmaf(f, wo[(w * 16 + r) * 128 + d] + wvb[(w * 16 + r) * 2 + (d >> 6)], num);
      den = fmaf(f, wl[w * 16 + r], den);
    }
    const int qi = q0 + r / rep, h = hk * rep + r % rep;
    const size_t orow = (size_t(b) * a.Hq + h) * a.L + qi;
    if (a.nsplit == 1) {
      const size_t od = a.out_tokens_major ? ((size_t(b) * a.L + qi) * a.Hq + h) : orow;
      a.out[od * 128 + d] = f2bf(num / fmaxf(den, 1e-30f));
    } else {
      a.part_o[(orow * a.nsplit + split) * 128 + d] = num;
      if (d == 0) {
        a.part_ml[(orow * a.nsplit + split) * 2 + 0] = M;
        a.part_ml[(orow * a.nsplit + split) * 2 + 1] = den;
      }
    }
  }
}

static size_t am_smem(int bits) {
  const size_t stage = bits == 8 ? AmLayout<8>::STAGE : AmLayout<4>::STAGE;
  const size_t main = AM_STAGES * stage;
  const size_t merge = size_t(AM_CW) * 16 * (2 + 128 + 2) * 4;
  return std::max(main, merge) + 2 * AM_STAGES * 8 + 16 * 128 * 4 + 16 * 4 + 32 * 4;
}

bool attn_mma_eligible(const AttnArgs& a) {
  if (a.D != 128 || (a.bits != 8 && a.bits != 4)) return false;
  if (a.mask_kind != M5_MASK_NONE && a.mask_kind != M5_MASK_CAUSAL) return false;
  if (a.QB * (a.Hq / a.Hkv) > 16) return false;
  const int krow = 128 * a.bits / 8;
  // 16-byte aligned bulk copies: row bases and scale rows (4 bytes per key).
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.k.data) || !al(a.v.data) || !al(a.k.scales) || !al(a.k.biases) || !al(a.v.scales) || !al(a.v.biases))
    return false;
  if ((a.k.head_stride % 4) || (a.v.head_stride % 4) || (a.k.batch_stride % 4) || (a.v.batch_stride % 4))
    return false;
  // a tile copy may read up to 3 rows past the last key (whole 16-byte scale
  // rows): they must lie inside the head's rows
  if (!a.d_S) {
    const long long s4 = (a.S_host + 3LL) / 4 * 4;
    if (s4 > a.k.head_stride || s4 > a.v.head_stride) return false;
  }
  (void)krow;
  return true;
}

int attn_mma_launch(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = am_smem(a.bits);
  static bool conf8 = false, conf4 = false;
  dim3 grid(a.nsplit, (a.L + a.QB - 1) / a.QB, a.B * a.Hkv);
  if (a.bits == 8) {
    if (!conf8) {
      M5_CUDA(cudaFuncSetAttribute(attn_mma_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      conf8 = true;
    }
    M5_CUDA(launch_pdl(attn_mma_kernel<8>, dim3(grid), dim3(AM_THREADS), smem, stream, a));
  } else {
    if (!conf4) {
      M5_CUDA(cudaFuncSetAttribute(attn_mma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      conf4 = true;
    }
    M5_CUDA(launch_pdl(attn_mma_kernel<4>, dim3(grid), dim3(AM_THREADS), smem, stream, a));
  }
  M5_LAUNCH_CHECK("attention (tensor core) launch");
  return M5_OK;
}

int attn_mma_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_mma_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_mma_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
