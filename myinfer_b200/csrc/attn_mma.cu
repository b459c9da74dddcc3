// Split-KV flash decoding over an 8/4-bit KV cache on the tensor cores
// (kernel K4, rows = GQA group x queries <= 16).
//
// Work of one CTA: one kv head, one contiguous key range (a split).  A
// producer warp streams 64-key tiles of K, V and their bf16 scales/biases
// with 1-D bulk copies (each head's rows are contiguous) into a shared-memory
// ring guarded by mbarriers (bounded waits): 3 stages and 3 CTAs per SM for
// one 8-row block of queries (decode), 4 stages and 2 CTAs for two.  Four
// consumer warps take 16 keys of every tile each and keep their own
// online-softmax state; the states are merged at the end of the split.
//
// The MMAs run transposed, keys (and value dims) as the 16-row M side and the
// query rows as the 8-column N side, so a GQA group of 8 heads fills an MMA
// and nothing is padded.  Per 16-key step of a consumer warp (mma.sync
// m16n8k16, fp16 in, fp32 acc):
//   S^T = K Q^T : A = K codes (a code becomes an fp16 operand with one PRMT
//               per two codes, byte | 0x6400 = 1024 + code, and one HSUB2),
//               B = q^T (scaled by `scale` and rounded to bf16 like
//               attention.py:49; exact in fp16).  Contraction dims are
//               permuted so a lane reads 16 contiguous code bytes per 64-dim
//               group, and every MMA stays inside one scale group, so
//               s = sum_g scale_g * (q . code_g) + bias_g * sum(q_g)
//               is the reference's dequantized dot product.
//   scores rounded to bf16 (attention.py:66-69), fp32 online softmax; p rounded
//   to bf16 for PV (attention.py:87-90), fp32 p in the denominator.
//   O^T += V^T P^T : A = V codes, 8 dims x 2 keys per lane built with byte
//               permutes across two key rows; B = p * vscale_g * 2^6 (fp16, one
//               per scale group), moved from the score layout with one
//               movmatrix per 8 keys; the per-key value bias adds p * vbias_g
//               to an fp32 side sum.
#include <algorithm>
#include <cmath>

#include "attn.cuh"
#include "tma.cuh"

namespace m5 {

static __device__ int g_attn_mma_err = 0;

constexpr int AM_TK = 64;       // keys per stage
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

// Integer MMAs for S^T = K Q^T: u8 key codes against the s8 high and u8 low
// planes of the 16-bit fixed-point queries; exact int32 sums.
__device__ __forceinline__ void am_imma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void am_imma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Physical dim of byte e (0..3) of the A register `half` (0: a0/a1, 1: a2/a3)
// in k32 step j of group G for lane quad t, as the int8 S path reads the
// codes: 8-bit rows give a lane 16 contiguous bytes per group (words 2j,
// 2j+1); 4-bit rows 8 bytes per group, word j split into its even-dim (low
// nibble) and odd-dim (high nibble) codes.
template <int BITS>
__device__ __forceinline__ int i8s_dim(int G, int t, int j, int half, int e) {
  if constexpr (BITS == 8) return 64 * G + 16 * t + 8 * j + 4 * half + e;
  else return 64 * G + 16 * t + 8 * j + 2 * e + half;
}

// S^T on integer MMAs (no code conversion) instead of fp16 MMAs on codes
// converted in registers (decode: one 8-row block of query rows).
constexpr bool AM_I8S = true;

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

// fp16 pair x / 16 - 64: (1024 + 16 c) -> c exactly (4-bit codes in the high nibble)
__device__ __forceinline__ uint32_t hsixteenth(uint32_t x) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(0x2C002C00u), "r"(0xD400D400u));
  return r;
}

// 2^x (ex2.approx; -inf gives 0).  exp(x) is taken as 2^(x log2 e): relative
// error ~1e-6, far below the bf16 rounding p goes through.
__device__ __forceinline__ float am_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float AM_LOG2E = 1.4426950408889634f;

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

// Stages of the ring and CTAs per SM: one 8-row block of queries (decode)
// keeps three CTAs of 4 + 1 warps resident per SM, two blocks two CTAs.
template <int NB>
struct AmCfg {
  static constexpr int STAGES = NB == 1 ? 3 : 4;
  static constexpr int MINB = NB == 1 ? 3 : 2;
};

template <int BITS, int NB>
__global__ void __launch_bounds__(AM_THREADS, AmCfg<NB>::MINB) attn_mma_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  using LY = AmLayout<BITS>;
  // integer S for one 8-row block (two blocks would spill at 2 CTAs per SM)
  constexpr bool I8S = AM_I8S && NB == 1;
  constexpr int STAGES = AmCfg<NB>::STAGES;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * LY::STAGE);
  uint64_t* empty = full + STAGES;
  float* q_s = reinterpret_cast<float*>(empty + STAGES);  // [16][128] scaled, bf16-rounded q
  int* qpos = reinterpret_cast<int*>(q_s + 16 * 128);     // [16]

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
    for (int s = 0; s < STAGES; ++s) {
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
        const int st = it % STAGES;
        const uint32_t par = (it / STAGES) & 1;
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
  // stage scaled q (bf16-rounded) for the 16 MMA columns; padding rows are zero.
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

  // per-(row, group) sums of q: 4 threads x 16 elements per (row, group)
  float* qsum_s = reinterpret_cast<float*>(qpos + 16);  // [16][2]
  float* qxs_s = qsum_s + 32;                           // [16] 2^-sh of a row's fixed-point planes
  if constexpr (I8S) {
    // Each query row becomes 16-bit fixed point v = rint(q * 2^sh), sh set by
    // the row's largest |q| so |v| < 2^15 (every value at or above 2^-7 of
    // the row's maximum exact: q is bf16), split into an s8 high and a u8 low
    // plane; 8 threads per row.
    const int r = tid >> 3, part = tid & 7;
    const float4* src = reinterpret_cast<const float4*>(q_s + r * 128 + part * 16);
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 f = src[k];
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    if (part == 0) {
      const int E = int((__float_as_uint(mx) >> 23) & 0xFFu);
      const int sh = mx > 0.f ? 141 - E : 0;
      qxs_s[r] = __uint_as_float(uint32_t(max(1, min(254, 127 - sh))) << 23);
    }
  }
  // B fragments of q^T: column g of n-block nb is query row g + 8 nb, the
  // contraction dims permuted as the K codes are read.  fp16 path: 8 k16
  // slices; int8 path: per group and k32 step, the high and low planes.
  uint32_t qb[NB][8][2];
  if constexpr (!I8S) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d0 = qk_dim<BITS>(j, t, 2 * t), d1 = qk_dim<BITS>(j, t, 2 * t + 1);
      const int d8 = qk_dim<BITS>(j, t, 2 * t + 8), d9 = qk_dim<BITS>(j, t, 2 * t + 9);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const float* r = q_s + (g + 8 * nb) * 128;
        qb[nb][j][0] = pack_h2(r[d0], r[d1]);
        qb[nb][j][1] = pack_h2(r[d8], r[d9]);
      }
    }
  }
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
  if constexpr (I8S) {
    // planes of this lane's B fragments: qb[nb][4 G + 2 j + plane][b0 / b1]
    // (plane 0 high, 1 low); v + 2^22 sits in the low mantissa bits of
    // fma(q, 2^sh, 1.5 * 2^23), byte 0 its low byte, byte 1 its high byte
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int r = g + 8 * nb;
      const float* qr = q_s + r * 128;
      const float up = 1.f / qxs_s[r];
#pragma unroll
      for (int G = 0; G < 2; ++G)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t f[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) f[e] = __float_as_uint(fmaf(qr[i8s_dim<BITS>(G, t, j, hf, e)], up, 12582912.f));
            qb[nb][4 * G + 2 * j + 0][hf] =
                __byte_perm(__byte_perm(f[0], f[1], 0x0051), __byte_perm(f[2], f[3], 0x0051), 0x5410);
            qb[nb][4 * G + 2 * j + 1][hf] =
                __byte_perm(__byte_perm(f[0], f[1], 0x0040), __byte_perm(f[2], f[3], 0x0040), 0x5410);
          }
    }
  }
  // this lane's score columns: rows 2t + e + 8 nb
  float qsr[NB][2][2];  // [nb][e][group]
  float qxr[NB][2];     // [nb][e] 2^-sh of the row's planes (int8 S path)
  int qp[NB][2];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = 2 * t + e + 8 * nb;
      qsr[nb][e][0] = qsum_s[r * 2];
      qsr[nb][e][1] = qsum_s[r * 2 + 1];
      qxr[nb][e] = I8S ? qxs_s[r] : 1.f;
      qp[nb][e] = qpos[r];
    }
  const bool causal = a.mask_kind == M5_MASK_CAUSAL;
  const int qp_first = S - a.L + q0;  // position of the CTA's first query

  // O^T accumulators: block (G, jj) rows g / g+8 are dims 64G + 8g + 2jj (+1),
  // columns 2t, 2t+1 are query rows 2t + 8nb, 2t + 1 + 8nb
  float o[NB][8][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int i = 0; i < 8; ++i) o[nb][i][0] = o[nb][i][1] = o[nb][i][2] = o[nb][i][3] = 0.f;
  float vb_acc[NB][2][2];  // [nb][e][group] sum p * vbias over this lane's keys
  float m_run[NB][2], l_run[NB][2];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      vb_acc[nb][e][0] = vb_acc[nb][e][1] = 0.f;
      m_run[nb][e] = -INFINITY;
      l_run[nb][e] = 0.f;
    }

  // A timed-out wait ends this warp's key loop (its state stays as is) but the
  // warp still joins the merge barriers below.
  for (int it = 0; it < ntiles; ++it) {
    const int st = it % STAGES;
    const uint32_t par = (it / STAGES) & 1;
    if (!mbar_wait(&full[st], par, &g_attn_mma_err)) break;
    const unsigned char* sb = smem + st * LY::STAGE;
    const int kw0 = warp * 16;  // this warp's first key within the tile
    const int key_base = k_begin + it * AM_TK + kw0;

    // ---------------- S^T = K Q^T: A rows g / g+8 are keys kw0 + g / kw0 + 8 + g
    float dG[NB][2][4];
    int dh[NB][2][4], dl[NB][2][4];  // int8 path: high / low plane sums per group
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int G = 0; G < 2; ++G)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dG[nb][G][i] = 0.f;
          dh[nb][G][i] = dl[nb][G][i] = 0;
        }
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      if constexpr (I8S) {
        // the codes are the A operand as they lie: 8-bit rows 16 bytes per
        // lane and group, 4-bit rows 8 bytes split into even / odd dims
        uint32_t A[2][4];  // [k32 step j]
        if constexpr (BITS == 8) {
          const uint4 c0 = *reinterpret_cast<const uint4*>(sb + LY::K_OFF + (kw0 + g) * 128 + 64 * G + 16 * t);
          const uint4 c1 = *reinterpret_cast<const uint4*>(sb + LY::K_OFF + (kw0 + 8 + g) * 128 + 64 * G + 16 * t);
          A[0][0] = c0.x;
          A[0][1] = c1.x;
          A[0][2] = c0.y;
          A[0][3] = c1.y;
          A[1][0] = c0.z;
          A[1][1] = c1.z;
          A[1][2] = c0.w;
          A[1][3] = c1.w;
        } else {
          const uint2 c0 = *reinterpret_cast<const uint2*>(sb + LY::K_OFF + (kw0 + g) * 64 + 32 * G + 8 * t);
          const uint2 c1 = *reinterpret_cast<const uint2*>(sb + LY::K_OFF + (kw0 + 8 + g) * 64 + 32 * G + 8 * t);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t wa = j ? c0.y : c0.x, wb = j ? c1.y : c1.x;
            A[j][0] = wa & 0x0F0F0F0Fu;
            A[j][1] = wb & 0x0F0F0F0Fu;
            A[j][2] = (wa >> 4) & 0x0F0F0F0Fu;
            A[j][3] = (wb >> 4) & 0x0F0F0F0Fu;
          }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            am_imma_s8(dh[nb][G], A[j], qb[nb][4 * G + 2 * j][0], qb[nb][4 * G + 2 * j][1]);
            am_imma_u8(dl[nb][G], A[j], qb[nb][4 * G + 2 * j + 1][0], qb[nb][4 * G + 2 * j + 1][1]);
          }
      } else if constexpr (BITS == 8) {
        const uint4 c0 = *reinterpret_cast<const uint4*>(sb + LY::K_OFF + (kw0 + g) * 128 + 64 * G + 16 * t);
        const uint4 c1 = *reinterpret_cast<const uint4*>(sb + LY::K_OFF + (kw0 + 8 + g) * 128 + 64 * G + 16 * t);
        const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w}, w1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const uint32_t A[4] = {code8_pair<0x4140>(w0[sub]), code8_pair<0x4140>(w1[sub]),
                                 code8_pair<0x4342>(w0[sub]), code8_pair<0x4342>(w1[sub])};
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) mma_f16(dG[nb][G], A, qb[nb][4 * G + sub][0], qb[nb][4 * G + sub][1]);
        }
      } else {
        const uint2 c0 = *reinterpret_cast<const uint2*>(sb + LY::K_OFF + (kw0 + g) * 64 + 32 * G + 8 * t);
        const uint2 c1 = *reinterpret_cast<const uint2*>(sb + LY::K_OFF + (kw0 + 8 + g) * 64 + 32 * G + 8 * t);
        const uint32_t w0[2] = {c0.x, c0.y}, w1[2] = {c1.x, c1.y};
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int i0 = 2 * (sub & 1);
          const uint32_t A[4] = {code4_pair(w0[sub >> 1], i0), code4_pair(w1[sub >> 1], i0),
                                 code4_pair(w0[sub >> 1], i0 + 1), code4_pair(w1[sub >> 1], i0 + 1)};
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) mma_f16(dG[nb][G], A, qb[nb][4 * G + sub][0], qb[nb][4 * G + sub][1]);
        }
      }
    }
    // key scale/bias of keys g (fragments 0,1) and 8 + g (fragments 2,3), both groups
    const uint32_t ksA = *reinterpret_cast<const uint32_t*>(sb + LY::KS_OFF + (kw0 + g) * 4);
    const uint32_t ksB = *reinterpret_cast<const uint32_t*>(sb + LY::KS_OFF + (kw0 + 8 + g) * 4);
    const uint32_t kbA = *reinterpret_cast<const uint32_t*>(sb + LY::KB_OFF + (kw0 + g) * 4);
    const uint32_t kbB = *reinterpret_cast<const uint32_t*>(sb + LY::KB_OFF + (kw0 + 8 + g) * 4);
    const float sk[2][2] = {{bf16_lo(ksA), bf16_hi(ksA)}, {bf16_lo(ksB), bf16_hi(ksB)}};
    const float bk[2][2] = {{bf16_lo(kbA), bf16_hi(kbA)}, {bf16_lo(kbB), bf16_hi(kbB)}};
    const int keyA = key_base + g, keyB = key_base + 8 + g;
    // a tile that reaches past the range end or across the causal diagonal
    // masks per key and row; inside ones skip the tests (warp-uniform)
    const int tile_end = k_begin + (it + 1) * AM_TK;
    const bool edge = tile_end > k_end || (causal && tile_end - 1 > qp_first);
    float sc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kk = i >> 1, e = i & 1;
        float s;
        if constexpr (I8S) {
          // exact: |256 dh + dl| < 2^30 (64 codes <= 255 times |v| < 2^15)
          const float a0 = float(dh[nb][0][i] * 256 + dl[nb][0][i]);
          const float a1 = float(dh[nb][1][i] * 256 + dl[nb][1][i]);
          s = fmaf(qxr[nb][e], fmaf(sk[kk][0], a0, sk[kk][1] * a1),
                   fmaf(bk[kk][0], qsr[nb][e][0], bk[kk][1] * qsr[nb][e][1]));
        } else {
          s = fmaf(sk[kk][0], dG[nb][0][i], bk[kk][0] * qsr[nb][e][0]) +
              fmaf(sk[kk][1], dG[nb][1][i], bk[kk][1] * qsr[nb][e][1]);
        }
        sc[nb][i] = rbf(s);
        if (edge) {
          const int key = kk ? keyB : keyA;
          if (!(key < k_end && (!causal || key <= qp[nb][e]))) sc[nb][i] = -INFINITY;
        }
      }

    // ---------------- online softmax: column (row) maxima over the 8 key lanes
    float p[NB][4];
    bool changed = false;
    float corr[NB][2];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float pm = fmaxf(sc[nb][e], sc[nb][2 + e]);
        pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 4));
        pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
        pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 16));
        const float mn = fmaxf(m_run[nb][e], pm);
        corr[nb][e] = (m_run[nb][e] == mn) ? 1.f : (m_run[nb][e] == -INFINITY ? 0.f : am_ex2((m_run[nb][e] - mn) * AM_LOG2E));
        changed |= corr[nb][e] != 1.f;
        m_run[nb][e] = mn;
      }
    if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[nb][i][0] *= corr[nb][0];
          o[nb][i][1] *= corr[nb][1];
          o[nb][i][2] *= corr[nb][0];
          o[nb][i][3] *= corr[nb][1];
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          vb_acc[nb][e][0] *= corr[nb][e];
          vb_acc[nb][e][1] *= corr[nb][e];
          l_run[nb][e] *= corr[nb][e];
        }
      }
    }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      float ml[2];  // m log2 e (0 while a row has seen no key: its scores are -inf and p = 0)
#pragma unroll
      for (int e = 0; e < 2; ++e) ml[e] = m_run[nb][e] == -INFINITY ? 0.f : m_run[nb][e] * AM_LOG2E;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        p[nb][i] = am_ex2(fmaf(sc[nb][i], AM_LOG2E, -ml[i & 1]));
        l_run[nb][i & 1] += p[nb][i];
      }
    }

    // ---------------- O^T += V^T P^T
    uint32_t vsA = *reinterpret_cast<const uint32_t*>(sb + LY::VS_OFF + (kw0 + g) * 4);
    uint32_t vsB = *reinterpret_cast<const uint32_t*>(sb + LY::VS_OFF + (kw0 + 8 + g) * 4);
    uint32_t vbA = *reinterpret_cast<const uint32_t*>(sb + LY::VB_OFF + (kw0 + g) * 4);
    uint32_t vbB = *reinterpret_cast<const uint32_t*>(sb + LY::VB_OFF + (kw0 + 8 + g) * 4);
    // keys past the range end have p == 0 but stale stage bytes (possibly NaN
    // scales): their scales become 0 so no product with them is formed
    if (edge) {
      if (keyA >= k_end) vsA = vbA = 0u;
      if (keyB >= k_end) vsB = vbB = 0u;
    }
    auto mul = [](float r, float x) { return r * x; };
    // B fragments per value group: p * vscale * 2^6 of this lane's keys, moved
    // to the (keys 2t, 2t+1 ; row g) layout with one transpose per 8 keys
    uint32_t pb[NB][2][2];  // [nb][group][b0 / b1]
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const float r0 = rbf(p[nb][0]), r1 = rbf(p[nb][1]), r2 = rbf(p[nb][2]), r3 = rbf(p[nb][3]);
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        const float sA = (G ? bf16_hi(vsA) : bf16_lo(vsA)) * AM_PSCALE;
        const float sB = (G ? bf16_hi(vsB) : bf16_lo(vsB)) * AM_PSCALE;
        const float bA = G ? bf16_hi(vbA) : bf16_lo(vbA), bB = G ? bf16_hi(vbB) : bf16_lo(vbB);
        pb[nb][G][0] = movmatrix_t(pack_h2(mul(r0, sA), mul(r1, sA)));
        pb[nb][G][1] = movmatrix_t(pack_h2(mul(r2, sB), mul(r3, sB)));
        vb_acc[nb][0][G] += mul(r0, bA) + mul(r2, bB);
        vb_acc[nb][1][G] += mul(r1, bA) + mul(r3, bB);
      }
    }
    // V codes of keys 2t, 2t+1, 8+2t, 8+2t+1 at dims 64G + 8g .. +7
    const int kv0 = kw0 + 2 * t, kv8 = kw0 + 8 + 2 * t;
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      if constexpr (BITS == 8) {
        const unsigned char* vrow = sb + LY::V_OFF + 64 * G + 8 * g;
        const uint2 v0 = *reinterpret_cast<const uint2*>(vrow + kv0 * 128);
        const uint2 v1 = *reinterpret_cast<const uint2*>(vrow + (kv0 + 1) * 128);
        const uint2 v8 = *reinterpret_cast<const uint2*>(vrow + kv8 * 128);
        const uint2 v9 = *reinterpret_cast<const uint2*>(vrow + (kv8 + 1) * 128);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          // bytes 2jj, 2jj+1 of the 8 (dims 2jj, 2jj+1): [key a, key b] x 2 dims
          const int wd = jj >> 1;
          const uint32_t sel = (jj & 1) ? 0x7362u : 0x5140u;  // [a.b, b.b, a.b+1, b.b+1]
          const uint32_t x01 = __byte_perm(wd ? v0.y : v0.x, wd ? v1.y : v1.x, sel);
          const uint32_t x89 = __byte_perm(wd ? v8.y : v8.x, wd ? v9.y : v9.x, sel);
          const uint32_t A[4] = {code8_pair<0x4140>(x01), code8_pair<0x4342>(x01), code8_pair<0x4140>(x89),
                                 code8_pair<0x4342>(x89)};
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) mma_f16(o[nb][4 * G + jj], A, pb[nb][G][0], pb[nb][G][1]);
        }
      } else {
        const unsigned char* vrow = sb + LY::V_OFF + 32 * G + 4 * g;
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(vrow + kv0 * 64);
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(vrow + (kv0 + 1) * 64);
        const uint32_t v8 = *reinterpret_cast<const uint32_t*>(vrow + kv8 * 64);
        const uint32_t v9 = *reinterpret_cast<const uint32_t*>(vrow + (kv8 + 1) * 64);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          // byte jj holds dims 2jj (low nibble) and 2jj+1 (high nibble)
          const uint32_t sel = uint32_t(jj) | (uint32_t(4 + jj) << 8);  // [a.jj, -, b.jj, -]
          const uint32_t y01 = __byte_perm(v0, v1, sel), y89 = __byte_perm(v8, v9, sel);
          const uint32_t A[4] = {hsub1024((y01 & 0x000F000Fu) | 0x64006400u),
                                 hsixteenth((y01 & 0x00F000F0u) | 0x64006400u),
                                 hsub1024((y89 & 0x000F000Fu) | 0x64006400u),
                                 hsixteenth((y89 & 0x00F000F0u) | 0x64006400u)};
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) mma_f16(o[nb][4 * G + jj], A, pb[nb][G][0], pb[nb][G][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // ---------------- reduce over the 8 key lanes, merge the four warps
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
#pragma unroll
      for (int o_ = 4; o_ <= 16; o_ <<= 1) {
        l_run[nb][e] += __shfl_xor_sync(0xffffffffu, l_run[nb][e], o_);
        vb_acc[nb][e][0] += __shfl_xor_sync(0xffffffffu, vb_acc[nb][e][0], o_);
        vb_acc[nb][e][1] += __shfl_xor_sync(0xffffffffu, vb_acc[nb][e][1], o_);
      }
    }
  named_sync(1, AM_CW * 32);  // all consumers are done with the stages: reuse them
  float* wm = reinterpret_cast<float*>(smem);       // [CW][16]
  float* wl = wm + AM_CW * 16;                      // [CW][16]
  float* wo = wl + AM_CW * 16;                      // [CW][16][128]
  float* wvb = wo + AM_CW * 16 * 128;               // [CW][16][2]
  if (g == 0) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = 2 * t + e + 8 * nb;
        wm[warp * 16 + r] = m_run[nb][e];
        wl[warp * 16 + r] = l_run[nb][e];
        wvb[(warp * 16 + r) * 2 + 0] = vb_acc[nb][e][0];
        wvb[(warp * 16 + r) * 2 + 1] = vb_acc[nb][e][1];
      }
  }
  if (NB == 1) {  // rows 8..15 are unused: mark them empty
    if (lane < 8) {
      wm[warp * 16 + 8 + lane] = -INFINITY;
      wl[warp * 16 + 8 + lane] = 0.f;
    }
  }
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int G = 0; G < 2; ++G)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int d = 64 * G + 8 * g + 2 * jj;
        const int r0 = 2 * t + 8 * nb;
        const float* ob = o[nb][4 * G + jj];
        wo[(warp * 16 + r0) * 128 + d] = ob[0] / AM_PSCALE;
        wo[(warp * 16 + r0 + 1) * 128 + d] = ob[1] / AM_PSCALE;
        wo[(warp * 16 + r0) * 128 + d + 1] = ob[2] / AM_PSCALE;
        wo[(warp * 16 + r0 + 1) * 128 + d + 1] = ob[3] / AM_PSCALE;
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

static size_t am_smem(int bits, int nb) {
  const size_t stage = bits == 8 ? AmLayout<8>::STAGE : AmLayout<4>::STAGE;
  const int stages = nb == 1 ? AmCfg<1>::STAGES : AmCfg<2>::STAGES;
  const size_t main = stages * stage;
  const size_t merge = size_t(AM_CW) * 16 * (2 + 128 + 2) * 4;
  return std::max(main, merge) + 2 * stages * 8 + 16 * 128 * 4 + 16 * 4 + 32 * 4 + 16 * 4;
}

int attn_mma_rows(const AttnArgs& a) { return std::min(a.QB, a.L) * (a.Hq / a.Hkv); }
int attn_mma_ctas_per_sm(int rows) { return rows <= 8 ? AmCfg<1>::MINB : AmCfg<2>::MINB; }

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

template <int BITS, int NB>
static int am_launch_t(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = am_smem(BITS, NB);
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(attn_mma_kernel<BITS, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); }));
  dim3 grid(a.nsplit, (a.L + a.QB - 1) / a.QB, a.B * a.Hkv);
  M5_CUDA(launch_pdl(attn_mma_kernel<BITS, NB>, dim3(grid), dim3(AM_THREADS), smem, stream, a));
  return M5_OK;
}

int attn_mma_launch(const AttnArgs& a, cudaStream_t stream) {
  const bool one = attn_mma_rows(a) <= 8;
  int rc;
  if (a.bits == 8) rc = one ? am_launch_t<8, 1>(a, stream) : am_launch_t<8, 2>(a, stream);
  else rc = one ? am_launch_t<4, 1>(a, stream) : am_launch_t<4, 2>(a, stream);
  if (rc) return rc;
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
