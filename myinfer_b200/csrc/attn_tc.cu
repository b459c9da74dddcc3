// Prefill flash attention over an 8/4-bit KV cache on the fifth-generation
// tensor cores (kernel K4p, tcgen05 + TMEM): chunks of L queries, rows = GQA
// group x queries = 128 per CTA, one kv head and one key range per CTA.
//
// Roles (one CTA per SM, 448 threads):
//   warp 13     producer: 1-D bulk copies of 64-key tiles of packed K / V and
//               their bf16 scales / biases into a 3-stage ring;
//   warps 8-11  dequant, into one of two operand buffers: K codes as exact
//               fp16 in the 128-byte-swizzled K-major layout the MMA reads
//               ([key][dim], one 64-dim scale group per operand), K's scales
//               and biases as fp32 beside them, and V dequantized,
//               fp16(code * vscale + vbias), transposed to [dim][key];
//   warp 12     MMA issuer (one thread): per tile
//                 S_g[128 x 64 keys] = Q_g (TMEM, fp16) * Kcodes_g^T   (g = 0, 1)
//               into one of two S buffers, and after the softmax
//                 O[128 x 128] += P (TMEM, fp16) * V                  (4 MMAs)
//   warps 0-7   softmax: warps w and w + 4 share TMEM lanes 32 (w & 3) ..,
//               i.e. 32 query rows, and take keys 0-31 / 32-63 of each tile.
//               Per key
//                 s = rb(kscale_0 S_0 + kscale_1 S_1 + kbias_0 sum(q_0) + kbias_1 sum(q_1))
//               (the dequantized dot product, rounded to bf16 like
//               attention.py:66-69), causal / range mask on boundary tiles,
//               the row max exchanged between the two warps, fp32 online
//               softmax, p rounded to bf16 for PV (attention.py:87-90) and
//               stored as fp16 (exact), fp32 p in the denominator; O in TMEM
//               is rescaled in place when a row's max moves.
// exp(x) is evaluated as 2^(x log2 e) (ex2.approx): relative error ~1e-6,
// far below the bf16 rounding of p.  V in fp16 carries a relative rounding
// of 2^-12 per element, like the fp16 p * vscale of the mma.sync kernel.
// TMEM columns: S buffers [0,128) [128,256) (group g at +64g), O [256,384),
// Q [384,448) (fp16 pairs), P buffers [448,480) [480,512).  Every mbarrier
// wait is bounded; a timeout sets a CTA-wide failure flag that ends every
// role, records a device error and still frees TMEM.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "attn.cuh"
#include "tcgen05.cuh"

namespace m5 {

static __device__ int g_attn_tc_err = 0;

namespace atc {

constexpr int TK = 64;            // keys per tile
constexpr int STAGES = 3;         // packed ring
constexpr int ROWS = 128;         // query rows per CTA (MMA M)
constexpr int SMX_WARPS = 8, DQ_WARPS = 4;
constexpr int MMA_WARP = SMX_WARPS + DQ_WARPS, PROD_WARP = MMA_WARP + 1;
constexpr int THREADS = (PROD_WARP + 1) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0, O_COL = 256, Q_COL = 384, P_COL = 448;
constexpr float LOG2E = 1.4426950408889634f;

template <int BITS>
struct Packed {  // one ring stage: K codes, K scales, K biases, V codes, V scales, V biases
  static constexpr int KROW = 128 * BITS / 8;
  static constexpr int K_OFF = 0;
  static constexpr int KS_OFF = K_OFF + TK * KROW;
  static constexpr int KB_OFF = KS_OFF + TK * 4;
  static constexpr int V_OFF = KB_OFF + TK * 4;
  static constexpr int VS_OFF = V_OFF + TK * KROW;
  static constexpr int VB_OFF = VS_OFF + TK * 4;
  static constexpr int STAGE = (VB_OFF + TK * 4 + 1023) / 1024 * 1024;
};

// fp16 operand buffer (two per CTA): K codes of groups 0 / 1 (8 KB each: 64
// keys x 128 bytes, 128-byte swizzle), V [128 dims x 64 keys] (16 KB, same
// swizzle), then float4 (kscale_0, kscale_1, kbias_0, kbias_1) per key.
constexpr int OP_BYTES = 8192;
constexpr int OP_K = 0, OP_V = 2 * OP_BYTES;
constexpr int SB_OFF = 4 * OP_BYTES;
constexpr int OPBUF = SB_OFF + TK * 16;

template <int BITS, int OPB>
constexpr size_t smem_bytes() {
  return 1024 + size_t(STAGES) * Packed<BITS>::STAGE + OPB * size_t(OPBUF) + 512;
}

// Byte offset of 16-byte chunk j of row n in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128(int n, int j) {
  return uint32_t((n >> 3) * 1024 + (n & 7) * 128 + ((j ^ (n & 7)) << 4));
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
// fp16 pair of the 8-bit codes at bytes (i, i + 1) of w, exactly
__device__ __forceinline__ uint32_t c8(uint32_t w, int i) {
  return hsub1024(__byte_perm(w, 0x64u, i == 0 ? 0x4140 : 0x4342));
}
// fp16 pair of two 4-bit / 8-bit codes given as small integers
__device__ __forceinline__ uint32_t cpair(uint32_t lo, uint32_t hi) {
  return hsub1024(0x64006400u | lo | (hi << 16));
}
// fp16 pair a * b + c, one rounding
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// 2^x (ex2.approx; -inf gives 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Instruction descriptor of kind::f16 with fp16 A and B (K-major), fp32 D.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ uint64_t atc_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes (or the hint runs out) instead of issuing poll instructions that
// take slots from the working warps of its sub-partition.
__device__ __forceinline__ bool try_wait_hint(uint64_t* bar, uint32_t par, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(par), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait by one thread (~2 s), failure shared through `fail`.
// hint_ns = 0 polls without suspending.
__device__ __forceinline__ bool wait1(uint64_t* bar, uint32_t par, volatile int* fail, uint32_t hint_ns) {
  if (mbar_try_wait_fast(bar, par)) return true;
  const uint64_t t0 = atc_now();
  for (uint32_t i = 1;; ++i) {
    if (hint_ns ? try_wait_hint(bar, par, hint_ns) : mbar_try_wait_fast(bar, par)) return true;
    if (*fail) return false;
    if ((hint_ns || (i & 255) == 0) && atc_now() - t0 > 2000000000ull) break;
  }
  *fail = 1;
  atomicExch(&g_attn_tc_err, M5_DEV_ERR_WAIT_TIMEOUT);
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

__device__ __forceinline__ float max32(const float (&x)[32]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(fmaxf(x[i], x[i + 8]), fmaxf(x[i + 16], x[i + 24]));
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[i], m[i + 4]);
  return fmaxf(fmaxf(m[0], m[2]), fmaxf(m[1], m[3]));
}
__device__ __forceinline__ float sum32(const float (&x)[32]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = (x[i] + x[i + 8]) + (x[i + 16] + x[i + 24]);
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] += m[i + 4];
  return (m[0] + m[2]) + (m[1] + m[3]);
}

// OPB operand buffers: dequant runs up to OPB - 1 tiles ahead of the PV that
// frees a buffer.
template <int BITS, int OPB>
__global__ void __launch_bounds__(THREADS, 1) attn_tc_kernel(const AttnArgs a, const uint32_t hint_ns) {
  using PK = Packed<BITS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;
  uint8_t* opb = ring + size_t(STAGES) * PK::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(opb + OPB * size_t(OPBUF));
  uint64_t* full = bars;
  uint64_t* empty = full + STAGES;
  uint64_t* op_full = empty + STAGES;
  uint64_t* op_empty = op_full + OPB;
  uint64_t* s_full = op_empty + OPB;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* q_ready = pv_done + 1;
  uint64_t* mma_idle = q_ready + 1;
  uint64_t* xbar = mma_idle + 1;  // [4 row quarters][2 tile parities]: the two warps' row maxima
  uint64_t* xend = xbar + 8;      // [4]: the two warps' denominators
  __shared__ float s_xmax[2][2][ROWS];  // [tile parity][key half][row]
  __shared__ float s_xl[2][ROWS];
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  volatile int* fail = &s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.z / a.Hkv, hk = blockIdx.z % a.Hkv;
  const int rep = a.Hq / a.Hkv;
  const int S = a.d_S ? (*a.d_S + a.S_add) : a.S_host;
  const int q0 = blockIdx.y * a.QB;
  const int nq = min(a.QB, a.L - q0);
  const int rows = nq * rep;
  const bool causal = a.mask_kind == M5_MASK_CAUSAL;
  int chunk = a.chunk;
  if (chunk <= 0) chunk = ((S + a.nsplit - 1) / a.nsplit + TK - 1) / TK * TK;
  const int k_begin = split * chunk;
  int k_end = min(S, k_begin + chunk);
  if (causal) k_end = min(k_end, S - a.L + q0 + nq);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + TK - 1) / TK : 0;

  if (tid == 0) {
    s_fail = 0;
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], DQ_WARPS);
    }
    for (int i = 0; i < OPB; ++i) {
      mbar_init(&op_full[i], DQ_WARPS);
      mbar_init(&op_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], SMX_WARPS);
    }
    mbar_init(p_full, SMX_WARPS);
    mbar_init(pv_done, 1);
    mbar_init(q_ready, SMX_WARPS);
    mbar_init(mma_idle, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 2);
    for (int i = 0; i < 4; ++i) mbar_init(&xend[i], 2);
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

  if (warp == PROD_WARP) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      const size_t kbase = size_t(b) * a.k.batch_stride + size_t(hk) * a.k.head_stride;
      const size_t vbase = size_t(b) * a.v.batch_stride + size_t(hk) * a.v.head_stride;
      const uint8_t* kd = reinterpret_cast<const uint8_t*>(a.k.data);
      const uint8_t* vd = reinterpret_cast<const uint8_t*>(a.v.data);
      const uint8_t* ksd = reinterpret_cast<const uint8_t*>(a.k.scales);
      const uint8_t* kbd = reinterpret_cast<const uint8_t*>(a.k.biases);
      const uint8_t* vsd = reinterpret_cast<const uint8_t*>(a.v.scales);
      const uint8_t* vbd = reinterpret_cast<const uint8_t*>(a.v.biases);
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int st = t % STAGES;
        if (!wait1(&empty[st], ((t / STAGES) & 1) ^ 1, fail, hint_ns)) break;
        const int key0 = k_begin + t * TK;
        const int nk = (min(TK, k_end - key0) + 3) & ~3;  // whole 16-byte scale rows
        uint8_t* sb = ring + size_t(st) * PK::STAGE;
        const uint32_t rowb = nk * PK::KROW, sclb = nk * 4;
        mbar_arrive_expect_tx(&full[st], 2 * rowb + 4 * sclb);
        bulk_g2s(sb + PK::K_OFF, kd + (kbase + key0) * PK::KROW, rowb, &full[st]);
        bulk_g2s(sb + PK::KS_OFF, ksd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + PK::KB_OFF, kbd + (kbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + PK::V_OFF, vd + (vbase + key0) * PK::KROW, rowb, &full[st]);
        bulk_g2s(sb + PK::VS_OFF, vsd + (vbase + key0) * 4, sclb, &full[st]);
        bulk_g2s(sb + PK::VB_OFF, vbd + (vbase + key0) * 4, sclb, &full[st]);
        issued = t + 1;
      }
      // the copies in flight land before the CTA may exit
      for (int t = std::max(0, issued - STAGES); t < issued; ++t) (void)wait1(&full[t % STAGES], (t / STAGES) & 1, fail, hint_ns);
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(ROWS, TK), idesc_o = idesc_f16(ROWS, 128);
      bool ok = ntiles > 0 && wait1(q_ready, 0, fail, hint_ns);
      auto issue_s = [&](int t) -> bool {
        const int bb = t & 1, ob = t % OPB;  // S buffer, operand buffer
        if (!wait1(&op_full[ob], (t / OPB) & 1, fail, hint_ns) || !wait1(&s_empty[bb], ((t >> 1) & 1) ^ 1, fail, hint_ns)) return false;
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const uint64_t bdesc = tc_sdesc_sw128(smem_addr(opb + size_t(ob) * OPBUF + OP_K + g * OP_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_ts(tmem + S_COL + 128u * bb + 64u * g, tmem + Q_COL + 32u * g + 8u * kk, bdesc + 2u * kk, idesc_s,
                      kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[bb]);
        return true;
      };
      // S runs two tiles ahead (both S buffers), and PV(t) goes out as soon as
      // P(t) is in TMEM: S(t + 2) needs the softmax to have read S(t), which it
      // did before publishing P(t)
      if (ok) ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      for (int t = 0; t < ntiles && ok; ++t) {
        if (!(ok = wait1(p_full, t & 1, fail, hint_ns))) break;
        tc_fence_after();
        const int ob = t % OPB;
        const uint64_t bdesc = tc_sdesc_sw128(smem_addr(opb + size_t(ob) * OPBUF + OP_V));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_ts(tmem + O_COL, tmem + P_COL + 32u * (t & 1) + 8u * kk, bdesc + 2u * kk, idesc_o,
                    (t > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pv_done);
        tc_commit(&op_empty[ob]);
        if (t + 2 < ntiles && !(ok = issue_s(t + 2))) break;
      }
      // every MMA issued has completed before TMEM may be freed
      tc_commit(mma_idle);
      (void)wait1(mma_idle, 0, fail, hint_ns);
    }
  } else if (warp >= SMX_WARPS) {
    // ---------------------------------------------------------------- dequant
    const int d = tid - SMX_WARPS * 32;  // 0..127
    const int vkb = d >> 4, vdw = d & 15, vg = vdw >> 3;  // V task: keys 8 vkb .., dims 8 vdw ..
    for (int t = 0; t < ntiles; ++t) {
      const int st = t % STAGES, bb = t % OPB;
      if (!waitw(&full[st], (t / STAGES) & 1, fail, lane, hint_ns) || !waitw(&op_empty[bb], ((t / OPB) & 1) ^ 1, fail, lane, hint_ns))
        break;
      const uint8_t* sb = ring + size_t(st) * PK::STAGE;
      uint8_t* ob = opb + size_t(bb) * OPBUF;
      const int valid = k_end - (k_begin + t * TK);
      // K codes: 64 keys x 2 groups x 8 chunks of 8 dims, exact fp16
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = d + 128 * i, n = c >> 4, g = (c >> 3) & 1, j = c & 7;
        uint4 o;
        if constexpr (BITS == 8) {
          const uint2 w = *reinterpret_cast<const uint2*>(sb + PK::K_OFF + n * 128 + 64 * g + 8 * j);
          o = make_uint4(c8(w.x, 0), c8(w.x, 1), c8(w.y, 0), c8(w.y, 1));
        } else {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(sb + PK::K_OFF + n * 64 + 32 * g + 4 * j);
          o = make_uint4(cpair(w & 15u, (w >> 4) & 15u), cpair((w >> 8) & 15u, (w >> 12) & 15u),
                         cpair((w >> 16) & 15u, (w >> 20) & 15u), cpair((w >> 24) & 15u, w >> 28));
        }
        *reinterpret_cast<uint4*>(ob + OP_K + g * OP_BYTES + sw128(n, j)) = o;
      }
      // V: keys 8 vkb .. 8 vkb + 7 x dims 8 vdw .. 8 vdw + 7, transposed and
      // dequantized two keys at a time in fp16: the exact code pair (keys 2m,
      // 2m + 1 at one dim) times the pair's scales plus their biases, one
      // fp16 rounding (scales and biases are bf16 values, exact in fp16 within
      // its normal range); zero past the last key.  Chunk e of the 8 dims is
      // taken in the rotated order (e' + vdw) & 7, so the 8 lanes of a store
      // phase hit 8 different 16-byte bank groups of the swizzled rows.
      {
        uint32_t wlo[8], whi[8], vs2[4], vb2[4];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int key = 8 * vkb + q;
          if constexpr (BITS == 8) {
            const uint2 w = *reinterpret_cast<const uint2*>(sb + PK::V_OFF + key * 128 + 8 * vdw);
            wlo[q] = w.x;
            whi[q] = w.y;
          } else {
            wlo[q] = *reinterpret_cast<const uint32_t*>(sb + PK::V_OFF + key * 64 + 4 * vdw);
            whi[q] = 0;
          }
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int k0 = 8 * vkb + 2 * m;
          float sv[2], bv[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint32_t s2 = *reinterpret_cast<const uint32_t*>(sb + PK::VS_OFF + 4 * (k0 + i));
            const uint32_t b2 = *reinterpret_cast<const uint32_t*>(sb + PK::VB_OFF + 4 * (k0 + i));
            const bool in = k0 + i < valid;
            sv[i] = in ? (vg ? bf16_hi(s2) : bf16_lo(s2)) : 0.f;
            bv[i] = in ? (vg ? bf16_hi(b2) : bf16_lo(b2)) : 0.f;
          }
          vs2[m] = pack_h2(sv[0], sv[1]);
          vb2[m] = pack_h2(bv[0], bv[1]);
        }
#pragma unroll
        for (int e0 = 0; e0 < 8; ++e0) {
          const int e = (e0 + vdw) & 7;
          uint32_t o[4];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            uint32_t cp;  // fp16 pair (code of key 2m, code of key 2m + 1) at dim e, exact
            if constexpr (BITS == 8) {
              const uint32_t wa = e < 4 ? wlo[2 * m] : whi[2 * m], wb = e < 4 ? wlo[2 * m + 1] : whi[2 * m + 1];
              const uint32_t ab = __byte_perm(wa, wb, uint32_t(e & 3) | (uint32_t(4 + (e & 3)) << 4));
              cp = c8(ab, 0);
            } else {
              const uint32_t ab = __byte_perm(wlo[2 * m], wlo[2 * m + 1], uint32_t(e >> 1) | (uint32_t(4 + (e >> 1)) << 8));
              cp = hsub1024(((ab >> (4 * (e & 1))) & 0x000F000Fu) | 0x64006400u);
            }
            o[m] = hfma2(cp, vs2[m], vb2[m]);
          }
          *reinterpret_cast<uint4*>(ob + OP_V + sw128(8 * vdw + e, vkb)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      // K scales / biases of the tile as fp32 (zero past the last key)
      if (d < TK) {
        const uint32_t ks = *reinterpret_cast<const uint32_t*>(sb + PK::KS_OFF + 4 * d);
        const uint32_t kbv = *reinterpret_cast<const uint32_t*>(sb + PK::KB_OFF + 4 * d);
        const bool in = d < valid;
        reinterpret_cast<float4*>(ob + SB_OFF)[d] = in ? make_float4(bf16_lo(ks), bf16_hi(ks), bf16_lo(kbv), bf16_hi(kbv))
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&op_full[bb]);
        mbar_arrive(&empty[st]);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int rq = warp & 3, kh = warp >> 2;  // row quarter, key half
    const int r = 32 * rq + lane;             // query row = TMEM lane
    const uint32_t lrow = uint32_t(32 * rq) << 16;
    const bool row_ok = r < rows;
    const int qi = q0 + (row_ok ? r / rep : 0), h = hk * rep + (row_ok ? r % rep : 0);
    const int qp = S - a.L + qi;                 // query position (causal mask)
    const int qp_first = S - a.L + q0;           // first query of the CTA
    // Q row: bf16-rounded q * scale (attention.py:49), exact in fp16; this
    // warp stores dims 64 kh .. 64 kh + 63 into TMEM, both group sums are kept
    float qsum[2] = {0.f, 0.f};
    {
      const bf16* qr = a.q + ((size_t(b) * a.Hq + h) * a.L + qi) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 32 dims per 16 TMEM columns
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0 = 0.f, x1 = 0.f;
          if (row_ok) {
            const __nv_bfloat162 p2 = *reinterpret_cast<const __nv_bfloat162*>(qr + 32 * c + 2 * i);
            x0 = rbf(__low2float(p2) * a.scale);
            x1 = rbf(__high2float(p2) * a.scale);
          }
          qsum[c >> 1] += x0 + x1;
          v[i] = pack_h2(x0, x1);
        }
        if ((c >> 1) == kh) tmem_st16(tmem + lrow + Q_COL + 16u * c, v);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int bb = t & 1;
      if (!(ok = waitw(&s_full[bb], (t >> 1) & 1, fail, lane, hint_ns))) break;
      if (!(ok = waitw(&op_full[t % OPB], (t / OPB) & 1, fail, lane, hint_ns))) break;  // K scales of the tile
      tc_fence_after();
      const float4* ksb = reinterpret_cast<const float4*>(opb + size_t(t % OPB) * OPBUF + SB_OFF) + 32 * kh;
      const int key0 = k_begin + t * TK + 32 * kh;
      float sc[32];
      {
        float s1[32];
        tmem_ld32(tmem + lrow + S_COL + 128u * bb + 32u * kh, sc);
        tmem_ld32(tmem + lrow + S_COL + 128u * bb + 64u + 32u * kh, s1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float4 kq = ksb[i];
          sc[i] = rbf(fmaf(kq.y, s1[i], fmaf(kq.x, sc[i], fmaf(kq.w, qsum[1], kq.z * qsum[0]))));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[bb]);  // the S buffer may take tile t + 2
      // masks only where the tile crosses the range end or the causal diagonal
      if (k_begin + (t + 1) * TK > k_end || (causal && k_begin + (t + 1) * TK - 1 > qp_first)) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + i;
          if (!(key < k_end && (!causal || key <= qp))) sc[i] = -INFINITY;
        }
      }
      // the row max over both key halves
      float tmax = max32(sc);
      s_xmax[t & 1][kh][r] = tmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[2 * rq + (t & 1)]);
      if (!(ok = waitw(&xbar[2 * rq + (t & 1)], (t >> 1) & 1, fail, lane, hint_ns))) break;
      tmax = fmaxf(tmax, s_xmax[t & 1][kh ^ 1][r]);
      const float mn = fmaxf(m_run, tmax);
      const float corr = (m_run == mn) ? 1.f : (m_run == -INFINITY ? 0.f : ex2((m_run - mn) * LOG2E));
      m_run = mn;
      const float mnl = mn == -INFINITY ? 0.f : mn * LOG2E;
#pragma unroll
      for (int i = 0; i < 32; ++i) sc[i] = ex2(fmaf(sc[i], LOG2E, -mnl));
      l_run = l_run * corr + sum32(sc);
      // P (this warp's 32 keys) = fp16 pairs of rb(p), into the tile's P buffer
      {
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = pack_h2(rbf(sc[2 * i]), rbf(sc[2 * i + 1]));
        tmem_st16(tmem + lrow + P_COL + 32u * (t & 1) + 16u * kh, v);
      }
      // the previous tile's PV has finished: O is stable
      if (t > 0 && !(ok = waitw(pv_done, (t - 1) & 1, fail, lane, hint_ns))) break;
      tc_fence_after();
      if (t > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // this warp's 64 columns of O
          float o[32];
          const uint32_t col = O_COL + 64u * kh + 32u * c;
          tmem_ld32(tmem + lrow + col, o);
          tmem_ld_wait();
          uint32_t u0[16], u1[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            u0[i] = __float_as_uint(o[i] * corr);
            u1[i] = __float_as_uint(o[16 + i] * corr);
          }
          tmem_st16(tmem + lrow + col, u0);
          tmem_st16(tmem + lrow + col + 16u, u1);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---- finish: wait for the last PV, add the two halves' denominators,
    // normalise this warp's 64 dims and write them
    if (ok && ntiles > 0) ok = waitw(pv_done, (ntiles - 1) & 1, fail, lane, hint_ns);
    if (ok) {
      s_xl[kh][r] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xend[rq]);
      ok = waitw(&xend[rq], 0, fail, lane, hint_ns);
    }
    tc_fence_after();
    if (ok) {
      const float l_tot = s_xl[0][r] + s_xl[1][r];
      const size_t orow = (size_t(b) * a.Hq + h) * a.L + qi;
      const float inv = 1.f / fmaxf(l_tot, 1e-30f);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float o[32];
        const int d0 = 64 * kh + 32 * c;  // first dim of the 32
        if (ntiles > 0) {
          tmem_ld32(tmem + lrow + O_COL + uint32_t(d0), o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (!row_ok) continue;
        if (a.nsplit == 1) {
          const size_t od = a.out_tokens_major ? ((size_t(b) * a.L + qi) * a.Hq + h) : orow;
          uint4* dst = reinterpret_cast<uint4*>(a.out + od * 128 + d0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __nv_bfloat162 v2 = __floats2bfloat162_rn(o[8 * i + 2 * j] * inv, o[8 * i + 2 * j + 1] * inv);
              w[j] = *reinterpret_cast<const uint32_t*>(&v2);
            }
            dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float4* po = reinterpret_cast<float4*>(a.part_o + (orow * a.nsplit + split) * 128 + d0);
#pragma unroll
          for (int i = 0; i < 8; ++i) po[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
      if (row_ok && a.nsplit > 1 && kh == 0) {
        a.part_ml[(orow * a.nsplit + split) * 2 + 0] = m_run;
        a.part_ml[(orow * a.nsplit + split) * 2 + 1] = l_tot;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace atc

// The tcgen05 kernel runs prefill attention; M5_ATTN_TC=0 selects the
// mma.sync kernel (attn_pf.cu) instead.
static bool attn_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("M5_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool attn_tc_eligible(const AttnArgs& a) {
  return attn_tc_enabled() && attn_pf_eligible(a);  // same shapes, masks and alignment as the mma.sync kernel
}

void attn_tc_plan(const AttnArgs& a, int S_max, int max_split, int& QB, int& nsplit) {
  const int rep = a.Hq / a.Hkv;
  QB = std::max(1, std::min(a.L, atc::ROWS / rep));
  const long long ctas = (long long)a.B * a.Hkv * ((a.L + QB - 1) / QB);
  const int tiles = std::max(1, (S_max + atc::TK - 1) / atc::TK);
  const long long want = ((long long)sm_count() + ctas - 1) / ctas;  // one CTA per SM
  nsplit = (int)std::max(1LL, std::min<long long>(std::min<long long>(want, tiles), max_split));
}

// Suspend-time hint of the kernel's mbarrier waits (M5_ATTN_TC_HINT_NS, 0 = poll).
static uint32_t attn_tc_hint_ns() {
  static const uint32_t v = [] {
    const char* e = getenv("M5_ATTN_TC_HINT_NS");
    return e ? uint32_t(strtoul(e, nullptr, 10)) : 1000000u;
  }();
  return v;
}

// Operand buffers of the kernel (M5_ATTN_TC_OPB, 2 or 3).
static int attn_tc_opb() {
  static const int v = [] {
    const char* e = getenv("M5_ATTN_TC_OPB");
    return e && e[0] == '2' ? 2 : 3;
  }();
  return v;
}

template <int BITS, int OPB>
static cudaError_t attn_tc_launch_t(const AttnArgs& a, dim3 grid, uint32_t hint, cudaStream_t stream) {
  constexpr size_t smem = atc::smem_bytes<BITS, OPB>();
  static DeviceOnce once;  // the attribute belongs to each device's context
  cudaError_t e = once.run([&] {
    return cudaFuncSetAttribute(atc::attn_tc_kernel<BITS, OPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (e != cudaSuccess) return e;
  atc::attn_tc_kernel<BITS, OPB><<<grid, atc::THREADS, smem, stream>>>(a, hint);
  return cudaSuccess;
}

int attn_tc_launch(const AttnArgs& a, cudaStream_t stream) {
  dim3 grid(a.nsplit, (a.L + a.QB - 1) / a.QB, a.B * a.Hkv);
  const uint32_t hint = attn_tc_hint_ns();
  const bool three = attn_tc_opb() == 3;
  cudaError_t e;
  if (a.bits == 8) e = three ? attn_tc_launch_t<8, 3>(a, grid, hint, stream) : attn_tc_launch_t<8, 2>(a, grid, hint, stream);
  else e = three ? attn_tc_launch_t<4, 3>(a, grid, hint, stream) : attn_tc_launch_t<4, 2>(a, grid, hint, stream);
  M5_CUDA(e);
  M5_LAUNCH_CHECK("prefill attention (tcgen05) launch");
  return M5_OK;
}

int attn_tc_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_tc_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_attn_tc_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
