// Decode dequant-GEMV: TMA tiles into shared memory + tensor-core dot
// products (kernel K1, M <= 8 tokens, K % 512 == 0; a row's last 1024-column
// unit may be partial).
//
// The register-prefetch tensor-core GEMV (gemv_mma.cu) spends ~3.6 issue
// slots per weight and stalls on L1 load latency with 16 warps per SM; the
// TMA-fed CUDA-core GEMV (gemv_tma.cu) keeps enough bytes in flight but is
// issue-bound at ~5.3 slots per weight.  This kernel takes the best of both:
//   * a ring's producer warp streams units of (16 weight rows x 1024 columns)
//     with one 3-D tensor-map TMA box for the codes (128-byte swizzle, so the
//     8 rows a fragment load touches hit different banks) and one box each for
//     the bf16 scales and biases, into an mbarrier ring, no registers
//     involved.  A CTA holds one ring (three CTAs per SM, 5 stages) when three
//     copies of the staged activations fit an SM, else three rings (one CTA
//     per SM) that share one copy and take the memory it frees as deeper rings
//     (3-8 stages; down_proj's 25600-long rows);
//   * the consumer warps first stage the activations once per CTA (input
//     RMSNorm, 16-bit fixed-point planes per 64-column group), then four warps
//     per ring each take four 64-column scale groups of every unit of their
//     ring and run int8 mma.sync m16n8k32 products of the exact codes against
//     the planes (or, with M5_GEMV_I8=0, fp16 m16n8k16 products against
//     per-token scaled activations), folding s * D + b * sum(x) per group;
//   * units are dealt to rings as equal contiguous ranges (stream-K); a tile
//     shared by neighbouring rings is summed from their per-ring slots in ring
//     order by the ring that completes it (no floating-point atomics, so the
//     result is bitwise repeatable), which then runs the epilogue.
// All mbarrier waits are bounded (tma.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "frag_stage.cuh"
#include "gemv.cuh"
#include "rope_impl.cuh"
#include "tma.cuh"

namespace m5 {

static __device__ int g_gemv_tmap_err = 0;

constexpr int TP_CW = 4;                       // consumer warps of a ring
constexpr int TP_MAX_STAGES = 8;
constexpr int TP_UG = 16;                     // 64-column scale groups per unit (1024 columns)
constexpr int TP_W_STAGE = 16 * TP_UG * 32;    // 16 rows x UG groups x 32 bytes (1 KB swizzled boxes)
constexpr int TP_SB_STAGE = 16 * TP_UG * 2;    // 16 rows x UG bf16 (scales or biases)
// Rings per CTA: 1 (three CTAs per SM when their activation copies fit) or 3
// (one CTA per SM whose rings share one activation copy).
constexpr int tp_threads(int sub) { return sub * (TP_CW + 1) * 32; }
constexpr int tp_bars(int sub) { return sub * 2 * TP_MAX_STAGES + 2; }  // full, empty per ring; activation copy (+ pad)
// Row blocks of a unit fetched by separate boxes: the two 8-row halves of a
// SwiGLU tile come from the gate and the up matrix; any other tile's 16 rows
// are one block of one segment (segments are whole tiles).
#define TP_HALVES (EPI == EPI_SWIGLU ? 2 : 1)

struct TmapSet {
  CUtensorMap w[3], s[3], b[3];  // per segment
};

__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t tp_hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t tp_hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 8 codes of one word -> fp16 pairs (q0,q4) (q1,q5) (q2,q6) (q3,q7), exact.
// Under the fp16 exponent of 64 (0x5400) one mantissa step is 1/16, so a code
// byte placed in a half's low mantissa bits reads 64 + lo/16 + hi, and its low
// nibble alone reads 64 + lo/16.  The integer pipe builds those four halves
// per pair of bytes (three masks, one byte permute: 4 operations per word);
// the FMA pipe takes hi as their difference and lo = 16 (64 + lo/16) - 1024.
__device__ __forceinline__ void tp_codes_f16(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t f02 = (w & 0x00FF00FFu) | 0x54005400u;  // bytes 0 and 2
  const uint32_t l02 = (w & 0x000F000Fu) | 0x54005400u;
  const uint32_t f13 = __byte_perm(w, 0x54u, 0x4341);     // bytes 1 and 3 under 0x54
  const uint32_t l13 = f13 & 0xFF0FFF0Fu;
  p[0] = tp_hfma2(l02, 0x4C004C00u, 0xE400E400u);  // * 16 - 1024
  p[1] = tp_hsub2(f02, l02);
  p[2] = tp_hfma2(l13, 0x4C004C00u, 0xE400E400u);
  p[3] = tp_hsub2(f13, l13);
}

// Integer MMAs of the int8 variant: u8 weight codes (0..15) against the s8
// high plane and the u8 low plane of the 16-bit fixed-point activations;
// exact int32 sums.
__device__ __forceinline__ void tp_imma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void tp_imma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tp_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Half h (rows 8h..8h+7) of tile `tile`: segment and first row inside it.
template <int EPI>
__device__ __forceinline__ void tp_half(const GemvArgs& a, int tile, int h, int& si, int& row0) {
  if constexpr (EPI == EPI_SWIGLU) {
    si = h;
    row0 = tile * 8;
  } else {
    int v = tile * 16 + 8 * h;
    si = 0;
    while (si < a.nseg - 1 && v >= a.seg[si].rows) {
      v -= a.seg[si].rows;
      ++si;
    }
    row0 = v;
  }
}

// QK-norm + RoPE + KV append of head h for MT tokens, by one warp, once the
// head's 8 tiles are written (kept out of line: it runs once per 8 tiles and
// its trigonometric slow path must not weigh on the dot-product loop).
__device__ __noinline__ void tp_rope_head(const RopeAppendArgs& r, int MT, int h, int lane) {
  for (int t = 0; t < MT; ++t) rope_append_row_any<true>(r, t, h, lane);
}

// I8 selects the consumer: false = fp16 MMAs on exact codes against the
// activations scaled per token (stage_frag_bulk), true = int8 MMAs (u8 codes
// as they sit in the word, one mask or shift-and-mask per 4 codes) against
// per-group 16-bit fixed-point activation planes (stage_i8_bulk), int32 group
// sums folded as s * 2^(E - 14) * D + b * sum(x).
template <int MT, int EPI, bool I8, int SUB>
__global__ void __launch_bounds__(tp_threads(SUB), SUB == 1 ? 3 : 1) gemv_tmap_kernel(const __grid_constant__ GemvArgs a, const __grid_constant__ TmapSet tm,
                                                               float* part, int* cnt_buf, int nst) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 128-byte-swizzled boxes must start on 1 KB boundaries
  unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  const int K = a.K, NG = K >> 6, NCH = (NG + TP_UG - 1) / TP_UG;  // the last unit of a row may be partial
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warps 0 .. 4 SUB - 1: consumers, four per ring; then one producer per ring
  constexpr int NC = SUB * TP_CW * 32;  // consumer threads
  const bool producer = warp >= SUB * TP_CW;
  const int sub = producer ? warp - SUB * TP_CW : warp / TP_CW, cw = warp % TP_CW;
  const int stage_bytes = TP_W_STAGE + 2 * TP_SB_STAGE;
  unsigned char* wring = smem + size_t(sub) * nst * stage_bytes;  // [nst][4096], 1024-aligned boxes
  unsigned char* sbring = wring + nst * TP_W_STAGE;               // [nst][2 (s,b)][256]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(SUB) * nst * stage_bytes);
  uint64_t* full = bars + sub * 2 * TP_MAX_STAGES;
  uint64_t* empty = full + TP_MAX_STAGES;
  uint64_t* xbar = bars + SUB * 2 * TP_MAX_STAGES;                 // activation copy
  // activation staging, shared by the CTA's rings
  uint32_t* xf = reinterpret_cast<uint32_t*>(bars + tp_bars(SUB));  // [MT][NG][4][8] pairs
  uint32_t* nbuf = xf + MT * NG * 32;                             // [K] bf16 norm weight (if any)
  float* xg = reinterpret_cast<float*>(nbuf + (a.norm_w ? K / 2 : 0));  // [MT][NG]
  float* xsc = xg + MT * NG;                                      // [MT][NG] group scales (I8)
  float* red = xsc + (I8 ? MT * NG : 0);                          // [8], then the rings' tile sums

  const int vrows = a.total_rows * (EPI == EPI_SWIGLU ? 2 : 1);
  const int ntiles = vrows >> 4;
  const long long total = (long long)ntiles * NCH;
  // ring `sub` of CTA b is virtual CTA b * SUB + sub: equal contiguous unit ranges
  const long long G_ = (long long)gridDim.x * SUB, vid = (long long)blockIdx.x * SUB + sub;
  const long long u0 = total * vid / G_, u1 = total * (vid + 1) / G_;

  if (tid == 0) {
    for (int r = 0; r < SUB; ++r)
      for (int s = 0; s < nst; ++s) {
        mbar_init(&bars[r * 2 * TP_MAX_STAGES + s], 1);
        mbar_init(&bars[r * 2 * TP_MAX_STAGES + TP_MAX_STAGES + s], TP_CW);
      }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (producer) {
    // -------------------------------------------------------------- producer
    // streams constant weights: needs nothing from earlier kernels
    if (lane == 0) {
      int it = 0;
      int tile = int(u0 / NCH), ch = int(u0 % NCH);
      for (long long u = u0; u < u1; ++u, ++it) {
        const int st = it % nst;
        const uint32_t par = (it / nst) & 1;
        // the ring is full: from here on the consumers gate this warp, and they
        // start only once the previous kernel has finished
        if (it == nst) {
          pdl_wait();
          pdl_launch_dependents();
        }
        if (!mbar_wait(&empty[st], par ^ 1, &g_gemv_tmap_err)) return;
        mbar_arrive_expect_tx(&full[st], TP_W_STAGE + 2 * TP_SB_STAGE);
        unsigned char* ws = wring + st * TP_W_STAGE;
        unsigned char* ss = sbring + st * 2 * TP_SB_STAGE;
        // one 3-D box per row block: 32 words x rows x 4 128-byte chunks (the
        // unit's 1024 columns), landing as [chunk][row][128 B] with the
        // 128-byte swizzle keyed by the row; scales and biases one box each
#pragma unroll
        for (int h = 0; h < TP_HALVES; ++h) {
          int si, row0;
          tp_half<EPI>(a, tile, h, si, row0);
          tma3d(ws + h * (TP_W_STAGE / TP_HALVES), &tm.w[si], 0, row0, ch * (TP_UG / 4), &full[st]);
          tma2d(ss + h * (TP_SB_STAGE / TP_HALVES), &tm.s[si], ch * TP_UG, row0, &full[st]);
          tma2d(ss + TP_SB_STAGE + h * (TP_SB_STAGE / TP_HALVES), &tm.b[si], ch * TP_UG, row0, &full[st]);
        }
        if (++ch == NCH) {
          ch = 0;
          ++tile;
        }
      }
    }
    return;
  }

  // ---------------------------------------------- consumers: stage activations
  float* xinv = red;  // [MT] 2^-e of the fp16 activation scale (red[0..7] is free after staging)
  pdl_wait();         // activations, residual and split-tile scratch come from earlier kernels
  // The next kernel may launch only now: launched earlier, its CTAs could take
  // the SM slots this grid's own CTAs still wait for.
  pdl_launch_dependents();
  if constexpr (I8)
    stage_i8_bulk<MT, NC>(a.x, a.ldx, K, a.norm_w, a.eps, xf, nbuf, xg, xsc, red, 1, xbar, &g_gemv_tmap_err);
  else
    stage_frag_bulk<MT, NC, true>(a.x, a.ldx, K, a.norm_w, a.eps, xf, nbuf, xg, red, 1, xinv, xbar,
                                          &g_gemv_tmap_err);

  const int g = lane >> 2, tq = lane & 3;
  const int tok = g < MT ? g : MT - 1;
  const int t0c = 2 * tq < MT ? 2 * tq : MT - 1, t1c = 2 * tq + 1 < MT ? 2 * tq + 1 : MT - 1;
  const uint32_t* xfl = xf + tok * NG * 32 + tq * 8;
  const float* xg0 = xg + t0c * NG;
  const float* xg1 = xg + t1c * NG;
  const float* xs0 = xsc + t0c * NG;
  const float* xs1 = xsc + t1c * NG;
  const float xi0 = I8 ? 1.f : xinv[t0c], xi1 = I8 ? 1.f : xinv[t1c];
  // per-thread smem offsets of this warp's four groups inside a stage (the
  // 128-byte swizzle of the weight boxes depends only on g, tq and the group)
  // stage layout [half][chunk][8 rows][128 B] (SwiGLU) or [chunk][16 rows][128 B]
  constexpr uint32_t W_CHUNK = EPI == EPI_SWIGLU ? 1024 : 2048;  // bytes per 128-byte column chunk
  constexpr uint32_t W_ROW8 = EPI == EPI_SWIGLU ? 4096 : 1024;   // offset of rows g + 8
  uint32_t woff[TP_UG / TP_CW];
#pragma unroll
  for (int jj = 0; jj < TP_UG / TP_CW; ++jj) {
    const int c = 2 * jj + (tq >> 1);
    woff[jj] = cw * W_CHUNK + g * 128 + ((c ^ g) << 4) + 8 * (tq & 1);
  }
  const uint32_t soff = g * (TP_UG * 2) + cw * (TP_UG / TP_CW) * 2;  // 4 consecutive bf16 of row g

  float tot[4] = {0.f, 0.f, 0.f, 0.f};
  float totD[4] = {0.f, 0.f, 0.f, 0.f}, totB[4] = {0.f, 0.f, 0.f, 0.f};
  int cur_tile = u0 < u1 ? int(u0 / NCH) : 0;
  // Epilogue of one finished tile row r16 / token t with its complete sum v.
  auto epilogue = [&](int tile, int r16, int t, float v, float vu) {
    if constexpr (EPI == EPI_SWIGLU) {
      const float gv = rbf(v), uv = rbf(vu);
      const float sg = rbf(1.f / (1.f + expf(-gv)));
      a.seg[0].y[t * a.ldy + tile * 8 + r16] = f2bf(rbf(gv * sg) * uv);
    } else {
      int si, row0;
      tp_half<EPI>(a, tile, r16 >> 3, si, row0);
      const int rr = row0 + (r16 & 7);
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
  };
  // Called by the whole warp that wrote tile `tile` (EPI_STORE): the 8th tile
  // of a head to finish runs the head's QK-norm + RoPE + KV append.  The
  // counter wraps to 0 on the 8th arrival (atomicInc), ready for the next launch.
  auto rope_tile = [&](int tile) {
    if (a.rope_cnt == nullptr) return;
    __threadfence();  // this warp's rows of the tile, before the count
    __syncwarp();
    unsigned int old = 0;
    if (lane == 0) old = atomicInc(&a.rope_cnt[tile >> 3], 7u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == 7u) {
      __threadfence();  // the other tiles' rows, after their counts
      tp_rope_head(a.rope, MT, tile >> 3, lane);
    }
  };
  float* tred = red + 8 + sub * (TP_CW * MT * 16);  // this ring's [CW][MT][16] partial tile sums
  // Every tile is first reduced over the four consumer warps in shared memory
  // (warp order).  A tile whose units all lie in this CTA's range is finished
  // at once; a tile shared with neighbouring CTAs leaves this CTA's sum in its
  // own slot of `part` (slot 0: the CTA's first tile, 1: its last), and the
  // CTA that completes the tile's unit count adds the slots of the CTAs that
  // cover it in CTA order.  No floating-point atomics: the result does not
  // depend on which CTA finishes first.
  auto unit_begin = [&](long long c) { return total * c / G_; };
  auto cta_of = [&](long long u) {  // the CTA whose range holds unit u
    long long c = u * G_ / total;
    while (c + 1 < G_ && unit_begin(c + 1) <= u) ++c;
    while (c > 0 && unit_begin(c) > u) --c;
    return int(c);
  };
  auto flush = [&](int tile) {
    tot[0] = fmaf(totD[0], xi0, totB[0]);
    tot[1] = fmaf(totD[1], xi1, totB[1]);
    tot[2] = fmaf(totD[2], xi0, totB[2]);
    tot[3] = fmaf(totD[3], xi1, totB[3]);
    const int t0 = 2 * tq, t1 = 2 * tq + 1;
    const long long tb = (long long)tile * NCH, te = tb + NCH;  // the tile's units
    const bool whole = tb >= u0 && te <= u1;
    if (t0 < MT) {
      tred[(cw * MT + t0) * 16 + g] = tot[0];
      tred[(cw * MT + t0) * 16 + g + 8] = tot[2];
    }
    if (t1 < MT) {
      tred[(cw * MT + t1) * 16 + g] = tot[1];
      tred[(cw * MT + t1) * 16 + g + 8] = tot[3];
    }
    named_sync(2 + sub, TP_CW * 32);
    if (cw == 0) {
      if (whole) {
        for (int q = lane; q < 16 * MT; q += 32) {
          const int r16 = q & 15, t = q >> 4;
          float v = 0.f, vu = 0.f;
#pragma unroll
          for (int w = 0; w < TP_CW; ++w) {
            v += tred[(w * MT + t) * 16 + r16];
            if (EPI == EPI_SWIGLU && r16 < 8) vu += tred[(w * MT + t) * 16 + r16 + 8];
          }
          if (EPI != EPI_SWIGLU || r16 < 8) epilogue(tile, r16, t, v, vu);
        }
        if constexpr (EPI == EPI_STORE) rope_tile(tile);
      } else {
        float* mine = part + (size_t(vid) * 2 + (tb <= u0 ? 0 : 1)) * (MT * 16);
        for (int q = lane; q < 16 * MT; q += 32) {
          const int r16 = q & 15, t = q >> 4;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < TP_CW; ++w) v += tred[(w * MT + t) * 16 + r16];
          mine[q] = v;
        }
        __threadfence();  // the slot, before the count
        __syncwarp();
        const int here = int(min(u1, te) - max(u0, tb));
        int last = 0;
        if (lane == 0) last = (atomicAdd(&cnt_buf[tile], here) + here == NCH);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();  // the other CTAs' slots, after their counts
          const int c_lo = cta_of(tb), c_hi = cta_of(te - 1);
          constexpr int QN = (16 * MT + 31) / 32;  // rows x tokens per lane
          float v[QN], vu[QN];
#pragma unroll
          for (int k = 0; k < QN; ++k) v[k] = vu[k] = 0.f;
          for (int c = c_lo; c <= c_hi; ++c) {  // CTA order
            const float* p = part + (size_t(c) * 2 + (unit_begin(c) >= tb ? 0 : 1)) * (MT * 16);
#pragma unroll
            for (int k = 0; k < QN; ++k) {
              const int q = lane + 32 * k;
              if (q < 16 * MT) {
                v[k] += __ldcg(p + q);
                if (EPI == EPI_SWIGLU && (q & 15) < 8) vu[k] += __ldcg(p + q + 8);
              }
            }
          }
#pragma unroll
          for (int k = 0; k < QN; ++k) {
            const int q = lane + 32 * k, r16 = q & 15, t = q >> 4;
            if (q < 16 * MT && (EPI != EPI_SWIGLU || r16 < 8)) epilogue(tile, r16, t, v[k], vu[k]);
          }
          __syncwarp();
          if (lane == 0) cnt_buf[tile] = 0;
          if constexpr (EPI == EPI_STORE) rope_tile(tile);
        }
      }
    }
    named_sync(2 + sub, TP_CW * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[i] = totD[i] = totB[i] = 0.f;
  };

  bool failed = false;
  int tile = cur_tile, ch = u0 < u1 ? int(u0 % NCH) : 0;
  int st = 0;
  uint32_t par = 0;
  for (long long u = u0; u < u1; ++u) {
    if (tile != cur_tile) {
      flush(cur_tile);
      cur_tile = tile;
    }
    // On a timed-out wait the warp stops computing but keeps walking the units
    // so that every consumer warp still reaches the tile barriers in flush().
    if (!failed && !mbar_wait(&full[st], par, &g_gemv_tmap_err)) failed = true;
    // K % 512 == 0: a warp's four groups lie all inside the row or all past
    // its end (the partial last unit of a row: zero-filled by the copy and
    // skipped here, though the warp still takes its turn on the stage)
    const int G0 = ch * TP_UG + cw * (TP_UG / TP_CW);  // first global group of this warp
    if (!failed && G0 < NG) {
      const unsigned char* ws = wring + st * TP_W_STAGE;
      const unsigned char* ss = sbring + st * 2 * TP_SB_STAGE;
      // scales / biases of the warp's 4 groups, rows g and g + 8; group sums of x
      const uint2 sv0 = *reinterpret_cast<const uint2*>(ss + soff);
      const uint2 sv8 = *reinterpret_cast<const uint2*>(ss + TP_SB_STAGE / 2 + soff);
      const uint2 bv0 = *reinterpret_cast<const uint2*>(ss + TP_SB_STAGE + soff);
      const uint2 bv8 = *reinterpret_cast<const uint2*>(ss + TP_SB_STAGE + TP_SB_STAGE / 2 + soff);
      const float4 X0 = *reinterpret_cast<const float4*>(xg0 + G0);
      const float4 X1 = *reinterpret_cast<const float4*>(xg1 + G0);
      const float X0a[4] = {X0.x, X0.y, X0.z, X0.w}, X1a[4] = {X1.x, X1.y, X1.z, X1.w};
      const uint32_t sw0[2] = {sv0.x, sv0.y}, sw8[2] = {sv8.x, sv8.y}, bw0[2] = {bv0.x, bv0.y},
                     bw8[2] = {bv8.x, bv8.y};
      if constexpr (I8) {
        const float4 F0 = *reinterpret_cast<const float4*>(xs0 + G0);
        const float4 F1 = *reinterpret_cast<const float4*>(xs1 + G0);
        const float F0a[4] = {F0.x, F0.y, F0.z, F0.w}, F1a[4] = {F1.x, F1.y, F1.z, F1.w};
#pragma unroll
        for (int jj = 0; jj < TP_UG / TP_CW; ++jj) {
          const uint2 w0 = *reinterpret_cast<const uint2*>(ws + woff[jj]);
          const uint2 w8 = *reinterpret_cast<const uint2*>(ws + W_ROW8 + woff[jj]);
          const uint4 xh = *reinterpret_cast<const uint4*>(xfl + (G0 + jj) * 32);      // s8 plane
          const uint4 xl = *reinterpret_cast<const uint4*>(xfl + (G0 + jj) * 32 + 4);  // u8 plane
          int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0};
          {
            const uint32_t A[4] = {w0.x & 0x0F0F0F0Fu, w8.x & 0x0F0F0F0Fu, (w0.x >> 4) & 0x0F0F0F0Fu,
                                   (w8.x >> 4) & 0x0F0F0F0Fu};
            tp_imma_s8(dh, A, xh.x, xh.y);
            tp_imma_u8(dl, A, xl.x, xl.y);
          }
          {
            const uint32_t A[4] = {w0.y & 0x0F0F0F0Fu, w8.y & 0x0F0F0F0Fu, (w0.y >> 4) & 0x0F0F0F0Fu,
                                   (w8.y >> 4) & 0x0F0F0F0Fu};
            tp_imma_s8(dh, A, xh.z, xh.w);
            tp_imma_u8(dl, A, xl.z, xl.w);
          }
          const uint32_t s0w = sw0[jj >> 1], s8w = sw8[jj >> 1], b0w = bw0[jj >> 1], b8w = bw8[jj >> 1];
          const float sA = (jj & 1) ? bf16_hi(s0w) : bf16_lo(s0w), sB = (jj & 1) ? bf16_hi(s8w) : bf16_lo(s8w);
          const float bA = (jj & 1) ? bf16_hi(b0w) : bf16_lo(b0w), bB = (jj & 1) ? bf16_hi(b8w) : bf16_lo(b8w);
          // exact: |256 dh + dl| < 2^25 (64 codes <= 15 times |v| < 2^15)
          totD[0] = fmaf(sA * F0a[jj], float(dh[0] * 256 + dl[0]), totD[0]);
          totD[2] = fmaf(sB * F0a[jj], float(dh[2] * 256 + dl[2]), totD[2]);
          totB[0] = fmaf(bA, X0a[jj], totB[0]);
          totB[2] = fmaf(bB, X0a[jj], totB[2]);
          if constexpr (MT > 1) {  // the odd columns hold other tokens only when there are any
            totD[1] = fmaf(sA * F1a[jj], float(dh[1] * 256 + dl[1]), totD[1]);
            totD[3] = fmaf(sB * F1a[jj], float(dh[3] * 256 + dl[3]), totD[3]);
            totB[1] = fmaf(bA, X1a[jj], totB[1]);
            totB[3] = fmaf(bB, X1a[jj], totB[3]);
          }
        }
      } else {
#pragma unroll
      for (int jj = 0; jj < TP_UG / TP_CW; ++jj) {
        const uint2 w0 = *reinterpret_cast<const uint2*>(ws + woff[jj]);
        const uint2 w8 = *reinterpret_cast<const uint2*>(ws + W_ROW8 + woff[jj]);
        const uint4 xa = *reinterpret_cast<const uint4*>(xfl + (G0 + jj) * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xfl + (G0 + jj) * 32 + 4);
        uint32_t pa0[4], pa8[4], pb0[4], pb8[4];
        tp_codes_f16(w0.x, pa0);
        tp_codes_f16(w8.x, pa8);
        tp_codes_f16(w0.y, pb0);
        tp_codes_f16(w8.y, pb8);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const uint32_t A[4] = {pa0[0], pa8[0], pa0[1], pa8[1]};
          tp_mma(d, A, xa.x, xa.y);
        }
        {
          const uint32_t A[4] = {pa0[2], pa8[2], pa0[3], pa8[3]};
          tp_mma(d, A, xa.z, xa.w);
        }
        {
          const uint32_t A[4] = {pb0[0], pb8[0], pb0[1], pb8[1]};
          tp_mma(d, A, xb.x, xb.y);
        }
        {
          const uint32_t A[4] = {pb0[2], pb8[2], pb0[3], pb8[3]};
          tp_mma(d, A, xb.z, xb.w);
        }
        const uint32_t s0w = sw0[jj >> 1], s8w = sw8[jj >> 1], b0w = bw0[jj >> 1], b8w = bw8[jj >> 1];
        const float sA = (jj & 1) ? bf16_hi(s0w) : bf16_lo(s0w), sB = (jj & 1) ? bf16_hi(s8w) : bf16_lo(s8w);
        const float bA = (jj & 1) ? bf16_hi(b0w) : bf16_lo(b0w), bB = (jj & 1) ? bf16_hi(b8w) : bf16_lo(b8w);
        totD[0] = fmaf(sA, d[0], totD[0]);
        totD[1] = fmaf(sA, d[1], totD[1]);
        totD[2] = fmaf(sB, d[2], totD[2]);
        totD[3] = fmaf(sB, d[3], totD[3]);
        totB[0] = fmaf(bA, X0a[jj], totB[0]);
        totB[1] = fmaf(bA, X1a[jj], totB[1]);
        totB[2] = fmaf(bB, X0a[jj], totB[2]);
        totB[3] = fmaf(bB, X1a[jj], totB[3]);
      }
      }
    }
    if (!failed) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (++ch == NCH) {
      ch = 0;
      ++tile;
    }
    if (++st == nst) {
      st = 0;
      par ^= 1;
    }
  }
  if (u0 < u1) flush(cur_tile);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Maps of one segment; `brows` rows per box (16, or 8 for a SwiGLU half).
// Weights as 3-D: 32 words of a 128-byte chunk, rows (stride K/2 bytes), the
// K/256 chunks of a row (stride 128 bytes).
static int make_maps(const GemvSeg& sg, int K, TmapSet& ts, int i, int brows) {
  auto enc = encode_fn();
  if (!enc) return fail(M5_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t rows = (cuuint64_t)sg.rows;
  {
    cuuint64_t dims[3] = {32, rows, (cuuint64_t)K / 256};
    cuuint64_t strides[2] = {(cuuint64_t)K / 2, 128};
    cuuint32_t box[3] = {32, (cuuint32_t)brows, TP_UG / 4}, es[3] = {1, 1, 1};
    CUresult r = enc(&ts.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t*>(sg.w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(M5_ERR_CUDA, "tensor map (weights) encode failed");
  }
  const bf16* p2[2] = {sg.s, sg.b};
  CUtensorMap* m2[2] = {&ts.s[i], &ts.b[i]};
  for (int k = 0; k < 2; ++k) {
    cuuint64_t dims[2] = {(cuuint64_t)K / 64, rows};
    cuuint64_t strides[1] = {(cuuint64_t)K / 32};
    cuuint32_t box[2] = {TP_UG, (cuuint32_t)brows}, es[2] = {1, 1};
    CUresult r = enc(m2[k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16*>(p2[k]), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(M5_ERR_CUDA, "tensor map (scales) encode failed");
  }
  return M5_OK;
}

// Shared memory of a CTA: its rings of nst stages, their barriers, the shared
// activation staging (planes, norm weight, group sums and scales) and the
// rings' tile sums (which also hold the staging's per-warp partials).
static size_t tp_smem(int MT, int K, bool norm, bool i8, int sub, int nst) {
  return size_t(sub) * nst * (TP_W_STAGE + 2 * TP_SB_STAGE) + tp_bars(sub) * 8 + size_t(MT) * (K / 64) * 32 * 4 +
         (norm ? size_t(K) * 2 : 0) + size_t(MT) * (K / 64) * 4 * (i8 ? 2 : 1) + 8 * 4 +
         size_t(sub) * TP_CW * MT * 16 * 4 + 1024;
}

constexpr size_t TP_SMEM_MAX = 227 * 1024;  // opt-in dynamic shared memory of one CTA
constexpr size_t TP_SMEM_SM = 228 * 1024;   // shared memory of an SM (1 KB of it reserved per CTA)
constexpr int TP_STAGES1 = 5;               // ring depth of the one-ring CTA

// Launch shape of a GEMV: one-ring CTAs (5 stages) while three of them fit an
// SM; otherwise, for the int8 consumer, one CTA of three rings sharing the
// activation copy, as deep as the memory allows (3..8 stages).  sub = 0 when
// neither fits.
struct TpShape {
  int sub = 0, nst = 0;
  size_t smem = 0;
};
static TpShape tp_shape(int MT, int K, bool norm, bool i8) {
  TpShape r;
  const size_t one = tp_smem(MT, K, norm, i8, 1, TP_STAGES1);
  if (3 * (one + 1024) <= TP_SMEM_SM || (!i8 && one <= TP_SMEM_MAX)) {
    r.sub = 1;
    r.nst = TP_STAGES1;
    r.smem = one;
    return r;
  }
  if (!i8) return r;
  for (int n = TP_MAX_STAGES; n >= 3; --n)
    if (tp_smem(MT, K, norm, i8, 3, n) <= TP_SMEM_MAX) {
      r.sub = 3;
      r.nst = n;
      r.smem = tp_smem(MT, K, norm, i8, 3, n);
      return r;
    }
  return r;
}

// The int8 consumer is the default; M5_GEMV_I8=0 selects the fp16 one.
static bool tp_use_i8() {
  static const bool on = [] {
    const char* e = getenv("M5_GEMV_I8");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool gemv_tmap_eligible(const GemvArgs& a, int MT, int epi) {
  // K % 512: the scale / bias rows' byte stride (K / 32) must be a multiple of 16
  // for their tensor maps; the row's last 1024-column unit may be partial
  if (MT < 1 || MT > 8 || a.K % 512 || a.K <= 0) return false;
  if (tp_shape(MT, a.K, a.norm_w != nullptr, tp_use_i8()).sub == 0) return false;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  // activation rows and the norm weight arrive by bulk copy: 16-byte aligned
  if (!al(a.x) || (a.ldx % 8) || (a.norm_w && !al(a.norm_w))) return false;
  for (int i = 0; i < a.nseg; ++i) {
    if (!al(a.seg[i].w) || !al(a.seg[i].s) || !al(a.seg[i].b)) return false;
    if (epi == EPI_SWIGLU ? (a.seg[i].rows % 8) : (a.seg[i].rows % 16)) return false;
  }
  if (epi == EPI_SWIGLU && (a.nseg < 2 || a.seg[0].rows != a.total_rows || a.seg[1].rows != a.total_rows))
    return false;
  return encode_fn() != nullptr;
}

// Split-tile slots are sized for up to 8 virtual CTAs (rings) per SM.
constexpr int TP_MAX_CTAS_PER_SM = 8;

size_t gemv_part_floats() { return size_t(2) * 8 * 16 * TP_MAX_CTAS_PER_SM * sm_count(); }

// Resident CTAs per SM of one instantiation (setting its shared-memory
// opt-in first: the attribute belongs to each device's context).
template <int MT, int EPI, bool I8, int SUB>
static int tp_occupancy(size_t smem, int& per_sm) {
  auto kern = gemv_tmap_kernel<MT, EPI, I8, SUB>;
  static DeviceOnce once;
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TP_SMEM_MAX); }));
  per_sm = 0;
  M5_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, tp_threads(SUB), smem));
  per_sm = std::min(std::max(1, per_sm), TP_MAX_CTAS_PER_SM / SUB);
  return M5_OK;
}

// Grid of a launch: as many CTAs as stay resident, at most one ring per unit.
static int tp_grid(int per_sm, int sub, long long units) {
  return (int)std::max(1LL, std::min<long long>((long long)per_sm * sm_count(), (units + sub - 1) / sub));
}

static long long tp_units(const GemvArgs& a, int epi) {
  const int vrows = a.total_rows * (epi == EPI_SWIGLU ? 2 : 1);
  return (long long)(vrows / 16) * ((a.K / 64 + TP_UG - 1) / TP_UG);
}

template <int MT, int EPI, bool I8, int SUB>
static int tp_launch_s(const GemvArgs& a, const TmapSet& ts, const TpShape& sh, float* part, size_t part_floats,
                       int* cnt, cudaStream_t st) {
  int per_sm = 0;
  int rc = tp_occupancy<MT, EPI, I8, SUB>(sh.smem, per_sm);
  if (rc) return rc;
  const int grid = tp_grid(per_sm, SUB, tp_units(a, EPI));
  if (size_t(grid) * SUB * 2 * MT * 16 > part_floats) return fail(M5_ERR_INVALID, "gemv_tmap: split-tile slots too small");
  M5_CUDA(launch_pdl(gemv_tmap_kernel<MT, EPI, I8, SUB>, dim3(grid), dim3(tp_threads(SUB)), sh.smem, st, a, ts,
                     part, cnt, sh.nst));
  return M5_OK;
}

template <int MT, int EPI, bool I8>
static int tp_launch_t(const GemvArgs& a, const TmapSet& ts, float* part, size_t part_floats, int* cnt,
                       cudaStream_t st) {
  const TpShape sh = tp_shape(MT, a.K, a.norm_w != nullptr, I8);
  if (sh.sub == 1) return tp_launch_s<MT, EPI, I8, 1>(a, ts, sh, part, part_floats, cnt, st);
  if constexpr (I8) {
    if (sh.sub == 3) return tp_launch_s<MT, EPI, I8, 3>(a, ts, sh, part, part_floats, cnt, st);
  }
  return fail(M5_ERR_INVALID, "gemv_tmap: activations too large for shared memory");
}

template <int MT, bool I8>
static int tp_launch_epi(const GemvArgs& a, int epi, const TmapSet& ts, float* part, size_t pf, int* cnt,
                         cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: return tp_launch_t<MT, EPI_STORE, I8>(a, ts, part, pf, cnt, st);
    case EPI_RESIDUAL: return tp_launch_t<MT, EPI_RESIDUAL, I8>(a, ts, part, pf, cnt, st);
    case EPI_SWIGLU: return tp_launch_t<MT, EPI_SWIGLU, I8>(a, ts, part, pf, cnt, st);
    case EPI_F32: return tp_launch_t<MT, EPI_F32, I8>(a, ts, part, pf, cnt, st);
  }
  return fail(M5_ERR_INVALID, "gemv_tmap: bad epilogue");
}

int gemv_tmap_launch(const GemvArgs& a, int MT, int epi, float* part, size_t part_floats, int* cnt, int cnt_rows,
                     cudaStream_t st) {
  const int vrows = a.total_rows * (epi == EPI_SWIGLU ? 2 : 1);
  if (vrows > cnt_rows) return fail(M5_ERR_INVALID, "gemv_tmap: scratch too small for this matrix");
  if (!part) return fail(M5_ERR_INVALID, "gemv_tmap: no split-tile slots");
  TmapSet ts;
  memset(&ts, 0, sizeof(ts));
  for (int i = 0; i < a.nseg && i < 3; ++i) {
    int rc = make_maps(a.seg[i], a.K, ts, i, epi == EPI_SWIGLU ? 8 : 16);
    if (rc) return rc;
  }
  const bool i8 = tp_use_i8();
  switch (MT) {
    case 1: return i8 ? tp_launch_epi<1, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<1, false>(a, epi, ts, part, part_floats, cnt, st);
    case 2: return i8 ? tp_launch_epi<2, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<2, false>(a, epi, ts, part, part_floats, cnt, st);
    case 3: return i8 ? tp_launch_epi<3, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<3, false>(a, epi, ts, part, part_floats, cnt, st);
    case 4: return i8 ? tp_launch_epi<4, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<4, false>(a, epi, ts, part, part_floats, cnt, st);
    case 5: return i8 ? tp_launch_epi<5, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<5, false>(a, epi, ts, part, part_floats, cnt, st);
    case 6: return i8 ? tp_launch_epi<6, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<6, false>(a, epi, ts, part, part_floats, cnt, st);
    case 7: return i8 ? tp_launch_epi<7, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<7, false>(a, epi, ts, part, part_floats, cnt, st);
    case 8: return i8 ? tp_launch_epi<8, true>(a, epi, ts, part, part_floats, cnt, st)
                 : tp_launch_epi<8, false>(a, epi, ts, part, part_floats, cnt, st);
  }
  return fail(M5_ERR_INVALID, "gemv_tmap: MT must be 1..8");
}

int gemv_tmap_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_tmap_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_gemv_tmap_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace m5
