// Routed experts of one decode token on the tensor cores (kernel K6, T = 1).
//
// The expert projections run the register-prefetch MMA scheme of gemv_mma.cu
// (mma.sync m16n8k16 bf16, codes as exact (128 + q) pairs, per-group fold
// s*D + (b - 128 s)*sum(x), up to MX_PIPE (tile, group) steps of loads in
// flight per warp) over the rows of the routed experts only, and every tile
// is finished inside one CTA: the CTA's 8 warps split its tiles' steps, write
// their partial sums to shared memory and the tile is their sum in warp order
// (no global atomics, no fences, a fixed summation order):
//   gate/up - tile = 8 gate rows + the 8 matching up rows of one routed
//             expert, a few whole tiles per CTA (about two CTAs per SM);
//             input RMSNorm(h) staged once per CTA; the tile's SwiGLU rows
//             bf16(bf16(g * bf16(sigmoid g)) * u) (mlx-lm) go to
//             act[slot][I];
//   down    - one CTA per 16 output rows, all local slots: the k SwiGLU rows
//             are staged as the k B-columns of the MMA, tile ls (16 rows of
//             slot ls's expert) keeps its own column, and the CTA adds the
//             slots in slot order, h += bf16(sum_j bf16(bf16(y_j) * score_j))
//             (mlx-lm Qwen3MoeSparseMoeBlock), or writes the fp32 sum as this
//             rank's partial under expert parallelism.
// Only experts in [e_first, e_first + e_local) are streamed; each CTA lists
// the token's local slots from the router ids, so no host sync is needed.
#include <algorithm>

#include "frag_stage.cuh"
#include "gemv.cuh"
#include "gemv_impl.cuh"
#include "mma_dq.cuh"
#include "moe.cuh"

namespace m5 {

constexpr int MX_W = 8;     // warps per CTA
constexpr int MX_PIPE = 12;  // steps prefetched per warp
constexpr int MX_KMAX = 8;   // routed experts per token this path supports

// local slots of the token: ls -> (slot, local expert index); returns their
// count.  Lanes 0..k-1 of warp 0 read the k ids in one load and compact the
// local ones with a ballot, in slot order.
__device__ __forceinline__ int mx_local_slots(const MoeArgs& a, int* s_slot, int* s_eid, int* s_n) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int e = lane < a.k ? a.ids[lane] - a.e_first : -1;
    const bool local = lane < a.k && e >= 0 && e < a.e_local;
    const unsigned m = __ballot_sync(0xffffffffu, local);
    if (local) {
      const int pos = __popc(m & ((1u << lane) - 1u));
      s_slot[pos] = lane;
      s_eid[pos] = e;
    }
    if (lane == 0) *s_n = __popc(m);
  }
  __syncthreads();
  return *s_n;
}

// One warp's walk over steps [s_begin, s_end) of (tile, 64-column group):
// row_of(tile, r16) gives the weight row (and its matrix) of tile row r16,
// flush(tile, tot, done) receives the warp's partial sums of a tile.
template <int MT, class RowOf, class Flush>
__device__ __forceinline__ void mx_walk(long long s_begin, long long s_end, int K, const uint32_t* xf,
                                        const float* xg, RowOf row_of, Flush flush) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int NG = K >> 6;
  const size_t K8 = K >> 3, K64 = K >> 6;
  const int tok = g < MT ? g : MT - 1;  // B column n = g reads this token (slot)
  const uint32_t* xfl = xf + tok * NG * 32 + tq * 8;

  long long is = s_begin;
  int it_tile = int(is / NG), it_G = int(is % NG);
  const uint32_t *w_g = nullptr, *w_g8 = nullptr;
  const bf16 *s_g = nullptr, *b_g = nullptr, *s_g8 = nullptr, *b_g8 = nullptr;
  auto set_tile = [&](int tile) {
    QW m;
    size_t rr;
    row_of(tile, g, m, rr);
    w_g = m.w + rr * K8 + 2 * tq;
    s_g = m.s + rr * K64;
    b_g = m.b + rr * K64;
    row_of(tile, g + 8, m, rr);
    w_g8 = m.w + rr * K8 + 2 * tq;
    s_g8 = m.s + rr * K64;
    b_g8 = m.b + rr * K64;
  };
  set_tile(it_tile);
  uint2 rw[MX_PIPE], rw8[MX_PIPE];
  uint32_t rsb[MX_PIPE], rsb8[MX_PIPE];
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
  for (int s = 0; s < MX_PIPE; ++s) issue(s);

  int c_tile = int(s_begin / NG), c_G = int(s_begin % NG), c_done = 0;
  float tot[4] = {0.f, 0.f, 0.f, 0.f};  // (g, 2t) (g, 2t+1) (g8, 2t) (g8, 2t+1)
  const float* xgl0 = xg + (2 * tq < MT ? 2 * tq : MT - 1) * NG;
  const float* xgl1 = xg + (2 * tq + 1 < MT ? 2 * tq + 1 : MT - 1) * NG;
  for (long long s0 = s_begin; s0 < s_end; s0 += MX_PIPE) {
#pragma unroll
    for (int slot = 0; slot < MX_PIPE; ++slot) {
      if (s0 + slot < s_end) {
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
          flush(c_tile, tot, c_done);
#pragma unroll
          for (int i = 0; i < 4; ++i) tot[i] = 0.f;
          c_done = 0;
          c_G = 0;
          ++c_tile;
        }
      }
    }
  }
  if (c_done) flush(c_tile, tot, c_done);
}

// This CTA's whole tiles [tile0, tile0 + ntile) of NG steps each: the warps
// split the steps evenly (contiguous ranges), and each warp's partial sum of
// a tile lands in part[(tile - tile0) * MX_W + warp][16] (rows; the B column
// col_of(tile) of the MMA).  Slots no warp writes stay zero.  After the
// trailing barrier every tile's rows are the sum of its MX_W partials, added
// by the caller in warp order: no global atomics, a fixed summation order.
template <int MT, class RowOf, class ColOf>
__device__ __forceinline__ void mx_cta_tiles(int tile0, int ntile, int K, const uint32_t* xf, const float* xg,
                                             float* part, RowOf row_of, ColOf col_of) {
  const int NG = K >> 6, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  for (int i = threadIdx.x; i < ntile * MX_W * 16; i += blockDim.x) part[i] = 0.f;
  __syncthreads();
  const long long steps = (long long)ntile * NG;
  const long long b = (long long)tile0 * NG + steps * warp / MX_W, e = (long long)tile0 * NG + steps * (warp + 1) / MX_W;
  auto flush = [&](int tile, const float (&tot)[4], int) {
    const int j = col_of(tile);
    if ((j >> 1) == tq) {
      float* p = part + ((tile - tile0) * MX_W + warp) * 16;
      p[g] = tot[j & 1];
      p[g + 8] = tot[2 + (j & 1)];
    }
  };
  if (b < e) mx_walk<MT>(b, e, K, xf, xg, row_of, flush);
  __syncthreads();
}

// Sum of the MX_W warp partials of local tile t, row r (warp order).
__device__ __forceinline__ float mx_tile_sum(const float* part, int t, int r) {
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < MX_W; ++w) v += part[(t * MX_W + w) * 16 + r];
  return v;
}

// Gate/up of the token's local slots (nl of them, slot / local expert lists in
// shared memory): this CTA takes `tpc` whole (slot, 8-row) tiles; the tile's
// SwiGLU rows bf16(bf16(g * bf16(sigmoid g)) * u) (mlx-lm) go to act[slot][I].
__device__ __forceinline__ void mx_gu_body(const MoeArgs& a, int nl, const int* s_slot, const int* s_eid, int tpc,
                                           unsigned char* smem_raw) {
  const int H = a.H, I = a.I, NG = H >> 6;
  const int tpe = I / 8;  // tiles per expert
  uint32_t* xf = reinterpret_cast<uint32_t*>(smem_raw);  // [NG][4][8] bf16 pairs
  float* xg = reinterpret_cast<float*>(xf + NG * 32);    // [NG]
  float* red = xg + NG;                                  // [33]
  float* part = red + 33;                                // [tpc][MX_W][16]
  // every thread of the CTA stages (the staging synchronises the CTA)
  stage_frag<1, MX_W * 32>(a.x, H, H, a.norm_w, a.eps, xf, xg, red, 0);
  const int tile0 = blockIdx.x * tpc;
  const int ntile = min(tpc, nl * tpe - tile0);
  if (ntile <= 0) return;  // CTA-uniform
  auto row_of = [&](int tile, int r16, QW& m, size_t& rr) {
    const int ls = tile / tpe, rt = tile % tpe;
    m = r16 < 8 ? a.gate : a.up;
    rr = size_t(s_eid[ls]) * I + rt * 8 + (r16 & 7);
  };
  mx_cta_tiles<1>(tile0, ntile, H, xf, xg, part, row_of, [](int) { return 0; });
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < ntile; t += MX_W) {
    if (lane < 8) {
      const float gv = rbf(mx_tile_sum(part, t, lane)), uv = rbf(mx_tile_sum(part, t, lane + 8));
      const float sg = rbf(1.f / (1.f + expf(-gv)));
      const int tile = tile0 + t, ls = tile / tpe, rt = tile % tpe;
      a.act[size_t(s_slot[ls]) * I + rt * 8 + lane] = f2bf(rbf(gv * sg) * uv);
    }
  }
}

// Down projection of the nl local slots for the 16 output rows nb * 16 ..
// (nb = blockIdx.x): the k SwiGLU rows are staged as the MMA's B columns and
// tile ls (16 rows of local slot ls's expert) keeps column s_slot[ls]; then
// h += bf16(sum_j bf16(bf16(y_j) * score_j)) over the slots in slot order
// (mlx-lm Qwen3MoeSparseMoeBlock), or the fp32 sum as this rank's partial
// under expert parallelism.
template <int MT>
__device__ __forceinline__ void mx_down_body(const MoeArgs& a, int nl, const int* s_slot, const int* s_eid,
                                             unsigned char* smem_raw) {
  const int H = a.H, I = a.I, NG = I >> 6;
  uint32_t* xf = reinterpret_cast<uint32_t*>(smem_raw);  // [MT][NG][4][8]
  float* xg = reinterpret_cast<float*>(xf + MT * NG * 32);  // [MT][NG]
  float* red = xg + MT * NG;                                // [33]
  float* part = red + 33;                                   // [nl][MX_W][16]
  stage_frag<MT, MX_W * 32>(a.act, I, I, nullptr, 0.f, xf, xg, red, 0);
  const int nb = blockIdx.x;
  auto row_of = [&](int tile, int r16, QW& m, size_t& rr) {
    m = a.down;
    rr = size_t(s_eid[tile]) * H + nb * 16 + r16;
  };
  mx_cta_tiles<MT>(0, nl, I, xf, xg, part, row_of, [&](int tile) { return s_slot[tile]; });
  if (threadIdx.x < 16) {
    const int r = threadIdx.x, n = nb * 16 + r;
    float sum = 0.f;
    for (int ls = 0; ls < nl; ++ls)
      sum += rbf(rbf(mx_tile_sum(part, ls, r)) * bf2f(a.scores[s_slot[ls]]));
    if (a.partial) {
      a.partial[n] = sum;
    } else {
      bf16* o = a.h + n;
      *o = f2bf(bf2f(*o) + rbf(sum));
    }
  }
}

__global__ void __launch_bounds__(MX_W * 32, 2) moe_gu_mma_kernel(const MoeArgs a, const int tpc) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int s_slot[MX_KMAX], s_eid[MX_KMAX], s_n;
  const int nl = mx_local_slots(a, s_slot, s_eid, &s_n);
  if (nl == 0) return;
  mx_gu_body(a, nl, s_slot, s_eid, tpc, smem_raw);
}

template <int MT>
__global__ void __launch_bounds__(MX_W * 32, 2) moe_down_mma_kernel(const MoeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int s_slot[MX_KMAX], s_eid[MX_KMAX], s_n;
  const int nl = mx_local_slots(a, s_slot, s_eid, &s_n);
  if (nl == 0) {  // no expert of this token is local: this rank's share is zero
    if (a.partial && threadIdx.x < 16) a.partial[blockIdx.x * 16 + threadIdx.x] = 0.f;
    return;
  }
  mx_down_body<MT>(a, nl, s_slot, s_eid, smem_raw);
}

// Softmax (fp32, rounded to bf16) and top-k of the E router logits by one
// full warp (highest probability first, ties -> lower expert id), scores
// renormalised when norm_topk; writes ids[0..k) and scores[0..k).
template <class Logit>
__device__ __forceinline__ void router_topk_warp(const MoeRouterArgs& a, Logit logit) {
  const int lane = threadIdx.x & 31, E = a.E;
  constexpr int PER = 8;  // E <= 256
  float v[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? logit(e) : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    v[j] = (lane + 32 * j < E) ? expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
  sum = warp_sum(sum);
#pragma unroll
  for (int j = 0; j < PER; ++j) v[j] = (lane + 32 * j < E) ? rbf(__fdiv_rn(v[j], sum)) : -INFINITY;
  float chosen = 0.f, my_score = 0.f;
  int my_id = -1;
  for (int r = 0; r < a.k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (v[j] > bv || (v[j] == bv && e < bi))) {
        bv = v[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (lane + 32 * j == bi) v[j] = -INFINITY;
    chosen += bv;
    if (lane == r) {
      my_score = bv;
      my_id = bi;
    }
  }
  if (lane < a.k) {
    float sc = my_score;
    if (a.norm_topk) sc = rbf(__fdiv_rn(sc, rbf(chosen)));
    a.ids[lane] = my_id;
    a.scores[lane] = f2bf(sc);
  }
}

// Router + top-k of one decode token in one launch: each warp takes one of
// the E router rows (RMSNorm(h) staged once per CTA, CUDA-core dot product as
// moe.cu), rounds the logit to bf16 like the router projection's output, and
// the last CTA to finish (a zeroed counter it leaves zeroed) runs the top-k:
// softmax in fp32 rounded to bf16, the k largest probabilities (ties -> lower
// expert id) in order, renormalised when norm_topk (same rules as
// moe_topk_kernel for one token).
constexpr int RT_W = 8;
__global__ void __launch_bounds__(RT_W * 32) moe_router_topk_kernel(const MoeRouterArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) float rsm[];
  const int H = a.H, E = a.E;
  float* xs = rsm;
  float* xsum = xs + H;
  float* red = xsum + (H >> 5);
  const int lane = threadIdx.x & 31, row = blockIdx.x * RT_W + (threadIdx.x >> 5);
  const size_t H8 = H >> 3, H64 = H >> 6;
  // The row's codes, scales and biases depend on nothing earlier: for rows of
  // up to 4096 columns (4 16-byte blocks per lane) they are loaded before the
  // staging, so their round trip overlaps it; the sum below is row_dot's, in
  // its order.
  constexpr int RU = 4;
  const int K32 = H >> 5;
  const bool pre = K32 <= 32 * RU;
  uint4 wv[RU];
  float sv[RU], bv[RU];
  if (row < E && pre) {
    const uint4* wr = reinterpret_cast<const uint4*>(a.w + row * H8);
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      const int i = lane + 32 * u;
      if (i < K32) {
        wv[u] = ldg_stream(wr + i);
        sv[u] = bf2f(a.s[row * H64 + (i >> 1)]);
        bv[u] = bf2f(a.b[row * H64 + (i >> 1)]);
      }
    }
  }
  stage_rows<1>(a.x, H, H, a.norm_w, a.eps, xs, xsum, red);
  if (row < E) {
    float acc[1] = {0.f};
    if (pre) {
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int i = lane + 32 * u;
        if (i < K32) {
          const float off = fmaf(-128.f, sv[u], bv[u]);
          acc[0] = fmaf(sv[u], dot32(wv[u], xs, i), fmaf(off, xsum[i], acc[0]));
        }
      }
    } else {
      row_dot<1, 4>(a.w + row * H8, a.s + row * H64, a.b + row * H64, H, xs, xsum, acc);
    }
    const float v = rbf(warp_sum(acc[0]));
    if (lane == 0) a.logits[row] = f2bf(v);
  }
  __threadfence();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(a.counter, 1) == int(gridDim.x) - 1;
  __syncthreads();
  if (!last || threadIdx.x >= 32) return;
  __threadfence();
  router_topk_warp(a, [&](int e) { return bf2f(__ldcg(a.logits + e)); });
  if (lane == 0) *a.counter = 0;
}

int moe_router_topk_launch(const MoeRouterArgs& a, cudaStream_t st) {
  if (a.E > 256 || a.k <= 0 || a.k > 32 || a.k > a.E || a.H % 256) return fail(M5_ERR_INVALID, "moe router: shape");
  const size_t smem = size_t(a.H) * 4 + size_t(a.H / 32) * 4 + 33 * 4;
  static DeviceOnce once;  // the attribute belongs to each device's context
  M5_CUDA(once.run([&] { return cudaFuncSetAttribute(moe_router_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024); }));
  if (smem > 100 * 1024) return fail(M5_ERR_INVALID, "moe router: hidden size too large");
  M5_CUDA(launch_pdl(moe_router_topk_kernel, dim3(ceil_div(a.E, RT_W)), dim3(RT_W * 32), smem, st, a));
  M5_LAUNCH_CHECK("moe router/top-k launch");
  return M5_OK;
}

// staged activations, group sums, staging scratch, then the tile partials
static size_t mx_smem(int MT, int K, int tiles) {
  return size_t(MT) * (K / 64) * 32 * 4 + size_t(MT) * (K / 64) * 4 + 33 * 4 + size_t(tiles) * MX_W * 16 * 4;
}
// Whole (slot, 8-row) gate/up tiles per CTA: about two CTAs per SM.
static int mx_gu_tpc(const MoeArgs& a) {
  const long long tiles = (long long)a.k * (a.I / 8);
  return (int)std::max(1LL, (tiles + 2LL * sm_count() - 1) / (2LL * sm_count()));
}


bool moe_mma_eligible(const MoeArgs& a) {
  return a.T == 1 && a.k == MX_KMAX && a.H % 64 == 0 && a.I % 64 == 0 && a.I % 8 == 0 && a.H % 16 == 0 &&
         mx_smem(MX_KMAX, a.I, MX_KMAX) <= 200 * 1024 && mx_smem(1, a.H, mx_gu_tpc(a)) <= 200 * 1024;
}

int moe_mma_launch(const MoeArgs& a, cudaStream_t st) {
  static DeviceOnce once;  // the attributes belong to each device's context
  M5_CUDA(once.run([&] {
    cudaError_t e = cudaFuncSetAttribute(moe_gu_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(moe_down_mma_kernel<MX_KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024);
  }));
  {
    // grid for all k slots; CTAs past the local slots' tiles leave at once
    const int tpc = mx_gu_tpc(a);
    const int grid = (int)std::max(1LL, ((long long)a.k * (a.I / 8) + tpc - 1) / tpc);
    M5_CUDA(launch_pdl(moe_gu_mma_kernel, dim3(grid), dim3(MX_W * 32), mx_smem(1, a.H, tpc), st, a, tpc));
    M5_LAUNCH_CHECK("moe gate/up (tensor core) launch");
  }
  {
    const int grid = a.H / 16;  // one CTA per 16 output rows, every local slot
    M5_CUDA(launch_pdl(moe_down_mma_kernel<MX_KMAX>, dim3(grid), dim3(MX_W * 32), mx_smem(MX_KMAX, a.I, MX_KMAX), st,
                       a));
    M5_LAUNCH_CHECK("moe down (tensor core) launch");
  }
  return M5_OK;
}

}  // namespace m5
