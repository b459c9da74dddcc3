// Device helpers shared by the tensor-core GEMVs: stage activation rows in
// mma B-fragment order (bf16 pairs (e, e+4) of every 8-element block) with
// 16-byte loads that are all issued before they are used, so staging costs a
// couple of L2 round trips instead of one per element.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "tma.cuh"

namespace m5 {

// xf[(t * NG + G) * 32 + tq * 8 + half * 4 + i] = pair(x[64G + 16tq + 8half + i], +4)
// xg[t * NG + G] = sum of the 64 staged (bf16-rounded) values of group G.
// Threads [0, NT) of the block participate; `bar` is the named barrier id used
// among them (0 = __syncthreads when NT is the whole block).
//
// FP16: the pairs are fp16 values x * 2^e_t with one power of two per token
// chosen so the token's largest |x| lands in [2^14, 2^15): exact for every
// value above max|x| * 2^-29 (bf16 has 8 significant bits, fp16 11), and
// 2^-e_t is written to xinv[t] for the caller to undo after the dot product.
// CG: read x through L2 only (rows another CTA of the same launch wrote).
template <int MT, int NT, bool FP16 = false, bool CG = false>
__device__ __forceinline__ void stage_frag(const bf16* __restrict__ x, int64_t ldx, int K,
                                           const bf16* __restrict__ norm_w, float eps, uint32_t* xf, float* xg,
                                           float* red, int bar, float* xinv = nullptr) {
  constexpr int CH = 8;  // 16-byte loads in flight per thread per pass
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NG = K >> 6, K8 = K >> 3;
  auto sync = [&]() {
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
  };
  float amax[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) amax[t] = 0.f;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + t * ldx);
    float inv = 1.f;
    if (norm_w) {
      float ss = 0.f;
      for (int c0 = tid; c0 < K8; c0 += NT * CH) {
        uint4 v[CH];
#pragma unroll
        for (int k = 0; k < CH; ++k)
          if (c0 + k * NT < K8) v[k] = CG ? __ldcg(xr + c0 + k * NT) : xr[c0 + k * NT];
#pragma unroll
        for (int k = 0; k < CH; ++k)
          if (c0 + k * NT < K8) {
            const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float a = bf16_lo(w[q]), b = bf16_hi(w[q]);
              ss = fmaf(a, a, fmaf(b, b, ss));
            }
          }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      sync();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NT / 32; ++w) tot += red[w];
      inv = __frsqrt_rn(__fadd_rn(tot / float(K), eps));
      sync();
    }
    const uint4* nw = reinterpret_cast<const uint4*>(norm_w);
    for (int c0 = tid; c0 < K8; c0 += NT * CH) {
      uint4 v[CH], wv[CH];
#pragma unroll
      for (int k = 0; k < CH; ++k)
        if (c0 + k * NT < K8) {
          v[k] = CG ? __ldcg(xr + c0 + k * NT) : xr[c0 + k * NT];
          if (norm_w) wv[k] = nw[c0 + k * NT];
        }
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const int c = c0 + k * NT;  // 8-element block index
        if (c < K8) {
          float e[8];
          const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            e[2 * q] = bf16_lo(w[q]);
            e[2 * q + 1] = bf16_hi(w[q]);
          }
          if (norm_w) {
            const uint32_t n[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              e[2 * q] = rbf(__fmul_rn(bf16_lo(n[q]), rbf(__fmul_rn(e[2 * q], inv))));
              e[2 * q + 1] = rbf(__fmul_rn(bf16_hi(n[q]), rbf(__fmul_rn(e[2 * q + 1], inv))));
            }
          }
          if (FP16) {
#pragma unroll
            for (int q = 0; q < 8; ++q) amax[t] = fmaxf(amax[t], fabsf(e[q]));
          }
          uint4 o;
          o.x = uint32_t(__bfloat16_as_ushort(f2bf(e[0]))) | (uint32_t(__bfloat16_as_ushort(f2bf(e[4]))) << 16);
          o.y = uint32_t(__bfloat16_as_ushort(f2bf(e[1]))) | (uint32_t(__bfloat16_as_ushort(f2bf(e[5]))) << 16);
          o.z = uint32_t(__bfloat16_as_ushort(f2bf(e[2]))) | (uint32_t(__bfloat16_as_ushort(f2bf(e[6]))) << 16);
          o.w = uint32_t(__bfloat16_as_ushort(f2bf(e[3]))) | (uint32_t(__bfloat16_as_ushort(f2bf(e[7]))) << 16);
          const int G = c >> 3, tq = (c >> 1) & 3, half = c & 1;
          *reinterpret_cast<uint4*>(xf + (t * NG + G) * 32 + tq * 8 + half * 4) = o;
        }
      }
    }
  }
  sync();
  // group sums: 4 threads per (token, group), 8 pairs each.  The loop is
  // warp-uniform (every lane reaches the shuffles) whatever MT * NG is.
  const int total = MT * NG * 4;
  for (int q0 = tid - lane; q0 < total; q0 += NT) {
    const int q = q0 + lane;
    float s = 0.f;
    if (q < total) {
      const uint32_t* p = xf + (q >> 2) * 32 + (q & 3) * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += bf16_lo(p[j]) + bf16_hi(p[j]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (q < total && (q & 3) == 0) xg[q >> 2] = s;
  }
  if constexpr (FP16) {
    // per-token max |x| -> power-of-two scale, then convert the pairs in place
    float* rm = red + 32;  // [NT / 32][MT]
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const float m = warp_max(amax[t]);
      if (lane == 0) rm[warp * MT + t] = m;
    }
    sync();
    float sc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float m = 0.f;
#pragma unroll
      for (int w = 0; w < NT / 32; ++w) m = fmaxf(m, rm[w * MT + t]);
      // m = 1.f * 2^(E - 127): m * 2^(141 - E) lies in [2^14, 2^15)
      const int E = int((__float_as_uint(m) >> 23) & 0xFFu);
      const int ex = m > 0.f ? max(-126, min(126, 141 - E)) : 0;
      sc[t] = __uint_as_float(uint32_t(ex + 127) << 23);
      if (tid == 0 && xinv) xinv[t] = __uint_as_float(uint32_t(127 - ex) << 23);
    }
    const int words = MT * NG * 32;
    for (int i = tid; i < words; i += NT) {
      const int t = i / (NG * 32);
      float f = 1.f;
#pragma unroll
      for (int tt = 0; tt < MT; ++tt)
        if (tt == t) f = sc[tt];
      const uint32_t w = xf[i];
      __half2 h = __floats2half2_rn(bf16_lo(w) * f, bf16_hi(w) * f);
      xf[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  sync();
}

// The fp16 variant of stage_frag<MT, NT, true> for the TMA-fed GEMV, with the
// activation rows (and the norm weight) brought into shared memory by one
// bulk copy each, in two passes over the row:
//   1. per token, the sum of squares (RMSNorm) and a bound on the largest
//      staged magnitude, max_i |x_i w_i| * inv (or max_i |x_i|): the power-of-
//      two scale only has to keep the scaled maximum inside fp16 range, and the
//      bound is within 2^-7 of the true maximum, so the scaled maximum stays
//      below 2^15 * 1.01;
//   2. per 8-element block: normalize and round to bf16 exactly as the model
//      does, convert the pairs (e0,e4)(e1,e5)(e2,e6)(e3,e7) to fp16 with the
//      scale, and sum the group (the 8 lanes 8j..8j+7 hold one 64-element
//      group) with three shuffles.
// The raw bf16 row of token t is copied to xf + t * NG * 32: the uint4 of raw
// 8-element block c sits exactly where the pairs of block c go, so every
// thread converts its blocks in place.  Requirements: x rows and norm_w
// 16-byte aligned (ldx % 8 == 0), K % 256 == 0, nbuf holds K bf16 when
// norm_w is set, xbar is an initialised, unused mbarrier, red has room for
// 8 + 32 * MT floats (up to 16 staging warps).  Returns false (and records a device error) if the copy
// did not land in time.
template <int MT, int NT, bool FP16>
__device__ __forceinline__ bool stage_frag_bulk(const bf16* __restrict__ x, int64_t ldx, int K,
                                                const bf16* __restrict__ norm_w, float eps, uint32_t* xf,
                                                uint32_t* nbuf, float* xg, float* red, int bar, float* xinv,
                                                uint64_t* xbar, int* err) {
  static_assert(FP16 && NT % 32 == 0 && NT / 32 <= 16, "fp16 staging by whole warps");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NG = K >> 6, K8 = K >> 3;
  auto sync = [&]() {
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
  };
  if (tid == 0) {
    const uint32_t row = uint32_t(K) * 2u;
    mbar_arrive_expect_tx(xbar, MT * row + (norm_w ? row : 0u));
#pragma unroll
    for (int t = 0; t < MT; ++t) bulk_g2s(xf + size_t(t) * NG * 32, x + size_t(t) * ldx, row, xbar);
    if (norm_w) bulk_g2s(nbuf, norm_w, row, xbar);
  }
  const bool ok = mbar_wait(xbar, 0, err);
  const uint4* nw = reinterpret_cast<const uint4*>(nbuf);
  // ---- pass 1: sum of squares and max |x w| per token
  // red[0..MT) receives xinv while other threads still read the partials:
  // the partials live past it
  float* rs = red + 8;           // [NT/32][MT] sums of squares
  float* rm = red + 8 + 16 * MT;  // [NT/32][MT] maxima
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const uint4* blk = reinterpret_cast<const uint4*>(xf + size_t(t) * NG * 32);
    float ss = 0.f, mx = 0.f;
    for (int c = tid; c < K8; c += NT) {
      const uint4 v = blk[c];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      if (norm_w) {
        const uint4 nv = nw[c];
        const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float a = bf16_lo(w[q]), b = bf16_hi(w[q]);
          ss = fmaf(a, a, fmaf(b, b, ss));
          mx = fmaxf(mx, fmaxf(fabsf(a * bf16_lo(n[q])), fabsf(b * bf16_hi(n[q]))));
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) mx = fmaxf(mx, fmaxf(fabsf(bf16_lo(w[q])), fabsf(bf16_hi(w[q]))));
      }
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if (lane == 0) {
      rs[warp * MT + t] = ss;
      rm[warp * MT + t] = mx;
    }
  }
  sync();
  float inv[MT], sc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    float tot = 0.f, m = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) {
      tot += rs[w * MT + t];
      m = fmaxf(m, rm[w * MT + t]);
    }
    inv[t] = norm_w ? __frsqrt_rn(__fadd_rn(tot / float(K), eps)) : 1.f;
    m *= inv[t];
    const int E = int((__float_as_uint(m) >> 23) & 0xFFu);
    const int ex = m > 0.f ? max(-126, min(126, 141 - E)) : 0;
    sc[t] = __uint_as_float(uint32_t(ex + 127) << 23);
    if (tid == 0 && xinv) xinv[t] = __uint_as_float(uint32_t(127 - ex) << 23);
  }
  // ---- pass 2: normalize, round, convert, group sums (warp-uniform loop)
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    uint4* blk = reinterpret_cast<uint4*>(xf + size_t(t) * NG * 32);
    for (int c0 = tid - lane; c0 < K8; c0 += NT) {
      const int c = c0 + lane;
      const uint4 v = blk[c];
      float e[8];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        e[2 * q] = bf16_lo(w[q]);
        e[2 * q + 1] = bf16_hi(w[q]);
      }
      if (norm_w) {
        const uint4 nv = nw[c];
        const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          e[2 * q] = rbf(__fmul_rn(bf16_lo(n[q]), rbf(__fmul_rn(e[2 * q], inv[t]))));
          e[2 * q + 1] = rbf(__fmul_rn(bf16_hi(n[q]), rbf(__fmul_rn(e[2 * q + 1], inv[t]))));
        }
      }
      float gs = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) gs += e[q];
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      gs += __shfl_xor_sync(0xffffffffu, gs, 4);
      if ((lane & 7) == 0) xg[t * NG + (c >> 3)] = gs;
      const float f = sc[t];
      uint4 o;
      __half2 h = __floats2half2_rn(e[0] * f, e[4] * f);
      o.x = *reinterpret_cast<uint32_t*>(&h);
      h = __floats2half2_rn(e[1] * f, e[5] * f);
      o.y = *reinterpret_cast<uint32_t*>(&h);
      h = __floats2half2_rn(e[2] * f, e[6] * f);
      o.z = *reinterpret_cast<uint32_t*>(&h);
      h = __floats2half2_rn(e[3] * f, e[7] * f);
      o.w = *reinterpret_cast<uint32_t*>(&h);
      blk[c] = o;  // pairs of block c occupy the bytes its raw values came from
    }
  }
  sync();
  return ok;
}


// Block c (8 values e, already normalised and bf16-rounded) of token t in
// the int8 plane layout described below; the 8 lanes of a group (lanes
// 8j..8j+7 hold its blocks) reduce its sum and maximum by shuffles, and every
// lane of the warp must call this with its own block.  The planes are written
// over the raw block's words after a __syncwarp, so a warp whose 32 raw
// blocks are all in registers converts them in place.
__device__ __forceinline__ void i8_block(const float (&e)[8], int c, int t, int NG, uint32_t* xq, float* xg,
                                         float* xs, int lane) {
  float gs = 0.f, gm = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    gs += e[q];
    gm = fmaxf(gm, fabsf(e[q]));
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    gs += __shfl_xor_sync(0xffffffffu, gs, o);
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
  }
  const int G = c >> 3, cb = c & 7;  // group, block inside it
  const int E = int((__float_as_uint(gm) >> 23) & 0xFFu);  // biased exponent of the group max
  const int sh = gm > 0.f ? 141 - E : 0;                   // 2^(14 - (E - 127))
  const float up = __uint_as_float(uint32_t(max(1, min(254, sh + 127))) << 23);
  if (cb == 0) {
    xg[t * NG + G] = gs;
    xs[t * NG + G] = __uint_as_float(uint32_t(max(1, min(254, 127 - sh))) << 23);
  }
  // v = rint(e * up) by one fma against 1.5 * 2^23 (|e * up| < 2^15, so the
  // single round-to-nearest-even lands on the integer): the sum's low
  // mantissa bits hold v + 2^22, whose byte 0 is v's low byte and byte 1
  // its high byte (two's complement); byte permutes gather four of each.
  uint32_t f[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) f[q] = __float_as_uint(fmaf(e[q], up, 12582912.f));
  uint32_t hi[2], lo[2];  // r = 0 even, 1 odd elements
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lo[r] = __byte_perm(__byte_perm(f[r], f[r + 2], 0x0040), __byte_perm(f[r + 4], f[r + 6], 0x0040), 0x5410);
    hi[r] = __byte_perm(__byte_perm(f[r], f[r + 2], 0x0051), __byte_perm(f[r + 4], f[r + 6], 0x0051), 0x5410);
  }
  __syncwarp();  // every raw block of this warp's groups is in registers
  const int tq = cb >> 1, m = cb & 1;
  uint32_t* dst = xq + (size_t(t) * NG + G) * 32 + tq * 8 + m * 2;
  *reinterpret_cast<uint2*>(dst) = make_uint2(hi[0], hi[1]);
  *reinterpret_cast<uint2*>(dst + 4) = make_uint2(lo[0], lo[1]);
}

// Activation staging for the int8 tensor-core GEMV (mma.sync m16n8k32, u8
// weight codes against s8 / u8 activation planes), with the same bulk copy,
// RMSNorm and bf16 rounding points as stage_frag_bulk.  Per token t and
// 64-element group G the normalised bf16 values become 16-bit fixed point
//   v = rint(x * 2^(14 - E)),  E = exponent of the group's largest |x|,
// so |v| < 2^15 and every value at or above 2^-7 of the group's maximum is
// exact (bf16 keeps 8 significant bits); v = 256 hi + lo with hi s8, lo u8.
// xs[t * NG + G] = 2^(E - 14) undoes the scale, xg[t * NG + G] is the fp32
// sum of the group's bf16 values (the bias term).  Layout of the planes,
// 32 words per (t, G) like the fp16 pairs:
//   xq[(t*NG + G)*32 + tq*8 + plane*4 + m*2 + r],  plane 0 = hi, 1 = lo,
//   m = MMA (k 16tq..16tq+7 or 16tq+8..16tq+15), r = 0 even / 1 odd elements
// of that 8-element block, 4 bytes each -- the B fragment (b0, b1) of the
// MMA in which lane quad tq reads the weight word 2tq + m of the group.
// Each warp converts whole groups (8 lanes per group, one 8-element block
// each) and reads its 32 raw blocks into registers before any lane writes,
// so the conversion is in place.  Requirements as for stage_frag_bulk.
template <int MT, int NT>
__device__ __forceinline__ bool stage_i8_bulk(const bf16* __restrict__ x, int64_t ldx, int K,
                                              const bf16* __restrict__ norm_w, float eps, uint32_t* xq,
                                              uint32_t* nbuf, float* xg, float* xs, float* red, int bar,
                                              uint64_t* xbar, int* err) {
  static_assert(NT % 32 == 0 && NT / 32 <= 16, "int8 staging by whole warps");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NG = K >> 6, K8 = K >> 3;
  auto sync = [&]() {
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
  };
  if (tid == 0) {
    const uint32_t row = uint32_t(K) * 2u;
    mbar_arrive_expect_tx(xbar, MT * row + (norm_w ? row : 0u));
#pragma unroll
    for (int t = 0; t < MT; ++t) bulk_g2s(xq + size_t(t) * NG * 32, x + size_t(t) * ldx, row, xbar);
    if (norm_w) bulk_g2s(nbuf, norm_w, row, xbar);
  }
  const bool ok = mbar_wait(xbar, 0, err);
  const uint4* nw = reinterpret_cast<const uint4*>(nbuf);
  float inv[MT];
  if (norm_w) {
    float* rs = red + 8;  // [NT/32][MT] sums of squares
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const uint4* blk = reinterpret_cast<const uint4*>(xq + size_t(t) * NG * 32);
      float ss = 0.f;
      for (int c = tid; c < K8; c += NT) {
        const uint4 v = blk[c];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float a = bf16_lo(w[q]), b = bf16_hi(w[q]);
          ss = fmaf(a, a, fmaf(b, b, ss));
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) rs[warp * MT + t] = ss;
    }
    sync();
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NT / 32; ++w) tot += rs[w * MT + t];
      inv[t] = __frsqrt_rn(__fadd_rn(tot / float(K), eps));
    }
  } else {
#pragma unroll
    for (int t = 0; t < MT; ++t) inv[t] = 1.f;
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    uint4* blk = reinterpret_cast<uint4*>(xq + size_t(t) * NG * 32);
    for (int c0 = tid - lane; c0 < K8; c0 += NT) {  // K8 % 32 == 0: whole warps, whole groups
      const int c = c0 + lane;
      const uint4 v = blk[c];
      float e[8];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        e[2 * q] = bf16_lo(w[q]);
        e[2 * q + 1] = bf16_hi(w[q]);
      }
      if (norm_w) {
        const uint4 nv = nw[c];
        const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          e[2 * q] = rbf(__fmul_rn(bf16_lo(n[q]), rbf(__fmul_rn(e[2 * q], inv[t]))));
          e[2 * q + 1] = rbf(__fmul_rn(bf16_hi(n[q]), rbf(__fmul_rn(e[2 * q + 1], inv[t]))));
        }
      }
      i8_block(e, c, t, NG, xq, xg, xs, lane);
    }
  }
  sync();
  return ok;
}

}  // namespace m5
