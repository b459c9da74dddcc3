// Device helpers shared by the tensor-core GEMVs: stage activation rows in
// mma B-fragment order (bf16 pairs (e, e+4) of every 8-element block) with
// 16-byte loads that are all issued before they are used, so staging costs a
// couple of L2 round trips instead of one per element.
#pragma once

#include "common.cuh"

namespace m5 {

// xf[(t * NG + G) * 32 + tq * 8 + half * 4 + i] = pair(x[64G + 16tq + 8half + i], +4)
// xg[t * NG + G] = sum of the 64 staged (bf16-rounded) values of group G.
// Threads [0, NT) of the block participate; `bar` is the named barrier id used
// among them (0 = __syncthreads when NT is the whole block).
template <int MT, int NT>
__device__ __forceinline__ void stage_frag(const bf16* __restrict__ x, int64_t ldx, int K,
                                           const bf16* __restrict__ norm_w, float eps, uint32_t* xf, float* xg,
                                           float* red, int bar) {
  constexpr int CH = 8;  // 16-byte loads in flight per thread per pass
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NG = K >> 6, K8 = K >> 3;
  auto sync = [&]() {
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
  };
  for (int t = 0; t < MT; ++t) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + t * ldx);
    float inv = 1.f;
    if (norm_w) {
      float ss = 0.f;
      for (int c0 = tid; c0 < K8; c0 += NT * CH) {
        uint4 v[CH];
#pragma unroll
        for (int k = 0; k < CH; ++k)
          if (c0 + k * NT < K8) v[k] = xr[c0 + k * NT];
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
          v[k] = xr[c0 + k * NT];
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
  sync();
}

}  // namespace m5
