// Device building blocks of the streaming dequant-GEMV, shared by the dense
// GEMV (gemv.cu) and the grouped MoE expert kernels (moe.cu).
#pragma once

#include "common.cuh"

namespace m5 {

// Element e of a token row lives at this float offset of the staged row.
__device__ __forceinline__ int xs_index(int e) {
  const int blk = e >> 5, piece = (e >> 2) & 7;
  return (blk << 5) | ((piece ^ (blk & 7)) << 2) | (e & 3);
}

// sum_k x[k] * (128 + q[k]) over the 32 codes of one uint4, x from the
// swizzled staged row (block `blk`).
__device__ __forceinline__ float dot32(const uint4 wv, const float* __restrict__ xrow, int blk) {
  const float4* xb = reinterpret_cast<const float4*>(xrow + (blk << 5));
  const int sw = blk & 7;
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = words[k] & 0x0f0f0f0fu;          // codes of elements 8k + 0,2,4,6
    const uint32_t hi = (words[k] >> 4) & 0x0f0f0f0fu;   // codes of elements 8k + 1,3,5,7
    const float4 xa = xb[(2 * k) ^ sw];                  // x[8k .. 8k+3]
    const float4 xc = xb[(2 * k + 1) ^ sw];              // x[8k+4 .. 8k+7]
    acc0 = ffma2(make_float2(xa.x, xa.y), make_float2(nib128<0>(lo), nib128<0>(hi)), acc0);
    acc1 = ffma2(make_float2(xa.z, xa.w), make_float2(nib128<1>(lo), nib128<1>(hi)), acc1);
    acc0 = ffma2(make_float2(xc.x, xc.y), make_float2(nib128<2>(lo), nib128<2>(hi)), acc0);
    acc1 = ffma2(make_float2(xc.z, xc.w), make_float2(nib128<3>(lo), nib128<3>(hi)), acc1);
  }
  return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

// Stage MT activation rows (bf16, optionally RMS-normalised with norm_w) into
// shared memory as swizzled fp32, plus the sum of every 32-element block.
template <int MT>
__device__ __forceinline__ void stage_rows(const bf16* __restrict__ x, int64_t ldx, int K,
                                           const bf16* __restrict__ norm_w, float eps, float* xs,
                                           float* xsum, float* red) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int t = 0; t < MT; ++t) {
    const bf16* xr = x + t * ldx;
    float inv = 1.f;
    if (norm_w) {
      float ss = 0.f;
      for (int i = tid; i < K; i += nt) {
        const float v = bf2f(xr[i]);
        ss += v * v;
      }
      ss = warp_sum(ss);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
      __syncthreads();
      if (tid < 32) {
        float v = tid < (nt >> 5) ? red[tid] : 0.f;
        v = warp_sum(v);
        if (tid == 0) red[32] = v;
      }
      __syncthreads();
      inv = __frsqrt_rn(__fadd_rn(red[32] / float(K), eps));
      __syncthreads();
    }
    float* xrow = xs + t * K;
    for (int i = tid; i < K; i += nt) {
      float v = bf2f(xr[i]);
      if (norm_w) v = rbf(__fmul_rn(bf2f(norm_w[i]), rbf(__fmul_rn(v, inv))));
      xrow[xs_index(i)] = v;
    }
  }
  __syncthreads();
  const int K32 = K >> 5;
  for (int j = tid; j < MT * K32; j += nt) {
    const float4* p = reinterpret_cast<const float4*>(xs + (j / K32) * K + (j % K32) * 32);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 v = p[q];
      s += (v.x + v.y) + (v.z + v.w);
    }
    xsum[j] = s;
  }
  __syncthreads();
}

// Accumulate one weight row (all chunks of this lane) into acc[MT].
template <int MT, int U>
__device__ __forceinline__ void row_dot(const uint32_t* __restrict__ w, const bf16* __restrict__ s,
                                        const bf16* __restrict__ b, int K, const float* xs,
                                        const float* xsum, float (&acc)[MT]) {
  const int lane = threadIdx.x & 31;
  const int K32 = K >> 5;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  for (int c0 = 0; c0 * 32 < K32; c0 += U) {
    uint4 wv[U];
    float sv[U], bv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = lane + 32 * (c0 + u);
      if (i < K32) {
        wv[u] = ldg_stream(wr + i);
        sv[u] = bf2f(s[i >> 1]);
        bv[u] = bf2f(b[i >> 1]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = lane + 32 * (c0 + u);
      if (i < K32) {
        const float off = fmaf(-128.f, sv[u], bv[u]);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float A = dot32(wv[u], xs + t * K, i);
          acc[t] = fmaf(sv[u], A, fmaf(off, xsum[t * K32 + i], acc[t]));
        }
      }
    }
  }
}

}  // namespace m5
