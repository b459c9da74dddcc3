// QK-norm + RoPE/YaRN + KV quantize-on-append of one (token, head) row of the
// fused q|k|v projection, by one warp: shared by the standalone kernel
// (ops.cu) and the q|k|v GEMV's epilogue (gemv_tmap.cu), which runs it as
// soon as the last 16-row tile of a head is written.
#pragma once

#include "ops.cuh"
#include "quant_impl.cuh"

namespace m5 {

// One warp holds a 128-element row, 4 consecutive elements per lane.  Quantize
// it with the MLX rule (two groups of 64 = lanes 0-15 and 16-31) and store the
// packed words and the bf16 scale/bias of both groups.
template <int BITS>
__device__ __forceinline__ void quant_row128(const float (&x)[4], int lane, uint32_t* words, bf16* s, bf16* b) {
  float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
  float mn = fminf(fminf(x[0], x[1]), fminf(x[2], x[3]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  const QParams p = group_params<BITS>(mx, mn);
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = quant_code<BITS>(x[i], p);
  if constexpr (BITS == 8) {
    words[lane] = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
  } else {
    const uint32_t p16 = q[0] | (q[1] << 4) | (q[2] << 8) | (q[3] << 12);
    const uint32_t o = __shfl_down_sync(0xffffffffu, p16, 1);
    if ((lane & 1) == 0) words[lane >> 1] = p16 | (o << 16);
  }
  if ((lane & 15) == 0) {
    s[lane >> 4] = f2bf(p.scale);
    b[lane >> 4] = f2bf(p.bias);
  }
}

template <int BITS>
__device__ __forceinline__ void store_kv_row(const float (&x)[4], int lane, void* data, bf16* sc, bf16* bi,
                                             size_t row) {
  if constexpr (BITS == 0) {
    uint2 v;
    v.x = uint32_t(__bfloat16_as_ushort(f2bf(x[0]))) | (uint32_t(__bfloat16_as_ushort(f2bf(x[1]))) << 16);
    v.y = uint32_t(__bfloat16_as_ushort(f2bf(x[2]))) | (uint32_t(__bfloat16_as_ushort(f2bf(x[3]))) << 16);
    reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(data) + row * 128)[lane] = v;
  } else {
    quant_row128<BITS>(x, lane, reinterpret_cast<uint32_t*>(data) + row * (128 * BITS / 32), sc + row * 2,
                       bi + row * 2);
  }
}

// The row of token t, head h (q heads, then k, then v) of a.qkv.  CG: read the
// row through L2 (written by other CTAs of the same kernel).
template <int BITS, bool CG>
__device__ __forceinline__ void rope_append_row(const RopeAppendArgs& a, int t, int h, int lane) {
  constexpr int D = 128;
  const int H3 = a.Hq + 2 * a.Hkv;
  const bool batched = a.batch > 1;
  const int pos = *a.d_len + (batched ? 0 : t);
  const uint2* src = reinterpret_cast<const uint2*>(a.qkv + (size_t(t) * H3 + h) * D + 4 * lane);
  const uint2 raw = CG ? __ldcg(src) : *src;
  float x[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  const bool is_q = h < a.Hq;
  const bool is_k = !is_q && h < a.Hq + a.Hkv;
  if (is_q || is_k) {
    const bf16* nw = is_q ? a.q_norm : a.k_norm;
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float inv = __frsqrt_rn(__fadd_rn(ss / float(D), a.eps));
    const uint2 wr = *reinterpret_cast<const uint2*>(nw + 4 * lane);
    const float w[4] = {bf16_lo(wr.x), bf16_hi(wr.x), bf16_lo(wr.y), bf16_hi(wr.y)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[i] = rbf(__fmul_rn(w[i], rbf(__fmul_rn(x[i], inv))));
      if (a.mscale != 1.f) x[i] = rbf(__fmul_rn(x[i], a.mscale));
    }
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = 4 * (lane & 15) + i;
      const float theta = __fmul_rn(float(pos), a.inv_freq[f]);
      float sn, cs;
      sincosf(theta, &sn, &cs);
      float o;
      if (lane < 16) o = __fsub_rn(__fmul_rn(x[i], cs), __fmul_rn(pr[i], sn));  // x1 c - x2 s
      else o = __fadd_rn(__fmul_rn(pr[i], sn), __fmul_rn(x[i], cs));             // x1 s + x2 c
      x[i] = rbf(o);
    }
  }
  if (is_q) {
    uint2 v;
    v.x = uint32_t(__bfloat16_as_ushort(f2bf(x[0]))) | (uint32_t(__bfloat16_as_ushort(f2bf(x[1]))) << 16);
    v.y = uint32_t(__bfloat16_as_ushort(f2bf(x[2]))) | (uint32_t(__bfloat16_as_ushort(f2bf(x[3]))) << 16);
    const size_t qrow = batched ? size_t(t) * a.Hq + h : size_t(h) * a.L + t;
    reinterpret_cast<uint2*>(a.q_out + qrow * D)[lane] = v;
    return;
  }
  if (pos >= a.kv.capacity) return;  // the host checks capacity; never write past it
  const int kh = is_k ? h - a.Hq : h - a.Hq - a.Hkv;
  const size_t row = (size_t(batched ? t : 0) * a.Hkv + kh) * a.kv.capacity + pos;
  if (is_k) store_kv_row<BITS>(x, lane, a.kv.k, (bf16*)a.kv.k_scales, (bf16*)a.kv.k_biases, row);
  else store_kv_row<BITS>(x, lane, a.kv.v, (bf16*)a.kv.v_scales, (bf16*)a.kv.v_biases, row);
}

// rope_append_row for the cache's bits (0 = bf16, 4, 8).
template <bool CG>
__device__ __forceinline__ void rope_append_row_any(const RopeAppendArgs& a, int t, int h, int lane) {
  if (a.kv.bits == 8) rope_append_row<8, CG>(a, t, h, lane);
  else if (a.kv.bits == 4) rope_append_row<4, CG>(a, t, h, lane);
  else rope_append_row<0, CG>(a, t, h, lane);
}

}  // namespace m5
