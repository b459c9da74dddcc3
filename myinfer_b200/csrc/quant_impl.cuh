// Device-side pieces of the MLX affine quantizer, shared by the standalone
// quantize kernel and the fused KV-append kernel.  Each operation is a single
// IEEE-rounded fp32 step in the order of the MLX rule (see oracle/quant.py for
// the CPU restatement it must equal bit for bit).
#pragma once

#include "common.cuh"

namespace m5 {

struct QParams {
  float scale;  // fp32 scale used for coding; stored rounded to bf16
  float bias;
};

template <int BITS>
__device__ __forceinline__ QParams group_params(float w_max, float w_min) {
  const float nb = float((1 << BITS) - 1);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(w_max, w_min), nb), 1e-7f);
  const bool side = fabsf(w_min) > fabsf(w_max);
  scale = side ? scale : -scale;
  const float edge = side ? w_min : w_max;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  QParams p;
  if (q0 != 0.0f) {
    p.scale = __fdiv_rn(edge, q0);
    p.bias = edge;
  } else {
    p.scale = scale;
    p.bias = 0.0f;
  }
  return p;
}

template <int BITS>
__device__ __forceinline__ uint32_t quant_code(float v, QParams p) {
  const float nb = float((1 << BITS) - 1);
  float q = rintf(__fdiv_rn(__fsub_rn(v, p.bias), p.scale));
  q = fminf(fmaxf(q, 0.0f), nb);
  return (uint32_t)q;
}

// Lane l holds codes of elements 2l and 2l+1 of a 64-element group.  Packs
// them into the group's uint32 words (low bits first); `writer` lanes store
// word `widx` of the group.
template <int BITS>
__device__ __forceinline__ void pack_pair(uint32_t q0, uint32_t q1, int lane, uint32_t& word, bool& writer,
                                          int& widx) {
  if constexpr (BITS == 8) {
    const uint32_t p = q0 | (q1 << 8);
    const uint32_t o = __shfl_down_sync(0xffffffffu, p, 1);
    word = p | (o << 16);
    writer = (lane & 1) == 0;
    widx = lane >> 1;
  } else {
    const uint32_t p = q0 | (q1 << 4);
    const uint32_t o1 = __shfl_down_sync(0xffffffffu, p, 1);
    const uint32_t o2 = __shfl_down_sync(0xffffffffu, p, 2);
    const uint32_t o3 = __shfl_down_sync(0xffffffffu, p, 3);
    word = p | (o1 << 8) | (o2 << 16) | (o3 << 24);
    writer = (lane & 3) == 0;
    widx = lane >> 2;
  }
}

}  // namespace m5
