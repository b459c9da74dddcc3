// Small fused kernels of the token loop (norms, RoPE + KV append, embedding,
// greedy argmax, MoE routing) and their launchers.
#pragma once

#include "common.cuh"

namespace m5 {

// Attention prologue for L tokens of one layer: split the fused q/k/v GEMV
// output, RMS-normalise q and k per head, apply YaRN magnitude + split-half
// RoPE at positions *d_len + t, write q (bf16 [Hq, L, D]) and append k/v to
// the cache (quantized with the MLX rule when bits is 4/8, bf16 when 0).
struct RopeAppendArgs {
  const bf16* qkv;      // [L, (Hq + 2 Hkv) * D]
  int L, Hq, Hkv;       // local heads
  const bf16* q_norm;   // [D]
  const bf16* k_norm;
  float eps;
  const float* inv_freq;  // device [D/2]
  float mscale;
  const int32_t* d_len;   // position of token 0
  bf16* q_out;            // [Hq, L, D]; batch > 1: [batch, Hq, D]
  m5_layer_kv kv;
  int batch;              // > 1: token t is sequence t (L == batch), all at position *d_len;
                          // kv holds [batch, Hkv, capacity, ...]
};
int rope_append_launch(const RopeAppendArgs& a, cudaStream_t stream);

// x[T, H] bf16 = dequant(embedding rows of tokens).
int embed_launch(const int32_t* tokens, int T, const uint32_t* w, const bf16* s, const bf16* b, int H, int V,
                 bf16* out, cudaStream_t stream);

// Argmax over bf16 values (first index among equal values) into *out.
// Uses `scratch` (argmax_scratch_bytes) and leaves it ready for the next call.
size_t argmax_scratch_bytes();
int argmax_launch(const bf16* x, int64_t n, int32_t* out, void* scratch, cudaStream_t stream);
// out[r] = argmax over row r of x[rows, n] (one CTA per row, same tie rule).
int argmax_rows_launch(const bf16* x, int rows, int64_t n, int32_t* out, cudaStream_t stream);

// rms norm rows.
int rms_norm_launch(const bf16* x, const bf16* w, int64_t rows, int dim, float eps, bf16* y, cudaStream_t stream);

// Router: softmax over logits [T, E] (bf16) -> top-k ids/scores.
int moe_topk_launch(const bf16* logits, int T, int E, int k, int norm_topk, int32_t* ids, bf16* scores,
                    cudaStream_t stream);

// Residual add after a tensor-parallel reduce: h = bf16(h + bf16(sum_f32)).
int residual_add_f32_launch(bf16* h, const float* r, int64_t n, cudaStream_t stream);

// Copy one cache layer's rows [0, len) from bf16 into packed form.
int kv_quantize_layer_launch(const m5_layer_kv& src, const m5_layer_kv& dst, int Hkv, int D, int len,
                             cudaStream_t stream);

}  // namespace m5
