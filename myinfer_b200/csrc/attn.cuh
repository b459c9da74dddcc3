// Attention over the (quantized) KV cache: split-KV flash decoding plus the
// log-sum-exp combine (kernels K4 / K5 of the token loop).
#pragma once

#include "common.cuh"

namespace m5 {

struct AttnArgs {
  const bf16* q;        // [B, Hq, L, D]
  int B, Hq, L, D;
  m5_kv_view k, v;
  int bits;             // 0 (bf16 K/V), 4 or 8
  int Hkv;
  int S_host;           // number of keys when d_S is null
  const int32_t* d_S;   // device key count (decode steps inside a graph) ...
  int S_add;            // ... plus this constant
  float scale;
  int mask_kind;
  const void* mask;
  int64_t ms_b, ms_h, ms_l;
  int QB;               // queries per CTA
  int nsplit;
  int chunk;            // keys per split when d_S is null (0 = derive at run time)
  float* part_o;        // scratch [B*Hq*L, nsplit, D]
  float* part_ml;       // scratch [B*Hq*L, nsplit, 2]
  bf16* out;            // [B, Hq, L, D], or [B, L, Hq, D] when out_tokens_major
  int out_tokens_major;
};

// Scratch bytes attention with these launch parameters needs.
size_t attn_scratch_bytes(int B, int Hq, int L, int D, int nsplit);
// Pick queries per CTA and the number of key splits for a call.
void attn_plan(int B, int Hq, int Hkv, int L, int S_max, int& QB, int& nsplit);
// Launch (and combine when nsplit > 1).  part_* must hold attn_scratch_bytes.
int attn_launch(const AttnArgs& a, cudaStream_t stream);

// Tensor-core split-KV decode kernel (attn_mma.cu): 8/4-bit K/V, D = 128,
// rows (GQA group x queries per CTA) <= 16, no / causal mask, aligned views.
bool attn_mma_eligible(const AttnArgs& a);
int attn_mma_launch(const AttnArgs& a, cudaStream_t stream);
// CTAs per SM the tensor-core decode kernel keeps resident for `rows` MMA rows
int attn_mma_ctas_per_sm(int rows);
int attn_mma_error(int reset);

// Prefill tensor-core kernel (attn_pf.cu): 8/4-bit KV, D = 128, L * rep > 16.
bool attn_pf_eligible(const AttnArgs& a);
void attn_pf_plan(const AttnArgs& a, int S_max, int max_split, int& QB, int& nsplit);
int attn_pf_launch(const AttnArgs& a, cudaStream_t stream);
int attn_pf_error(int reset);

// Prefill kernel on tcgen05 / TMEM (attn_tc.cu): the shapes of attn_pf, one
// CTA of 128 rows per SM; used where attn_pf is eligible unless M5_ATTN_TC=0.
bool attn_tc_eligible(const AttnArgs& a);
void attn_tc_plan(const AttnArgs& a, int S_max, int max_split, int& QB, int& nsplit);
int attn_tc_launch(const AttnArgs& a, cudaStream_t stream);
int attn_tc_error(int reset);

}  // namespace m5
