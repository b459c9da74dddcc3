// Routed-expert MLP of a Qwen3-MoE layer (mlx-lm SwitchGLU via gather_qmm;
// the reference's wrapper contract is m5engine/expert_stream.py:381-403).
#pragma once

#include "common.cuh"

namespace m5 {

struct QW {
  const uint32_t* w;  // stacked local experts [E_local, N, K/8]
  const bf16* s;      // [E_local, N, K/64]
  const bf16* b;
};

struct MoeArgs {
  const bf16* x;        // [T, H] residual stream (normalised inside with norm_w)
  int T, H, I, k;
  int e_first, e_local; // global id of local expert 0, number of local experts
  const int32_t* ids;   // [T, k] global expert ids from the router
  const bf16* scores;   // [T, k]
  QW gate, up, down;
  const bf16* norm_w;
  float eps;
  bf16* act;            // scratch [T * k, I]
  bf16* h;              // [T, H], h += sum_j bf16(y_j * score_j)
  float* partial;       // when non-null: write fp32 sums here instead of h (expert parallel)
  // zeroed scratch of the tensor-core decode path (moe_mma.cu), left zeroed
  float* acc;           // >= max(2 k I, k H) floats
  int* cnt;             // >= acc_rows / 16 counters
  int acc_rows;
  float* ybuf;          // [k, H] per-slot score-weighted rows
  int* ncnt;            // [H / 16] slot counters
};

int moe_launch(const MoeArgs& a, cudaStream_t stream);
// Prefill grouped by expert: sort (token, slot) pairs by local expert, gather
// the normalised rows into expert order, and after the per-expert GEMMs add the
// slots back per token (moe.cu; the runtime drives the GEMMs).
int moe_sort_launch(const int32_t* ids, int pairs, int e_first, int e_local, int32_t* counts, int32_t* offsets,
                    int32_t* pos, cudaStream_t stream);
int moe_gather_launch(const bf16* x, int H, int pairs, int k, const int32_t* pos, bf16* out, cudaStream_t stream);
int moe_combine_launch(const bf16* y, int T, int H, int k, const int32_t* pos, const bf16* scores, bf16* h,
                       float* partial, cudaStream_t stream);
// Router logits + top-k of one decode token in one launch (moe_mma.cu).
struct MoeRouterArgs {
  const bf16* x;          // [H] residual stream, RMS-normalised inside with norm_w
  const bf16* norm_w;
  float eps;
  const uint32_t* w;      // router [E, H/8] w4g64
  const bf16* s;
  const bf16* b;
  int H, E, k, norm_topk;
  bf16* logits;           // [E] scratch
  int32_t* ids;           // [k]
  bf16* scores;           // [k]
  int* counter;           // zeroed, left zeroed
};
int moe_router_topk_launch(const MoeRouterArgs& a, cudaStream_t stream);
// One decode token (T == 1, k == 8) on the tensor cores; moe_launch otherwise.
bool moe_mma_eligible(const MoeArgs& a);
int moe_mma_launch(const MoeArgs& a, cudaStream_t stream);

}  // namespace m5
