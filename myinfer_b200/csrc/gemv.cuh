// Streaming w4g64 dequant-GEMV for decode (M <= 8 tokens per launch).
#pragma once

#include "common.cuh"
#include "ops.cuh"

namespace m5 {

enum GemvEpi {
  EPI_STORE = 0,     // y = bf16(acc)
  EPI_RESIDUAL = 1,  // y = bf16(y + bf16(acc))      (residual add in place)
  EPI_SWIGLU = 2,    // y = bf16(bf16(g * bf16(sigmoid(g))) * u), g/u = bf16(acc) of gate/up rows
  EPI_F32 = 3        // yf = acc (fp32; partial sums before a tensor-parallel reduce)
};

// A run of weight rows that share one output buffer.  Several segments let one
// launch cover q/k/v (or several experts) without repacking MLX tensors.
struct GemvSeg {
  const uint32_t* w;  // [rows, K/8]
  const bf16* s;      // [rows, K/64]
  const bf16* b;
  int rows;
  bf16* y;            // output column base: y[t * ldy + r]
  float* yf;          // fp32 output base (EPI_F32)
};

struct GemvArgs {
  const bf16* x;      // [MT, ldx]
  int64_t ldx;
  int K;
  int nseg;
  GemvSeg seg[4];     // SWIGLU: seg[0] gate, seg[1] up (same rows), output seg[0].y
  int64_t ldy;
  int total_rows;     // rows to produce (SWIGLU: gate rows)
  int rows_per_warp;
  const bf16* norm_w; // fused RMSNorm of x when non-null
  float eps;
  // Zero-initialised fp32 [8][mma_rows] + int [mma_rows/16] scratch for the
  // tensor-core GEMV's split tiles (left zeroed after every launch); when null
  // the launcher uses its own per-device scratch.
  float* mma_acc;
  int* mma_cnt;
  int mma_rows;
  // Per-CTA slots for the tensor-map GEMV's tiles shared between CTAs
  // (gemv_part_floats() floats; no zeroing needed); null: per-device scratch.
  float* mma_part;
  size_t mma_part_floats;
  // Row length of the weights, scales and biases when the call reduces over
  // only K columns of wider rows (a K slice; 0 = K).  Read by the prefill GEMM.
  int64_t ldk;
  // QK-norm + RoPE + KV append fused into the q|k|v projection (EPI_STORE on
  // the tensor-map GEMV, gemv_tmap_eligible): when rope_cnt is set, the warp
  // that writes the last of the 8 16-row tiles of a 128-row head runs that
  // head's rope_append_row for every token.  rope.qkv must be the output of
  // the segments laid end to end (row = head * 128 + d) and rope.L = MT;
  // rope_cnt is one zeroed int per head, left zeroed.
  RopeAppendArgs rope;
  unsigned int* rope_cnt;
};

// Launch y = epi(x @ W^T) for up to 8 tokens.  Chooses rows per warp so the
// grid fits the device in one wave.  Returns an M5 status.
int gemv_launch(const GemvArgs& a, int MT, int epi, cudaStream_t stream);

// Largest number of tokens one launch can stage for this K (shared memory).
int gemv_max_tokens(int K);

// TMA tensor-map + tensor-core variant (gemv_tmap.cu): K % 512 == 0.  `part`
// holds part_floats floats of per-CTA split-tile slots, `cnt` one zeroed
// counter per 16-row tile for cnt_rows rows (both left as found).
bool gemv_tmap_eligible(const GemvArgs& a, int MT, int epi);
int gemv_tmap_launch(const GemvArgs& a, int MT, int epi, float* part, size_t part_floats, int* cnt, int cnt_rows,
                     cudaStream_t stream);
// Slot floats a tensor-map GEMV launch of this device may need.
size_t gemv_part_floats();
int gemv_tmap_error(int reset);

// Tensor-core variant (gemv_mma.cu): K % 64 == 0, segments of 16-row multiples.
bool gemv_mma_eligible(const GemvArgs& a, int MT, int epi);
int gemv_mma_launch(const GemvArgs& a, int MT, int epi, float* acc, int* cnt, int acc_rows, cudaStream_t stream);
// Bytes of zeroed scratch gemv_mma needs for matrices of up to `rows` rows.
size_t gemv_mma_scratch_bytes(int rows);

// TMA-fed variant (gemv_tma.cu): K % 512 == 0 and MT <= 2.
bool gemv_tma_eligible(int K, int MT, int epi);
int gemv_tma_launch(const GemvArgs& a, int MT, int epi, cudaStream_t stream);
// Sticky device error word of the bounded waits in gemv_tma.cu (-1 if unreadable).
int gemv_tma_error(int reset);

// Prefill tensor-core dequant-GEMM (gemm_tc.cu, tcgen05 + TMEM): any M >= 1,
// K % 64 == 0, no fused norm, segments of 128-row multiples (SwiGLU: 64).
// `xs` is caller scratch of gemm_tc_xs_bytes(M, K) bytes (per-token group sums).
bool gemm_tc_eligible(const GemvArgs& a, int M, int epi);
size_t gemm_tc_xs_bytes(int M, int K);
int gemm_tc_launch(const GemvArgs& a, int M, int epi, bf16* xs, size_t xs_bytes, cudaStream_t stream);
// Adds the fp32 partial products of S K slices (part [S][M][N], in slice order)
// and applies EPI_STORE (y = bf16(sum)), EPI_RESIDUAL (y += bf16(sum)) or
// EPI_F32 (yf = sum).
int gemm_splitk_reduce_launch(const float* part, int S, int M, int N, int epi, bf16* y, float* yf, int64_t ldy,
                              cudaStream_t stream);
int gemm_tc_error(int reset);

}  // namespace m5
