/*
 * libm5cuda - B200 (sm_100a) implementation of M5Engine's token loop.
 *
 * Plain C ABI: every entry point returns an int status (M5_OK = 0) and never
 * throws or aborts; m5_last_error() returns the text of the calling thread's
 * last failure.  Device buffers are owned by the caller and passed as raw
 * pointers; the library owns only its scratch arenas.  Every call is ordered
 * on the cudaStream_t passed as `stream` (NULL = legacy default stream) and
 * none synchronises the host unless it says so.
 *
 * bf16 tensors are IEEE bfloat16 bit patterns (uint16).  Packed quantized
 * tensors use the MLX layout: uint32 words holding 32/bits codes, low bits
 * first, `scales`/`biases` bf16 with one value per group of `group_size`
 * consecutive elements of the last axis; element = scale * code + bias.
 *
 * Reference interfaces these entry points replace (paths inside tdcb/myinfer):
 *   m5_affine_quantize      mx.quantize, called for the KV cache through
 *                           m5engine/attention.py:111-112 (to_quantized) and
 *                           mlx-lm QuantizedKVCache.update_and_fetch
 *   m5_affine_dequantize    mx.dequantize (mlx-lm QuantizedEmbedding rows)
 *   m5_quantized_matmul     mx.quantized_matmul(transpose=True), the call at
 *                           m5engine/attention.py:66-69 and every mlx-lm
 *                           QuantizedLinear
 *   m5_quantized_sdpa       blocked_quantized_sdpa, m5engine/attention.py:29-37
 *                           (and the mlx-lm SDPA it falls back to, :42-45)
 *   m5_rms_norm             mx.fast.rms_norm (mlx-lm Qwen3 norms)
 *   m5_forward              model(tokens[1, L], cache=list) -> logits, the
 *                           contract used at m5engine/context.py:53 and inside
 *                           mlx-lm generate_step (m5engine/engine.py:420-423)
 *   m5_moe_route            Qwen3-MoE router (softmax -> top-k -> renormalise)
 *                           feeding SwitchGLU, m5engine/expert_stream.py:381-403
 */
#ifndef M5CUDA_H
#define M5CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define M5_API __attribute__((visibility("default")))
#else
#define M5_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  M5_OK = 0,
  M5_ERR_INVALID = 1,     /* bad argument, shape or alignment */
  M5_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  M5_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
  M5_ERR_TIMEOUT = 4,     /* a bounded device wait expired */
  M5_ERR_COMM = 5,        /* NCCL / peer communication failure */
  M5_ERR_STATE = 6        /* handle used in the wrong state */
};

enum { M5_DTYPE_BF16 = 0, M5_DTYPE_F32 = 1 };
enum { M5_MASK_NONE = 0, M5_MASK_CAUSAL = 1, M5_MASK_BOOL = 2, M5_MASK_ADDITIVE = 3 };
enum { M5_LOGITS_NONE = 0, M5_LOGITS_LAST = 1, M5_LOGITS_ALL = 2 };

/* Library version (major * 10000 + minor * 100 + patch). */
M5_API int m5_version(void);
/* Copies the calling thread's last error text into buf (NUL-terminated);
 * returns the full length of the message. */
M5_API size_t m5_last_error(char* buf, size_t n);

/* Sticky device-side error word: nonzero when a bounded wait inside a kernel
 * gave up (the kernel then returned early and its output is invalid).
 * Synchronises the device.  reset != 0 clears it. */
M5_API int m5_device_status(int* code, int reset);

/* ------------------------------------------------------------ quantization */
/* Affine group quantization of x [rows, cols] (row stride ld_x elements,
 * x_dtype M5_DTYPE_BF16 or M5_DTYPE_F32) into wq [rows, cols*bits/32] uint32,
 * scales/biases [rows, cols/group_size] bf16.  Bit-exact MLX rule: fp32
 * scale/bias with the endpoint-exact edge adjustment, round-half-to-even,
 * IEEE division.  bits in {4, 8}; group_size 64 (32 and 128 also accepted). */
M5_API int m5_affine_quantize(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ld_x,
                       int group_size, int bits, uint32_t* wq, void* scales, void* biases,
                       void* stream);

/* out[rows, cols] bf16 = scale * code + bias (computed as one fp32 fma). */
M5_API int m5_affine_dequantize(const uint32_t* wq, const void* scales, const void* biases, int64_t rows,
                         int64_t cols, int group_size, int bits, void* out, void* stream);

/* y[M, N] bf16 = x[M, K] bf16 @ dequant(W[N, K])^T with fp32 accumulation.
 * bits 4, group_size 64.  M <= 16 runs the streaming GEMV; larger M the GEMM. */
M5_API int m5_quantized_matmul(const void* x, int64_t M, int64_t K, const uint32_t* wq,
                        const void* scales, const void* biases, int64_t N, int group_size,
                        int bits, void* y, void* stream);

/* Same result as m5_quantized_matmul, for callers that cannot allocate device
 * memory (a serving host whose own allocator owns the whole device pool, an
 * embedder that forbids allocation after start-up).  It never calls
 * cudaMalloc/cudaFree: its scratch is an 8 MiB array built into the library
 * (held by every GPU that loads it) whose address is looked up on the first
 * call on each device, so that first call should come before any stream
 * capture.  Limit: N <= 262144 weight rows (M and K as for
 * m5_quantized_matmul).  All calls share the array, which keeps the last
 * call's contents; calls that overlap on the GPU race and must not be issued.
 * This entry point has no counterpart in the reference. */
M5_API int m5_quantized_matmul_noalloc(const void* x, int64_t M, int64_t K, const uint32_t* wq,
                                       const void* scales, const void* biases, int64_t N,
                                       int group_size, int bits, void* y, void* stream);

/* y[rows, dim] = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))), x/w/y bf16. */
M5_API int m5_rms_norm(const void* x, const void* w, int64_t rows, int64_t dim, float eps, void* y,
                void* stream);

/* -------------------------------------------------------------- attention */
/* One K or V operand of the attention: rows of head_dim elements, token-major
 * inside a head.  bits 8/4: data = packed uint32 rows, scales/biases bf16;
 * bits 0: data = bf16 rows, scales = biases = NULL.  Strides count rows. */
typedef struct m5_kv_view {
  const void* data;
  const void* scales;
  const void* biases;
  int64_t batch_stride; /* rows between batch entries */
  int64_t head_stride;  /* rows between kv heads */
} m5_kv_view;

/* out[B, Hq, L, D] bf16 = softmax(q * scale @ K^T + mask) @ V over S keys.
 * q bf16 [B, Hq, L, D] contiguous; Hq % Hkv == 0 (GQA); D in {64, 128}.
 * mask_kind: NONE; CAUSAL (query i sits at position S - L + i); BOOL (uint8
 * [.., L, S], nonzero = keep); ADDITIVE (fp32 [.., L, S], added to scores).
 * mask_strides = {batch, head, row} in elements (0 broadcasts), last axis
 * contiguous.  Scores are rounded to bf16 before the fp32 online softmax, as
 * m5engine/attention.py:66-69 does. */
M5_API int m5_quantized_sdpa(const void* q, int B, int Hq, int L, int D, m5_kv_view keys,
                      m5_kv_view values, int Hkv, int S, float scale, int mask_kind,
                      const void* mask, const int64_t* mask_strides, int group_size, int bits,
                      void* out, void* stream);

/* ------------------------------------------------------------- the model */
typedef struct m5_model_cfg {
  int hidden_size;
  int num_layers;
  int num_heads;        /* q heads of the whole model */
  int num_kv_heads;     /* kv heads of the whole model */
  int head_dim;         /* 128 */
  int intermediate_size;
  int vocab_size;
  int num_experts;      /* 0 = dense */
  int experts_per_tok;
  int moe_intermediate_size;
  int norm_topk_prob;
  int tie_word_embeddings;
  float rms_norm_eps;
  int group_size;       /* weight quantization: 64 */
  int bits;             /* 4 */
  int tp_size;          /* ranks the dense layers are split over (1 = none) */
  int tp_rank;
  int ep_size;          /* ranks the experts are split over (1 = none) */
  int ep_rank;
} m5_model_cfg;

/* One layer's KV cache as the caller allocated it (MLX layout, batch 1):
 * bits 8/4: k/v packed uint32 [Hkv_local, capacity, D*bits/32],
 * scales/biases bf16 [Hkv_local, capacity, D/group_size];
 * bits 0: k/v bf16 [Hkv_local, capacity, D], scales/biases NULL. */
typedef struct m5_layer_kv {
  void* k;
  void* k_scales;
  void* k_biases;
  void* v;
  void* v_scales;
  void* v_biases;
  int64_t capacity;
  int bits;
  int group_size;
} m5_layer_kv;

M5_API int m5_model_create(const m5_model_cfg* cfg, void** model);
M5_API int m5_model_destroy(void* model);
/* Bind one weight tensor by its MLX safetensors name, e.g.
 * "model.layers.3.self_attn.q_proj.weight" / ".scales" / ".biases",
 * "model.layers.3.input_layernorm.weight", "model.embed_tokens.weight".
 * The pointer must stay valid while the model is used. */
M5_API int m5_model_bind(void* model, const char* name, const void* ptr);
/* Fails with M5_ERR_STATE naming the first tensor that is still unbound. */
M5_API int m5_model_check(void* model);
/* RoPE table: inv_freq[head_dim/2] (host fp32) and the YaRN magnitude
 * factor applied to q and k before rotation (1.0 = plain RoPE). */
M5_API int m5_model_set_rope(void* model, const float* inv_freq, float mscale);
/* Size the activation scratch for chunks of up to max_tokens tokens. */
M5_API int m5_model_reserve(void* model, int max_tokens);

/* Run L tokens (device int32 [L]) through the model at the cache position
 * *d_len (device int32), append their K/V to every layer's cache, and add L
 * to *d_len.  logits_mode: NONE, LAST (logits bf16 [V]) or ALL ([L, V]).
 * d_argmax (device int32, may be NULL) receives argmax of the last row (first
 * index among equal bf16 logits).  All launch shapes depend only on L and the
 * cache capacities, so a call can be captured once into a CUDA graph and
 * replayed for successive decode steps. */
M5_API int m5_forward(void* model, const m5_layer_kv* kv, int32_t* d_len, const int32_t* d_tokens, int L,
               void* logits, int logits_mode, int32_t* d_argmax, void* stream);

/* Batched decode: one new token for each of B independent sequences, all at
 * position *d_len (so *d_len += 1 after the call), over caches whose layers
 * hold the B sequences back to back: k/v [B, Hkv_local, capacity, ...], batch
 * stride Hkv_local * capacity rows.  logits [B, V] bf16 (LAST and ALL both
 * give the B rows), d_argmax [B] (needs logits).  The batched model call of
 * mlx-lm (model(tokens[B, 1], cache) -> logits[B, 1, V], the contract used at
 * m5engine/context.py:53) at the batch sizes of the benchmark configs
 * (16/32/64); projections take the tensor-core GEMM from 16 rows on. */
M5_API int m5_forward_batch(void* model, const m5_layer_kv* kv, int32_t* d_len, const int32_t* d_tokens, int B,
                            void* logits, int logits_mode, int32_t* d_argmax, void* stream);

/* Convert rows [0, len) of a bf16 cache layer into a packed one (the
 * reference's KVCache.to_quantized at m5engine/attention.py:111-112). */
M5_API int m5_kv_quantize_layer(const m5_layer_kv* src, const m5_layer_kv* dst, int num_kv_heads, int head_dim,
                         int len, void* stream);

/* Greedy sampler: out[0] = argmax(x[n]) over bf16 logits, first index wins. */
M5_API int m5_argmax_bf16(const void* x, int64_t n, int32_t* out, void* stream);

/* Sampling parameters: the sampler and logits processors the reference builds
 * per request (m5engine/engine.py:384-392: mlx-lm 0.31.3 make_sampler(temp,
 * top_p, min_p, top_k) and make_logits_processors(repetition_penalty,
 * presence_penalty, frequency_penalty)).  A filter is off at its neutral
 * value: top_p outside (0, 1), min_p <= 0, top_k <= 0 or >= vocab,
 * repetition_penalty 1 (or 0), presence/frequency 0.  Row r draws the
 * uniform number with counter offset (+ state[0]) + r of the SplitMix64
 * stream of seed. */
typedef struct m5_sample_params {
  float temperature;  /* <= 0: greedy (first index of the max after penalties) */
  float top_p;
  float min_p;
  int top_k;
  float repetition_penalty;
  float presence_penalty;
  float frequency_penalty;
  int flags;          /* M5_SAMPLE_APPEND_HISTORY */
  uint64_t seed;
  uint64_t offset;
} m5_sample_params;

#define M5_SAMPLE_APPEND_HISTORY 1

/* One token per row of bf16 logits [rows, vocab] (row stride ld).  history:
 * int32 [rows, hist_ld], the first hist_len entries per row are the penalty
 * window, oldest first (negative entries are empty); with
 * M5_SAMPLE_APPEND_HISTORY each window rolls left by one and ends with the
 * drawn token.  Penalised logits are written back in place (mlx-lm returns
 * the processed logits).  state: NULL, or two zero-initialised uint64 on the
 * device holding the draw counter, which the call advances by rows (so a
 * captured graph draws new numbers on every replay).  out: int32 [rows].
 * vocab <= 524288, hist_len <= 1024.  Logits must be free of NaN. */
M5_API int m5_sample_bf16(void* logits, int rows, int64_t vocab, int64_t ld, int32_t* history, int hist_len,
                          int64_t hist_ld, const m5_sample_params* p, uint64_t* state, int32_t* out, void* stream);

/* Qwen3-MoE router for T tokens: logits = x @ gate^T (w4g64), probabilities =
 * softmax (fp32 math, bf16 result), top-k by probability (ties -> lower
 * expert id), renormalised when norm_topk_prob.  ids int32 [T, k], scores
 * bf16 [T, k], logits_out bf16 [T, E] (may be NULL). */
M5_API int m5_moe_route(const void* x, int T, int H, const uint32_t* gate_w, const void* gate_s,
                 const void* gate_b, int E, int k, int norm_topk_prob, int32_t* ids, void* scores,
                 void* logits_out, void* stream);

/* ---------------------------------------------------------------- multi-GPU
 * One process per GPU.  A model created with tp_size > 1 (dense: q/k/v heads,
 * gate/up rows, o/down columns and lm_head rows split over ranks) or
 * ep_size > 1 (MoE: experts split, attention replicated) needs a
 * communicator before m5_model_check / m5_forward: rank 0 makes an id with
 * m5_comm_unique_id, the caller hands the bytes to every rank (the reference
 * has no multi-GPU path; torch.distributed is the usual carrier), each rank
 * calls m5_comm_init.  m5_forward then all-reduces the o_proj / down (or MoE)
 * partial sums in fp32 and all-gathers the vocabulary shards of the logits, so
 * every rank returns the full logits and the same argmax. */
#define M5_COMM_ID_BYTES 128
M5_API int m5_comm_unique_id(void* out, size_t len);
/* Set-up is non-blocking and bounded (M5_COMM_INIT_TIMEOUT_S, default 300 s):
 * if a rank never joins, the call aborts the communicator and returns
 * M5_ERR_TIMEOUT instead of hanging. */
M5_API int m5_comm_init(const void* id, size_t len, int nranks, int rank, void** comm);
M5_API int m5_comm_destroy(void* comm);
M5_API int m5_model_set_comm(void* model, void* comm);
/* In-place fp32 sum over the communicator's ranks (stream-ordered). */
M5_API int m5_allreduce_f32(void* comm, float* buf, int64_t n, void* stream);
/* Failure detection (the reference's counterpart is its error state:
 * EngineError and the load/generate error handling, m5engine/engine.py:47-56,
 * 192-205).  m5_comm_check returns M5_ERR_COMM when NCCL reports an
 * asynchronous error on the communicator (M5_ERR_STATE once aborted);
 * m5_comm_abort aborts it (every later collective fails fast) so a rank that
 * learned of a failed peer can leave without waiting on it;
 * m5_comm_set_wait_ms bounds the peer all-reduce's wait for the other ranks
 * (default 2000 ms; on expiry the call records a device error read by
 * m5_device_status and leaves the residual stream unchanged). */
M5_API int m5_comm_check(void* comm);
M5_API int m5_comm_abort(void* comm);
M5_API int m5_comm_set_wait_ms(void* comm, int ms);
/* Runs the peer all-reduce kernel on the current GPU against a stand-in
 * second rank that never arrives, with a `wait_ms` bound: returns the device
 * error word it left (*device_code), the call's wall time and whether the
 * residual stream was left unchanged.  Diagnostic; needs no communicator. */
M5_API int m5_comm_peer_wait_selftest(int wait_ms, int* device_code, double* elapsed_ms, int* h_unchanged);

#ifdef __cplusplus
}
#endif

#endif /* M5CUDA_H */
