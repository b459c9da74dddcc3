// The model handle and the forward pass of the token loop (C ABI).
//
// m5_forward is the device-side body of one mlx-lm model call
// (model(tokens[1, L], cache) at m5engine/context.py:53, driven by
// generate_step behind m5engine/engine.py:420-423): embedding, then per layer
//   fused-RMSNorm q|k|v GEMV -> QK-norm + RoPE/YaRN + KV quantize-append ->
//   split-KV attention -> o_proj GEMV (+ residual) -> fused-RMSNorm gate|up
//   GEMV with SwiGLU -> down GEMV (+ residual)      [dense layers]
//   fused-RMSNorm router GEMV -> top-k -> grouped expert GEMVs  [MoE layers]
// then the final norm fused into the lm_head GEMV and a greedy argmax.
// Positions come from a device counter so one captured CUDA graph replays
// every decode step; every launch shape depends only on L and capacities.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attn.cuh"
#include "comm.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "ops.cuh"

namespace m5 {

struct Linear {
  const uint32_t* w = nullptr;
  const bf16* s = nullptr;
  const bf16* b = nullptr;
  bool ok() const { return w && s && b; }
};

struct Layer {
  const bf16* in_norm = nullptr;
  const bf16* post_norm = nullptr;
  const bf16* q_norm = nullptr;
  const bf16* k_norm = nullptr;
  Linear q, k, v, o;
  Linear gate, up, down;        // dense MLP
  Linear router;                // MoE: mlp.gate
  Linear e_gate, e_up, e_down;  // MoE: stacked local experts
};

struct Model {
  m5_model_cfg cfg{};
  int Hq = 0, Hkv = 0, I = 0, E_local = 0, e_first = 0;  // this rank's shard
  Linear embed, lm_head;
  const bf16* final_norm = nullptr;
  std::vector<Layer> layers;
  float* d_inv_freq = nullptr;
  float mscale = 1.f;
  bool rope_set = false;
  // scratch arena
  int max_tokens = 0;
  char* arena = nullptr;
  size_t arena_bytes = 0;
  bf16 *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits_last = nullptr;
  bf16 *rlogits = nullptr, *rscores = nullptr;
  int32_t* rids = nullptr;
  float* attn_part = nullptr;
  size_t attn_part_bytes = 0;
  void* argmax_scratch = nullptr;
  float* mma_acc = nullptr;  // zeroed split-tile scratch of the tensor-core GEMV
  int* mma_cnt = nullptr;
  int mma_rows = 0;
  unsigned int* rope_cnt = nullptr;  // zeroed per-head counters of the q|k|v GEMV's fused rope epilogue
  float* gemv_part = nullptr;        // split-tile slots of the tensor-map GEMV (gemv_part_floats())
  float* moe_ybuf = nullptr;  // zeroed [k, H] and [H/16] scratch of the tensor-core expert path
  int* moe_ncnt = nullptr;
  // MoE prefill grouped by expert (T >= kMoeGroupedMinTokens): expert-ordered rows and
  // the per-expert GEMMs' side streams
  bf16* moe_x = nullptr;       // [T k, H]
  bf16* moe_act = nullptr;     // [T k, I]
  bf16* moe_y = nullptr;       // [T k, H]
  bf16* moe_xs = nullptr;      // [T k, 64 (C_H + C_I)] group sums of the GEMM inputs
  int32_t* moe_pos = nullptr;  // [T k]
  int32_t* moe_cnt = nullptr;  // [E_local] counts, [E_local] offsets
  int32_t* h_moe_cnt = nullptr;  // pinned copy of the counts
  static constexpr int kMoeStreams = 4;
  cudaStream_t moe_st[kMoeStreams] = {};
  cudaEvent_t moe_fork = nullptr, moe_join[kMoeStreams] = {};
  bf16* xn = nullptr;        // RMSNorm(h) materialised for the prefill GEMM [T, H]
  bf16* gxs = nullptr;       // per-token group sums of the prefill GEMM input
  size_t gxs_bytes = 0;
  // multi-GPU: communicator, fp32 partial sums [T, H], vocabulary shard logits
  void* comm = nullptr;
  int Vl = 0, v_rows = 0;    // this rank's vocabulary rows; head rows per gather chunk
  float* hf = nullptr;
  bf16* vpart = nullptr;     // [v_rows, Vl]
  bf16* vgather = nullptr;   // [tp, v_rows, Vl]
  // GEMMs of few rows split over K (batched decode): fp32 slice products, the
  // slices' group-sum scratch and the side streams they run on
  static constexpr int kSplitK = 4;
  static constexpr int kSplitKMaxRows = 64;
  float* sk_f = nullptr;     // [kSplitK][rows <= kSplitKMaxRows][N <= sk_n]
  int sk_n = 0;              // widest projection the slice products hold
  char* sk_xs = nullptr;     // kSplitK regions of sk_xs_stride bytes
  size_t sk_xs_stride = 0;
  cudaStream_t sk_st[kSplitK] = {};
  cudaEvent_t sk_fork = nullptr, sk_join[kSplitK] = {};
};

// Token count from which a projection runs as the tensor-core GEMM instead of
// chunks of the streaming GEMV (the GEMV re-reads the weights every 8 tokens).
constexpr int kGemmMinTokens = 16;
// Projections take the tensor-core GEMM from this many rows on (split over K
// when few output tiles would leave SMs idle).  Its dequant
// work per weight does not shrink with the row count, but neither do GEMV
// passes of 8 rows (2 rows for K = 25600) win below it: Qwen3-32B batch 16 at
// 32K measured 224.9 tok/s with the GEMM and 216.7 with GEMV passes.
constexpr int kGemmMinRows = 16;
// Routed experts of a call go through the per-expert GEMMs from this many
// tokens on (below, the per-token expert GEMVs: too few rows per expert).
constexpr int kMoeGroupedMinTokens = 64;


static bool parse_layer(const char* name, int& idx, const char*& rest) {
  const char* p = "model.layers.";
  if (strncmp(name, p, strlen(p)) != 0) return false;
  const char* s = name + strlen(p);
  char* end = nullptr;
  long v = strtol(s, &end, 10);
  if (end == s || *end != '.') return false;
  idx = (int)v;
  rest = end + 1;
  return true;
}

static bool bind_linear(Linear& l, const char* suffix, const void* ptr) {
  if (!strcmp(suffix, "weight")) l.w = (const uint32_t*)ptr;
  else if (!strcmp(suffix, "scales")) l.s = (const bf16*)ptr;
  else if (!strcmp(suffix, "biases")) l.b = (const bf16*)ptr;
  else return false;
  return true;
}

// `base` names a module ("self_attn.q_proj"); the tensor is base + "." + suffix.
static bool match(const char* rest, const char* base, const char*& suffix) {
  size_t n = strlen(base);
  if (strncmp(rest, base, n) != 0 || rest[n] != '.') return false;
  suffix = rest + n + 1;
  return true;
}

static int bind(Model* m, const char* name, const void* ptr) {
  const char* suffix = nullptr;
  if (match(name, "model.embed_tokens", suffix)) return bind_linear(m->embed, suffix, ptr) ? M5_OK : -1;
  if (match(name, "lm_head", suffix)) return bind_linear(m->lm_head, suffix, ptr) ? M5_OK : -1;
  if (!strcmp(name, "model.norm.weight")) { m->final_norm = (const bf16*)ptr; return M5_OK; }
  int li;
  const char* rest;
  if (!parse_layer(name, li, rest) || li < 0 || li >= (int)m->layers.size()) return -1;
  Layer& L = m->layers[li];
  if (!strcmp(rest, "input_layernorm.weight")) { L.in_norm = (const bf16*)ptr; return M5_OK; }
  if (!strcmp(rest, "post_attention_layernorm.weight")) { L.post_norm = (const bf16*)ptr; return M5_OK; }
  if (!strcmp(rest, "self_attn.q_norm.weight")) { L.q_norm = (const bf16*)ptr; return M5_OK; }
  if (!strcmp(rest, "self_attn.k_norm.weight")) { L.k_norm = (const bf16*)ptr; return M5_OK; }
  struct { const char* base; Linear* l; } table[] = {
      {"self_attn.q_proj", &L.q}, {"self_attn.k_proj", &L.k}, {"self_attn.v_proj", &L.v},
      {"self_attn.o_proj", &L.o}, {"mlp.gate_proj", &L.gate}, {"mlp.up_proj", &L.up},
      {"mlp.down_proj", &L.down}, {"mlp.gate", &L.router}, {"mlp.switch_mlp.gate_proj", &L.e_gate},
      {"mlp.switch_mlp.up_proj", &L.e_up}, {"mlp.switch_mlp.down_proj", &L.e_down},
  };
  for (auto& t : table)
    if (match(rest, t.base, suffix)) return bind_linear(*t.l, suffix, ptr) ? M5_OK : -1;
  return -1;
}

static std::string missing(const Model* m) {
  const bool moe = m->cfg.num_experts > 0;
  if (!m->embed.ok()) return "model.embed_tokens";
  if (!m->final_norm) return "model.norm.weight";
  if ((!m->cfg.tie_word_embeddings || m->cfg.tp_size > 1) && !m->lm_head.ok())
    return m->cfg.tp_size > 1 ? "lm_head (this rank's vocabulary rows; tied models bind a slice of the embedding)"
                              : "lm_head";
  for (size_t i = 0; i < m->layers.size(); ++i) {
    const Layer& L = m->layers[i];
    std::string p = "model.layers." + std::to_string(i) + ".";
    if (!L.in_norm) return p + "input_layernorm.weight";
    if (!L.post_norm) return p + "post_attention_layernorm.weight";
    if (!L.q_norm) return p + "self_attn.q_norm.weight";
    if (!L.k_norm) return p + "self_attn.k_norm.weight";
    if (!L.q.ok()) return p + "self_attn.q_proj";
    if (!L.k.ok()) return p + "self_attn.k_proj";
    if (!L.v.ok()) return p + "self_attn.v_proj";
    if (!L.o.ok()) return p + "self_attn.o_proj";
    if (moe) {
      if (!L.router.ok()) return p + "mlp.gate";
      if (!L.e_gate.ok()) return p + "mlp.switch_mlp.gate_proj";
      if (!L.e_up.ok()) return p + "mlp.switch_mlp.up_proj";
      if (!L.e_down.ok()) return p + "mlp.switch_mlp.down_proj";
    } else {
      if (!L.gate.ok()) return p + "mlp.gate_proj";
      if (!L.up.ok()) return p + "mlp.up_proj";
      if (!L.down.ok()) return p + "mlp.down_proj";
    }
  }
  return "";
}

static char* carve(char*& p, size_t bytes) {
  char* r = p;
  p += (bytes + 255) & ~size_t(255);
  return r;
}

// y rows for x [T, K] through one or more weight segments, in chunks of the
// largest token count the GEMV can stage.
static int linear_tokens(const GemvArgs& proto, int T, int epi, cudaStream_t st) {
  const int cap = gemv_max_tokens(proto.K);
  if (cap <= 0) return fail(M5_ERR_UNSUPPORTED, "linear: K too large for the decode GEMV");
  for (int t0 = 0; t0 < T;) {
    int mt = std::min(8, T - t0);
    if (!gemv_mma_eligible(proto, mt, epi)) {
      mt = 1;
      while (mt * 2 <= std::min(cap, T - t0)) mt *= 2;
    }
    GemvArgs a = proto;
    a.x = proto.x + size_t(t0) * proto.ldx;
    for (int i = 0; i < a.nseg; ++i) {
      if (a.seg[i].y) a.seg[i].y = proto.seg[i].y + size_t(t0) * proto.ldy;
      if (a.seg[i].yf) a.seg[i].yf = proto.seg[i].yf + size_t(t0) * proto.ldy;
    }
    int rc = gemv_launch(a, mt, epi, st);
    if (rc) return rc;
    t0 += mt;
  }
  return M5_OK;
}

static void attach(const Model* m, GemvArgs& a) {
  a.mma_acc = m->mma_acc;
  a.mma_cnt = m->mma_cnt;
  a.mma_rows = m->mma_rows;
  a.mma_part = m->gemv_part;
  a.mma_part_floats = m->gemv_part ? gemv_part_floats() : 0;
}

// One projection of T tokens: the tensor-core GEMM for prefill-sized T (with
// the fused RMSNorm materialised first), the streaming GEMV otherwise.
// A projection of few rows with few output tiles (batched decode's o_proj and
// down: N / 128 = 40 tiles on a 148-SM GPU; MoE shapes' q|k|v and router)
// leaves most SMs idle as one GEMM.  Its
// K range is cut into slices of whole 8-group blocks that run as concurrent
// GEMMs on side streams, each writing fp32 products, and one kernel adds the
// slices in order and applies the epilogue.
static int gemm_splitk(const Model* m, const GemvArgs& a, int T, int epi, cudaStream_t st) {
  const int N = a.seg[0].rows, G = a.K / 64;
  const int tiles = (N / 128) * ((T + 127) / 128);
  const int S = std::min({Model::kSplitK, sm_count() / std::max(1, tiles), G / 8});
  if (S < 2 || N > m->sk_n || a.ldk || a.K % 512)
    return gemm_tc_launch(a, T, epi, m->gxs, m->gxs_bytes, st);
  M5_CUDA(cudaEventRecord(m->sk_fork, st));
  const int G8 = G / 8;
  const size_t slice = size_t(T) * N;
  for (int sl = 0; sl < S; ++sl) {
    const int g0 = 8 * (G8 * sl / S), g1 = 8 * (G8 * (sl + 1) / S);
    GemvArgs b = a;
    b.K = (g1 - g0) * 64;
    b.ldk = a.K;
    b.x = a.x + size_t(g0) * 64;
    b.seg[0].w = a.seg[0].w + size_t(g0) * 8;  // 8 words of codes per group
    b.seg[0].s = a.seg[0].s + g0;
    b.seg[0].b = a.seg[0].b + g0;
    b.seg[0].y = nullptr;
    b.seg[0].yf = m->sk_f + sl * slice;
    b.ldy = N;
    M5_CUDA(cudaStreamWaitEvent(m->sk_st[sl], m->sk_fork, 0));
    const int rc = gemm_tc_launch(b, T, EPI_F32, reinterpret_cast<bf16*>(m->sk_xs + sl * m->sk_xs_stride),
                                  m->sk_xs_stride, m->sk_st[sl]);
    M5_CUDA(cudaEventRecord(m->sk_join[sl], m->sk_st[sl]));
    M5_CUDA(cudaStreamWaitEvent(st, m->sk_join[sl], 0));
    if (rc) return rc;
  }
  return gemm_splitk_reduce_launch(m->sk_f, S, T, N, epi, a.seg[0].y, a.seg[0].yf, a.ldy, st);
}

static int linear_auto(const Model* m, const GemvArgs& proto, int T, int epi, cudaStream_t st) {
  if (T >= kGemmMinRows && m->gxs && gemm_tc_xs_bytes(T, proto.K) <= m->gxs_bytes) {
    GemvArgs a = proto;
    if (proto.norm_w) {
      a.norm_w = nullptr;
      a.x = m->xn;
      a.ldx = a.K;
    }
    const bool norm_fits = !proto.norm_w || proto.K == m->cfg.hidden_size;  // xn holds [T, H]
    if (norm_fits && gemm_tc_eligible(a, T, epi)) {
      if (proto.norm_w) {
        int rc = rms_norm_launch(proto.x, proto.norm_w, T, a.K, proto.eps, m->xn, st);
        if (rc) return rc;
      }
      if (T <= Model::kSplitKMaxRows && m->sk_f && a.nseg == 1 && epi != EPI_SWIGLU)
        return gemm_splitk(m, a, T, epi, st);
      return gemm_tc_launch(a, T, epi, m->gxs, m->gxs_bytes, st);
    }
  }
  return linear_tokens(proto, T, epi, st);
}

static GemvSeg seg_of(const Linear& l, int rows, bf16* y) {
  GemvSeg s{};
  s.w = l.w;
  s.s = l.s;
  s.b = l.b;
  s.rows = rows;
  s.y = y;
  return s;
}

// vgather [tp][R][Vl] (rank-major, as the all-gather leaves it) -> out [R][tp * Vl]
__global__ void vocab_unshard_kernel(const bf16* __restrict__ g, int tp, int R, int Vl, bf16* __restrict__ out) {
  const int64_t n = int64_t(tp) * R * Vl;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t j = i % Vl, rr = (i / Vl) % R, k = i / (int64_t(Vl) * R);
    out[rr * (int64_t(tp) * Vl) + k * Vl + j] = g[i];
  }
}

// Sum the fp32 partials of every rank and add them to the residual stream.
static int reduce_into_h(Model* m, int L, cudaStream_t st) {
  return comm_allreduce_residual(m->comm, m->hf, m->h, int64_t(L) * m->cfg.hidden_size, st);
}

// Final norm + lm_head of `rows` tokens starting at hidden row `h0`; under
// tensor parallelism each rank computes its vocabulary rows and the shards
// are gathered, so `out` ([rows, V]) is complete on every rank.
static int head_rows(Model* m, const Linear& head, int h0, int rows, bf16* out, cudaStream_t st) {
  const m5_model_cfg& c = m->cfg;
  const int H = c.hidden_size, V = c.vocab_size, tp = c.tp_size;
  GemvArgs hd{};
  hd.ldx = H;
  hd.K = H;
  hd.nseg = 1;
  hd.norm_w = m->final_norm;
  hd.eps = c.rms_norm_eps;
  attach(m, hd);
  if (tp == 1) {
    hd.x = m->h + size_t(h0) * H;
    hd.ldy = V;
    hd.total_rows = V;
    hd.seg[0] = seg_of(head, V, out);
    return linear_auto(m, hd, rows, EPI_STORE, st);
  }
  for (int r0 = 0; r0 < rows; r0 += m->v_rows) {
    const int R = std::min(m->v_rows, rows - r0);
    hd.x = m->h + size_t(h0 + r0) * H;
    hd.ldy = m->Vl;
    hd.total_rows = m->Vl;
    hd.seg[0] = seg_of(head, m->Vl, m->vpart);
    int rc = linear_auto(m, hd, R, EPI_STORE, st);
    if (rc) return rc;
    if ((rc = comm_allgather_bf16(m->comm, m->vpart, m->vgather, int64_t(R) * m->Vl, st))) return rc;
    bf16* dst = out + size_t(r0) * V;
    if (R == 1) {
      M5_CUDA(cudaMemcpyAsync(dst, m->vgather, size_t(tp) * m->Vl * sizeof(bf16), cudaMemcpyDeviceToDevice, st));
    } else {
      const int64_t n = int64_t(tp) * R * m->Vl;
      const int blocks = (int)std::min<int64_t>((n + 255) / 256, sm_count() * 8);
      vocab_unshard_kernel<<<blocks, 256, 0, st>>>(m->vgather, tp, R, m->Vl, dst);
      M5_LAUNCH_CHECK("vocabulary gather launch");
    }
  }
  return M5_OK;
}

__global__ void add_len_kernel(int32_t* d_len, int L) {
  pdl_wait();
  pdl_launch_dependents();
  *d_len += L;
}

// Routed experts of T >= kMoeGroupedMinTokens tokens grouped by expert: counting
// sort of the (token, slot) pairs, the normalised rows gathered into expert
// order, one host sync for the per-expert counts, then per local expert a
// gate/up (SwiGLU) and a down tensor-core GEMM over just its rows, spread over
// side streams, and a per-token combine in slot order.  Each expert's weights
// stream once per chunk instead of once per routed token.
static int moe_prefill_grouped(Model* m, const Layer& ly, int T, cudaStream_t st) {
  const m5_model_cfg& c = m->cfg;
  const int H = c.hidden_size, I = m->I, k = c.experts_per_tok, El = m->E_local, pairs = T * k;
  int rc = rms_norm_launch(m->h, ly.post_norm, T, H, c.rms_norm_eps, m->xn, st);
  if (!rc) rc = moe_sort_launch(m->rids, pairs, m->e_first, El, m->moe_cnt, m->moe_cnt + El, m->moe_pos, st);
  if (!rc) rc = moe_gather_launch(m->xn, H, pairs, k, m->moe_pos, m->moe_x, st);
  if (rc) return rc;
  M5_CUDA(cudaMemcpyAsync(m->h_moe_cnt, m->moe_cnt, size_t(El) * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  M5_CUDA(cudaStreamSynchronize(st));
  M5_CUDA(cudaEventRecord(m->moe_fork, st));
  for (int i = 0; i < Model::kMoeStreams; ++i) M5_CUDA(cudaStreamWaitEvent(m->moe_st[i], m->moe_fork, 0));
  const size_t xs_h = size_t(64) * ((H / 64 + 31) / 32), xs_i = size_t(64) * ((I / 64 + 31) / 32);
  bf16* xs_gu = m->moe_xs;
  bf16* xs_dn = m->moe_xs + size_t(pairs) * xs_h;
  const size_t H8 = H / 8, H64 = H / 64, I8 = I / 8, I64 = I / 64;
  int off = 0, used = 0;
  for (int e = 0; e < El && !rc; ++e) {
    const int n = m->h_moe_cnt[e];
    if (n <= 0) continue;
    cudaStream_t ss = m->moe_st[used++ % Model::kMoeStreams];
    GemvArgs g{};
    g.x = m->moe_x + size_t(off) * H;
    g.ldx = H;
    g.K = H;
    g.nseg = 2;
    g.seg[0] = GemvSeg{ly.e_gate.w + size_t(e) * I * H8, ly.e_gate.s + size_t(e) * I * H64,
                       ly.e_gate.b + size_t(e) * I * H64, I, m->moe_act + size_t(off) * I, nullptr};
    g.seg[1] = GemvSeg{ly.e_up.w + size_t(e) * I * H8, ly.e_up.s + size_t(e) * I * H64,
                       ly.e_up.b + size_t(e) * I * H64, I, nullptr, nullptr};
    g.ldy = I;
    g.total_rows = I;
    rc = gemm_tc_launch(g, n, EPI_SWIGLU, xs_gu + size_t(off) * xs_h, size_t(n) * xs_h * 2, ss);
    if (rc) break;
    GemvArgs d{};
    d.x = m->moe_act + size_t(off) * I;
    d.ldx = I;
    d.K = I;
    d.nseg = 1;
    d.seg[0] = GemvSeg{ly.e_down.w + size_t(e) * H * I8, ly.e_down.s + size_t(e) * H * I64,
                       ly.e_down.b + size_t(e) * H * I64, H, m->moe_y + size_t(off) * H, nullptr};
    d.ldy = H;
    d.total_rows = H;
    rc = gemm_tc_launch(d, n, EPI_STORE, xs_dn + size_t(off) * xs_i, size_t(n) * xs_i * 2, ss);
    off += n;
  }
  for (int i = 0; i < Model::kMoeStreams; ++i) {  // join even after an error: no stream is left behind
    M5_CUDA(cudaEventRecord(m->moe_join[i], m->moe_st[i]));
    M5_CUDA(cudaStreamWaitEvent(st, m->moe_join[i], 0));
  }
  if (rc) return rc;
  return moe_combine_launch(m->moe_y, T, H, k, m->moe_pos, m->rscores, m->h, c.ep_size > 1 ? m->hf : nullptr, st);
}

// QK-norm + RoPE + KV append run in the q|k|v GEMV's epilogue for decode-sized
// calls (M5_FUSE_ROPE=0 keeps the separate kernel).
static bool fuse_rope() {
  static const bool on = [] {
    const char* e = getenv("M5_FUSE_ROPE");
    return !(e && e[0] == '0');
  }();
  return on;
}

static bool stream_capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
}

// One model call: L tokens of one sequence at positions *d_len.., or (B > 1,
// L == 1) one token of each of B sequences, all at position *d_len, over a
// cache of [B, Hkv, capacity, ...] layers.  T = L * B activation rows.
static int forward(Model* m, const m5_layer_kv* kv, int32_t* d_len, const int32_t* d_tokens, int L, void* logits,
                   int logits_mode, int32_t* d_argmax, cudaStream_t st, int B = 1) {
  const int T = L * B;
  const m5_model_cfg& c = m->cfg;
  const int H = c.hidden_size, D = c.head_dim;
  const int Hq = m->Hq, Hkv = m->Hkv;
  const int QKV = (Hq + 2 * Hkv) * D;
  int rc = embed_launch(d_tokens, T, m->embed.w, m->embed.s, m->embed.b, H, c.vocab_size, m->h, st);
  if (rc) return rc;
  for (int li = 0; li < c.num_layers; ++li) {
    const Layer& ly = m->layers[li];
    const m5_layer_kv& lk = kv[li];
    // q | k | v projections of RMSNorm(h)
    GemvArgs a{};
    a.x = m->h;
    a.ldx = H;
    a.K = H;
    a.nseg = 3;
    a.seg[0] = seg_of(ly.q, Hq * D, m->qkv);
    a.seg[1] = seg_of(ly.k, Hkv * D, m->qkv + Hq * D);
    a.seg[2] = seg_of(ly.v, Hkv * D, m->qkv + (Hq + Hkv) * D);
    a.ldy = QKV;
    a.total_rows = QKV;
    a.norm_w = ly.in_norm;
    a.eps = c.rms_norm_eps;
    attach(m, a);
    // QK-norm + RoPE + KV append
    RopeAppendArgs r{};
    r.qkv = m->qkv;
    r.L = T;
    r.batch = B;
    r.Hq = Hq;
    r.Hkv = Hkv;
    r.q_norm = ly.q_norm;
    r.k_norm = ly.k_norm;
    r.eps = c.rms_norm_eps;
    r.inv_freq = m->d_inv_freq;
    r.mscale = m->mscale;
    r.d_len = d_len;
    r.q_out = m->q;
    r.kv = lk;
    if (T < kGemmMinRows && T <= 8 && D == 128 && fuse_rope() && gemv_tmap_eligible(a, T, EPI_STORE)) {
      // one launch: the GEMV's epilogue appends each head once its rows are written
      a.rope = r;
      a.rope_cnt = m->rope_cnt;
      if ((rc = gemv_launch(a, T, EPI_STORE, st))) return rc;
    } else {
      if ((rc = linear_auto(m, a, T, EPI_STORE, st))) return rc;
      if ((rc = rope_append_launch(r, st))) return rc;
    }
    // attention over the cache (S = *d_len + L keys after the append)
    AttnArgs at{};
    at.q = m->q;
    at.B = B;
    at.Hq = Hq;
    at.L = L;
    at.D = D;
    at.k = m5_kv_view{lk.k, lk.k_scales, lk.k_biases, int64_t(Hkv) * lk.capacity, lk.capacity};
    at.v = m5_kv_view{lk.v, lk.v_scales, lk.v_biases, int64_t(Hkv) * lk.capacity, lk.capacity};
    at.bits = lk.bits;
    at.Hkv = Hkv;
    at.d_S = d_len;
    at.S_add = L;
    at.scale = 1.f / sqrtf(float(D));
    at.mask_kind = L > 1 ? M5_MASK_CAUSAL : M5_MASK_NONE;
    attn_plan(B, Hq, Hkv, L, (int)lk.capacity, at.QB, at.nsplit);
    if (attn_scratch_bytes(B, Hq, L, D, at.nsplit) > m->attn_part_bytes) at.nsplit = 1;
    at.part_o = m->attn_part;
    at.part_ml = m->attn_part + size_t(B) * Hq * L * at.nsplit * D;
    at.out = m->attn;
    at.out_tokens_major = 1;
    if ((rc = attn_launch(at, st))) return rc;
    // o_proj, residual add into h
    GemvArgs o{};
    o.x = m->attn;
    o.ldx = Hq * D;
    o.K = Hq * D;
    o.nseg = 1;
    o.seg[0] = seg_of(ly.o, H, m->h);
    o.ldy = H;
    o.total_rows = H;
    attach(m, o);
    if (c.tp_size > 1) {  // this rank's heads give a partial sum over o_proj's columns
      o.seg[0].yf = m->hf;
      if ((rc = linear_auto(m, o, T, EPI_F32, st)) || (rc = reduce_into_h(m, T, st))) return rc;
    } else if ((rc = linear_auto(m, o, T, EPI_RESIDUAL, st))) {
      return rc;
    }
    if (c.num_experts == 0) {
      GemvArgs g{};
      g.x = m->h;
      g.ldx = H;
      g.K = H;
      g.nseg = 2;
      g.seg[0] = seg_of(ly.gate, m->I, m->act);
      g.seg[1] = seg_of(ly.up, m->I, nullptr);
      g.ldy = m->I;
      g.total_rows = m->I;
      g.norm_w = ly.post_norm;
      g.eps = c.rms_norm_eps;
      attach(m, g);
      if ((rc = linear_auto(m, g, T, EPI_SWIGLU, st))) return rc;
      GemvArgs d{};
      d.x = m->act;
      d.ldx = m->I;
      d.K = m->I;
      d.nseg = 1;
      d.seg[0] = seg_of(ly.down, H, m->h);
      d.ldy = H;
      d.total_rows = H;
      attach(m, d);
      if (c.tp_size > 1) {  // this rank's intermediate columns give a partial sum
        d.seg[0].yf = m->hf;
        if ((rc = linear_auto(m, d, T, EPI_F32, st)) || (rc = reduce_into_h(m, T, st))) return rc;
      } else if ((rc = linear_auto(m, d, T, EPI_RESIDUAL, st))) {
        return rc;
      }
    } else {
      // router logits of RMSNorm(h), top-k, then the routed experts
      GemvArgs g{};
      g.x = m->h;
      g.ldx = H;
      g.K = H;
      g.nseg = 1;
      g.seg[0] = seg_of(ly.router, c.num_experts, m->rlogits);
      g.ldy = c.num_experts;
      g.total_rows = c.num_experts;
      g.norm_w = ly.post_norm;
      g.eps = c.rms_norm_eps;
      attach(m, g);
      MoeRouterArgs ra{m->h,          ly.post_norm,      c.rms_norm_eps,  ly.router.w,
                       ly.router.s,   ly.router.b,       H,               c.num_experts,
                       c.experts_per_tok, c.norm_topk_prob, m->rlogits,   m->rids,
                       m->rscores,    m->moe_ncnt + H / 16};
      if (T == 1 && m->moe_ncnt && c.num_experts <= 256 && H % 256 == 0) {  // one launch for a decode token
        if ((rc = moe_router_topk_launch(ra, st))) return rc;
      } else {
        if ((rc = linear_auto(m, g, T, EPI_STORE, st))) return rc;
        if ((rc = moe_topk_launch(m->rlogits, T, c.num_experts, c.experts_per_tok, c.norm_topk_prob, m->rids,
                                  m->rscores, st)))
          return rc;
      }
      MoeArgs me{};
      me.x = m->h;
      me.T = T;
      me.H = H;
      me.I = c.moe_intermediate_size;
      me.k = c.experts_per_tok;
      me.e_first = m->e_first;
      me.e_local = m->E_local;
      me.ids = m->rids;
      me.scores = m->rscores;
      me.gate = {ly.e_gate.w, ly.e_gate.s, ly.e_gate.b};
      me.up = {ly.e_up.w, ly.e_up.s, ly.e_up.b};
      me.down = {ly.e_down.w, ly.e_down.s, ly.e_down.b};
      me.norm_w = ly.post_norm;
      me.eps = c.rms_norm_eps;
      me.act = m->act;
      me.h = m->h;
      me.acc = m->mma_acc;
      me.cnt = m->mma_cnt;
      me.acc_rows = m->mma_rows;
      me.ybuf = m->moe_ybuf;
      me.ncnt = m->moe_ncnt;
      if (c.ep_size > 1) me.partial = m->hf;  // this rank's experts give a partial sum
      if (T >= kMoeGroupedMinTokens && m->moe_x && T <= m->max_tokens && !stream_capturing(st))
        rc = moe_prefill_grouped(m, ly, T, st);
      else
        rc = moe_mma_eligible(me) ? moe_mma_launch(me, st) : moe_launch(me, st);
      if (rc || (c.ep_size > 1 && (rc = reduce_into_h(m, T, st)))) return rc;
    }
  }
  // final norm + lm_head (+ argmax)
  const Linear& head = (c.tie_word_embeddings && c.tp_size == 1) ? m->embed : m->lm_head;
  const int V = c.vocab_size;
  bf16* last_row = nullptr;
  if (B > 1) {  // every row is the last (only) token of its sequence: logits [B, V]
    bf16* out = logits_mode == M5_LOGITS_NONE ? nullptr : (bf16*)logits;
    if (out || d_argmax) {
      if (!out) return fail(M5_ERR_INVALID, "batched forward: argmax needs a logits buffer");
      if ((rc = head_rows(m, head, 0, B, out, st))) return rc;
      if (d_argmax && (rc = argmax_rows_launch(out, B, V, d_argmax, st))) return rc;
    }
  } else if (logits_mode == M5_LOGITS_ALL) {
    if ((rc = head_rows(m, head, 0, L, (bf16*)logits, st))) return rc;
    last_row = (bf16*)logits + size_t(L - 1) * V;
  } else if (logits_mode == M5_LOGITS_LAST || d_argmax) {
    last_row = logits_mode == M5_LOGITS_LAST ? (bf16*)logits : m->logits_last;
    if ((rc = head_rows(m, head, L - 1, 1, last_row, st))) return rc;
  }
  if (d_argmax && last_row) {
    if ((rc = argmax_launch(last_row, V, d_argmax, m->argmax_scratch, st))) return rc;
  }
  M5_CUDA(launch_pdl(add_len_kernel, dim3(1), dim3(1), 0, st, d_len, L));
  return M5_OK;
}

// --------------------------------------------------- standalone scratch
// Grow-only per-device arena for the standalone attention entry point.
struct Arena {
  void* ptr = nullptr;
  size_t bytes = 0;
};
static std::mutex g_arena_mu;
enum { ARENA_ATTN = 0, ARENA_GEMM = 1 };
static Arena g_arena[2][64];

static int arena_get(size_t bytes, void** out, int slot = ARENA_ATTN) {
  int dev = 0;
  M5_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(M5_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_arena_mu);
  Arena& a = g_arena[slot][dev];
  if (a.bytes < bytes) {
    if (a.ptr) {
      M5_CUDA(cudaDeviceSynchronize());
      M5_CUDA(cudaFree(a.ptr));
      a.ptr = nullptr;
      a.bytes = 0;
    }
    M5_CUDA(cudaMalloc(&a.ptr, bytes));
    a.bytes = bytes;
  }
  *out = a.ptr;
  return M5_OK;
}

}  // namespace m5

using namespace m5;

extern "C" int m5_device_status(int* code, int reset) {
  M5_CHECK_ARG(code, "m5_device_status: null pointer");
  M5_CUDA(cudaDeviceSynchronize());
  const int g = gemv_tma_error(reset);
  const int gt = gemv_tmap_error(reset);
  const int at = attn_mma_error(reset);
  const int gm = gemm_tc_error(reset);
  const int ap = attn_pf_error(reset);
  const int ar = comm_ar_error(reset);
  const int atc = attn_tc_error(reset);
  if (g < 0 || gt < 0 || at < 0 || gm < 0 || ap < 0 || ar < 0 || atc < 0)
    return fail(M5_ERR_CUDA, "m5_device_status: cannot read the device error words");
  *code = g | gt | at | gm | ap | ar | atc;
  return M5_OK;
}

extern "C" int m5_quantized_matmul(const void* x, int64_t M, int64_t K, const uint32_t* wq, const void* scales,
                                   const void* biases, int64_t N, int group_size, int bits, void* y, void* stream) {
  M5_CHECK_ARG(x && wq && scales && biases && y, "m5_quantized_matmul: null pointer");
  M5_CHECK_ARG(bits == 4 && group_size == 64, "m5_quantized_matmul: only 4-bit group-64 weights");
  M5_CHECK_ARG(K > 0 && K % 64 == 0 && N > 0 && M >= 0, "m5_quantized_matmul: K must be a multiple of 64");
  M5_CHECK_ARG(N < (1LL << 31) && K < (1LL << 31) && M < (1LL << 31), "m5_quantized_matmul: size too large");
  if (M == 0) return M5_OK;
  GemvArgs a{};
  a.x = (const bf16*)x;
  a.ldx = K;
  a.K = (int)K;
  a.nseg = 1;
  a.seg[0].w = wq;
  a.seg[0].s = (const bf16*)scales;
  a.seg[0].b = (const bf16*)biases;
  a.seg[0].rows = (int)N;
  a.seg[0].y = (bf16*)y;
  a.ldy = N;
  a.total_rows = (int)N;
  if (M >= kGemmMinTokens && gemm_tc_eligible(a, (int)M, EPI_STORE)) {
    void* xs = nullptr;
    const size_t bytes = gemm_tc_xs_bytes((int)M, (int)K);
    int rc = arena_get(bytes, &xs, ARENA_GEMM);
    if (rc) return rc;
    return gemm_tc_launch(a, (int)M, EPI_STORE, (bf16*)xs, bytes, (cudaStream_t)stream);
  }
  return linear_tokens(a, (int)M, EPI_STORE, (cudaStream_t)stream);
}

extern "C" int m5_rms_norm(const void* x, const void* w, int64_t rows, int64_t dim, float eps, void* y, void* stream) {
  M5_CHECK_ARG(x && w && y, "m5_rms_norm: null pointer");
  M5_CHECK_ARG(dim > 0 && rows >= 0, "m5_rms_norm: bad shape");
  return rms_norm_launch((const bf16*)x, (const bf16*)w, rows, (int)dim, eps, (bf16*)y, (cudaStream_t)stream);
}

extern "C" int m5_quantized_sdpa(const void* q, int B, int Hq, int L, int D, m5_kv_view keys, m5_kv_view values,
                                 int Hkv, int S, float scale, int mask_kind, const void* mask,
                                 const int64_t* mask_strides, int group_size, int bits, void* out, void* stream) {
  M5_CHECK_ARG(q && out && keys.data && values.data, "m5_quantized_sdpa: null pointer");
  M5_CHECK_ARG(B > 0 && Hq > 0 && Hkv > 0 && L > 0 && S > 0, "m5_quantized_sdpa: empty shape");
  M5_CHECK_ARG(Hq % Hkv == 0, "m5_quantized_sdpa: Hq must be a multiple of Hkv");
  M5_CHECK_ARG(D == 64 || D == 128, "m5_quantized_sdpa: head_dim must be 64 or 128");
  M5_CHECK_ARG(bits == 0 || bits == 4 || bits == 8, "m5_quantized_sdpa: bits must be 0, 4 or 8");
  M5_CHECK_ARG(bits == 0 || group_size == 64, "m5_quantized_sdpa: group_size must be 64");
  M5_CHECK_ARG(bits == 0 || (keys.scales && keys.biases && values.scales && values.biases),
               "m5_quantized_sdpa: packed K/V need scales and biases");
  M5_CHECK_ARG(mask_kind >= M5_MASK_NONE && mask_kind <= M5_MASK_ADDITIVE, "m5_quantized_sdpa: mask kind");
  M5_CHECK_ARG(mask_kind < M5_MASK_BOOL || (mask && mask_strides), "m5_quantized_sdpa: mask pointer/strides");
  M5_CHECK_ARG(mask_kind != M5_MASK_CAUSAL || L <= S, "m5_quantized_sdpa: causal mask needs L <= S");
  M5_CHECK_ARG(Hq / Hkv <= 16, "m5_quantized_sdpa: GQA group larger than 16");
  AttnArgs a{};
  a.q = (const bf16*)q;
  a.B = B;
  a.Hq = Hq;
  a.L = L;
  a.D = D;
  a.k = keys;
  a.v = values;
  a.bits = bits;
  a.Hkv = Hkv;
  a.S_host = S;
  a.scale = scale;
  a.mask_kind = mask_kind;
  a.mask = mask;
  if (mask_kind >= M5_MASK_BOOL) {
    a.ms_b = mask_strides[0];
    a.ms_h = mask_strides[1];
    a.ms_l = mask_strides[2];
  }
  attn_plan(B, Hq, Hkv, L, S, a.QB, a.nsplit);
  a.out = (bf16*)out;
  const size_t need = attn_scratch_bytes(B, Hq, L, D, a.nsplit);
  if (need) {
    void* p = nullptr;
    int rc = arena_get(need, &p);
    if (rc) return rc;
    a.part_o = (float*)p;
    a.part_ml = a.part_o + size_t(B) * Hq * L * a.nsplit * D;
  }
  return attn_launch(a, (cudaStream_t)stream);
}

extern "C" int m5_argmax_bf16(const void* x, int64_t n, int32_t* out, void* stream) {
  M5_CHECK_ARG(x && out, "m5_argmax_bf16: null pointer");
  M5_CHECK_ARG(n > 0 && n < (1LL << 31), "m5_argmax_bf16: bad length");
  void* p = nullptr;
  int dev = 0;
  M5_CUDA(cudaGetDevice(&dev));
  static std::mutex mu;
  static void* scratch[64] = {nullptr};
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!scratch[dev]) {
      M5_CUDA(cudaMalloc(&scratch[dev], argmax_scratch_bytes()));
      M5_CUDA(cudaMemset(scratch[dev], 0, argmax_scratch_bytes()));
    }
    p = scratch[dev];
  }
  return argmax_launch((const bf16*)x, n, out, p, (cudaStream_t)stream);
}

extern "C" int m5_kv_quantize_layer(const m5_layer_kv* src, const m5_layer_kv* dst, int num_kv_heads, int head_dim,
                                    int len, void* stream) {
  M5_CHECK_ARG(src && dst && src->k && src->v && dst->k && dst->v, "m5_kv_quantize_layer: null pointer");
  M5_CHECK_ARG(dst->k_scales && dst->k_biases && dst->v_scales && dst->v_biases, "m5_kv_quantize_layer: scales");
  M5_CHECK_ARG(dst->group_size == 64, "m5_kv_quantize_layer: group_size must be 64");
  return kv_quantize_layer_launch(*src, *dst, num_kv_heads, head_dim, len, (cudaStream_t)stream);
}

extern "C" int m5_moe_route(const void* x, int T, int H, const uint32_t* gate_w, const void* gate_s, const void* gate_b,
                            int E, int k, int norm_topk_prob, int32_t* ids, void* scores, void* logits_out,
                            void* stream) {
  M5_CHECK_ARG(x && gate_w && gate_s && gate_b && ids && scores, "m5_moe_route: null pointer");
  M5_CHECK_ARG(T >= 0 && H > 0 && H % 64 == 0 && E > 0 && E <= 256 && k > 0 && k <= E && k <= 32,
               "m5_moe_route: bad shape");
  if (T == 0) return M5_OK;
  void* lg = logits_out;
  if (!lg) {
    int rc = arena_get(size_t(T) * E * sizeof(bf16), &lg);
    if (rc) return rc;
  }
  GemvArgs a{};
  a.x = (const bf16*)x;
  a.ldx = H;
  a.K = H;
  a.nseg = 1;
  a.seg[0].w = gate_w;
  a.seg[0].s = (const bf16*)gate_s;
  a.seg[0].b = (const bf16*)gate_b;
  a.seg[0].rows = E;
  a.seg[0].y = (bf16*)lg;
  a.ldy = E;
  a.total_rows = E;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = linear_tokens(a, T, EPI_STORE, st);
  if (rc) return rc;
  return moe_topk_launch((const bf16*)lg, T, E, k, norm_topk_prob, ids, (bf16*)scores, st);
}

extern "C" int m5_model_create(const m5_model_cfg* cfg, void** out) {
  M5_CHECK_ARG(cfg && out, "m5_model_create: null pointer");
  const m5_model_cfg& c = *cfg;
  M5_CHECK_ARG(c.head_dim == 128, "m5_model_create: head_dim must be 128");
  M5_CHECK_ARG(c.bits == 4 && c.group_size == 64, "m5_model_create: weights must be 4-bit group-64");
  M5_CHECK_ARG(c.hidden_size > 0 && c.hidden_size % 64 == 0, "m5_model_create: hidden_size % 64");
  M5_CHECK_ARG(c.num_layers > 0 && c.num_heads > 0 && c.num_kv_heads > 0 && c.num_heads % c.num_kv_heads == 0,
               "m5_model_create: heads");
  M5_CHECK_ARG(c.vocab_size > 0, "m5_model_create: vocab_size");
  const int tp = std::max(1, c.tp_size), ep = std::max(1, c.ep_size);
  M5_CHECK_ARG(c.tp_rank >= 0 && c.tp_rank < tp && c.ep_rank >= 0 && c.ep_rank < ep, "m5_model_create: rank");
  // kv heads split over the ranks, or (fewer kv heads than ranks) each
  // replicated on tp / Hkv consecutive ranks, which hold its group's q heads
  M5_CHECK_ARG(c.num_heads % tp == 0 && (c.num_kv_heads % tp == 0 || tp % c.num_kv_heads == 0),
               "m5_model_create: heads neither split over nor replicate onto tp_size ranks");
  Model* m = new Model();
  m->cfg = c;
  m->cfg.tp_size = tp;
  m->cfg.ep_size = ep;
  m->Hq = c.num_heads / tp;
  m->Hkv = c.num_kv_heads % tp == 0 ? c.num_kv_heads / tp : 1;
  if (c.num_experts > 0) {
    if (c.num_experts % ep || c.moe_intermediate_size % 64 || c.experts_per_tok <= 0) {
      delete m;
      return fail(M5_ERR_INVALID, "m5_model_create: experts not divisible by ep_size or bad MoE sizes");
    }
    m->E_local = c.num_experts / ep;
    m->e_first = c.ep_rank * m->E_local;
    m->I = c.moe_intermediate_size;
  } else {
    if (c.intermediate_size % (64 * tp)) {
      delete m;
      return fail(M5_ERR_INVALID, "m5_model_create: intermediate_size not divisible by 64 * tp_size");
    }
    m->I = c.intermediate_size / tp;
  }
  // a MoE model shards its attention heads only over the ranks that hold its
  // experts: one group, one communicator, two partial-sum reductions per layer
  if (c.num_experts > 0 && tp > 1 && (ep != tp || c.ep_rank != c.tp_rank)) {
    delete m;
    return fail(M5_ERR_UNSUPPORTED, "m5_model_create: a MoE model shards heads only with tp_size == ep_size on the same ranks");
  }
  if (c.num_experts == 0 && ep > 1) {
    delete m;
    return fail(M5_ERR_INVALID, "m5_model_create: ep_size > 1 needs a MoE model");
  }
  if (c.vocab_size % tp) {
    delete m;
    return fail(M5_ERR_INVALID, "m5_model_create: vocab_size not divisible by tp_size");
  }
  m->Vl = c.vocab_size / tp;
  m->layers.resize(c.num_layers);
  *out = m;
  return M5_OK;
}

extern "C" int m5_model_destroy(void* model) {
  Model* m = (Model*)model;
  if (!m) return M5_OK;
  if (m->arena) cudaFree(m->arena);
  if (m->d_inv_freq) cudaFree(m->d_inv_freq);
  if (m->h_moe_cnt) cudaFreeHost(m->h_moe_cnt);
  for (int i = 0; i < Model::kMoeStreams; ++i) {
    if (m->moe_st[i]) cudaStreamDestroy(m->moe_st[i]);
    if (m->moe_join[i]) cudaEventDestroy(m->moe_join[i]);
  }
  if (m->moe_fork) cudaEventDestroy(m->moe_fork);
  for (int i = 0; i < Model::kSplitK; ++i) {
    if (m->sk_st[i]) cudaStreamDestroy(m->sk_st[i]);
    if (m->sk_join[i]) cudaEventDestroy(m->sk_join[i]);
  }
  if (m->sk_fork) cudaEventDestroy(m->sk_fork);
  delete m;
  return M5_OK;
}

extern "C" int m5_model_bind(void* model, const char* name, const void* ptr) {
  M5_CHECK_ARG(model && name && ptr, "m5_model_bind: null argument");
  if (bind((Model*)model, name, ptr) != M5_OK)
    return fail(M5_ERR_INVALID, std::string("m5_model_bind: unknown tensor name '") + name + "'");
  return M5_OK;
}

extern "C" int m5_model_check(void* model) {
  M5_CHECK_ARG(model, "m5_model_check: null model");
  Model* m = (Model*)model;
  std::string miss = missing(m);
  if (!miss.empty()) return fail(M5_ERR_STATE, "model tensor not bound: " + miss);
  if (!m->rope_set) return fail(M5_ERR_STATE, "model RoPE table not set (m5_model_set_rope)");
  if ((m->cfg.tp_size > 1 || m->cfg.ep_size > 1) && !m->comm)
    return fail(M5_ERR_STATE, "multi-rank model has no communicator (m5_model_set_comm)");
  return M5_OK;
}

extern "C" int m5_model_set_comm(void* model, void* comm) {
  M5_CHECK_ARG(model && comm, "m5_model_set_comm: null argument");
  Model* m = (Model*)model;
  const int world = std::max(m->cfg.tp_size, m->cfg.ep_size);
  const int rank = m->cfg.tp_size > 1 ? m->cfg.tp_rank : m->cfg.ep_rank;
  if (comm_size(comm) != world || comm_rank(comm) != rank)
    return fail(M5_ERR_INVALID, "m5_model_set_comm: communicator size/rank do not match the model's shard");
  m->comm = comm;
  return M5_OK;
}

extern "C" int m5_model_set_rope(void* model, const float* inv_freq, float mscale) {
  M5_CHECK_ARG(model && inv_freq, "m5_model_set_rope: null argument");
  Model* m = (Model*)model;
  const int half = m->cfg.head_dim / 2;
  if (!m->d_inv_freq) M5_CUDA(cudaMalloc(&m->d_inv_freq, half * sizeof(float)));
  M5_CUDA(cudaMemcpy(m->d_inv_freq, inv_freq, half * sizeof(float), cudaMemcpyHostToDevice));
  m->mscale = mscale;
  m->rope_set = true;
  return M5_OK;
}

extern "C" int m5_model_reserve(void* model, int max_tokens) {
  M5_CHECK_ARG(model && max_tokens > 0, "m5_model_reserve: bad argument");
  Model* m = (Model*)model;
  if (max_tokens <= m->max_tokens) return M5_OK;
  const m5_model_cfg& c = m->cfg;
  const size_t T = max_tokens, H = c.hidden_size, D = c.head_dim;
  const size_t QKV = size_t(m->Hq + 2 * m->Hkv) * D;
  const size_t k = std::max(1, c.experts_per_tok);
  const size_t act = c.num_experts ? T * k * m->I : T * m->I;
  // Attention partials for decode-sized calls (L <= 16): nsplit <= 3 * SMs
  // (attn_plan fills the SMs once at up to 3 CTAs each).
  const size_t part = attn_scratch_bytes(1, m->Hq, (int)std::min<size_t>(T, 4), (int)D, 3 * sm_count());
  size_t total = 0;
  const int mrows = (int)std::max<size_t>({QKV, H, size_t(2) * m->I, size_t(c.vocab_size),
                                            size_t(std::max(1, c.num_experts)), size_t(16)});
  const int mrows16 = (mrows + 15) / 16 * 16;
  const int maxK = (int)std::max<size_t>({H, size_t(m->Hq) * D, size_t(m->I)});
  const size_t gxs = T >= kGemmMinTokens ? gemm_tc_xs_bytes((int)T, maxK) : 0;
  const bool moe_pre = c.num_experts > 0 && T >= kMoeGroupedMinTokens;  // prefill grouped by expert
  auto gxs_c = [](size_t K) { return (K / 64 + 31) / 32; };         // bias blocks of a GEMM input
  const size_t sk_rows = std::min<size_t>(T, Model::kSplitKMaxRows);
  const size_t sk_n = std::max<size_t>({H, QKV, size_t(std::max(1, c.num_experts))});
  const size_t sk_xs = (gemm_tc_xs_bytes((int)sk_rows, maxK) + 255) & ~size_t(255);  // per slice
  const size_t sizes[] = {T * H * 2, T * QKV * 2, T * m->Hq * D * 2, T * m->Hq * D * 2, act * 2,
                          size_t(c.vocab_size) * 2, T * std::max(1, c.num_experts) * 2, T * k * 2, T * k * 4,
                          part, argmax_scratch_bytes(), gemv_mma_scratch_bytes(mrows16),
                          T >= kGemmMinTokens ? T * H * 2 : 0, gxs,
                          (c.tp_size > 1 || c.ep_size > 1) ? T * H * 4 : 0,
                          c.tp_size > 1 ? std::min<size_t>(T, 16) * m->Vl * 2 : 0,
                          c.tp_size > 1 ? size_t(c.tp_size) * std::min<size_t>(T, 16) * m->Vl * 2 : 0,
                          c.num_experts ? k * H * sizeof(float) : 0,
                          c.num_experts ? (H / 16 + 1) * sizeof(int) : 0,
                          moe_pre ? T * k * H * 2 : 0,
                          moe_pre ? T * k * m->I * 2 : 0,
                          moe_pre ? T * k * H * 2 : 0,
                          moe_pre ? T * k * 64 * (gxs_c(H) + gxs_c(m->I)) * 2 : 0,
                          moe_pre ? T * k * 4 : 0,
                          moe_pre ? size_t(2) * m->E_local * 4 : 0,
                          T >= kGemmMinTokens ? size_t(Model::kSplitK) * sk_rows * sk_n * 4 : 0,
                          T >= kGemmMinTokens ? size_t(Model::kSplitK) * sk_xs : 0,
                          (QKV / 128 + 1) * sizeof(unsigned int), gemv_part_floats() * sizeof(float)};
  for (size_t s : sizes) total += (s + 255) & ~size_t(255);
  char* buf = nullptr;
  M5_CUDA(cudaMalloc(&buf, total));
  M5_CUDA(cudaMemset(buf, 0, total));
  if (m->arena) {
    cudaDeviceSynchronize();
    cudaFree(m->arena);
  }
  m->arena = buf;
  m->arena_bytes = total;
  char* p = buf;
  m->h = (bf16*)carve(p, sizes[0]);
  m->qkv = (bf16*)carve(p, sizes[1]);
  m->q = (bf16*)carve(p, sizes[2]);
  m->attn = (bf16*)carve(p, sizes[3]);
  m->act = (bf16*)carve(p, sizes[4]);
  m->logits_last = (bf16*)carve(p, sizes[5]);
  m->rlogits = (bf16*)carve(p, sizes[6]);
  m->rscores = (bf16*)carve(p, sizes[7]);
  m->rids = (int32_t*)carve(p, sizes[8]);
  m->attn_part = (float*)carve(p, sizes[9]);
  m->attn_part_bytes = sizes[9];
  m->argmax_scratch = carve(p, sizes[10]);
  char* mma = carve(p, sizes[11]);
  m->mma_acc = reinterpret_cast<float*>(mma);
  m->mma_cnt = reinterpret_cast<int*>(mma + size_t(8) * mrows16 * sizeof(float));
  m->mma_rows = mrows16;
  m->xn = sizes[12] ? (bf16*)carve(p, sizes[12]) : nullptr;
  m->gxs = sizes[13] ? (bf16*)carve(p, sizes[13]) : nullptr;
  m->gxs_bytes = sizes[13];
  m->hf = sizes[14] ? (float*)carve(p, sizes[14]) : nullptr;
  m->vpart = sizes[15] ? (bf16*)carve(p, sizes[15]) : nullptr;
  m->vgather = sizes[16] ? (bf16*)carve(p, sizes[16]) : nullptr;
  m->v_rows = (int)std::min<size_t>(T, 16);
  m->moe_ybuf = sizes[17] ? (float*)carve(p, sizes[17]) : nullptr;
  m->moe_ncnt = sizes[18] ? (int*)carve(p, sizes[18]) : nullptr;
  m->moe_x = sizes[19] ? (bf16*)carve(p, sizes[19]) : nullptr;
  m->moe_act = sizes[20] ? (bf16*)carve(p, sizes[20]) : nullptr;
  m->moe_y = sizes[21] ? (bf16*)carve(p, sizes[21]) : nullptr;
  m->moe_xs = sizes[22] ? (bf16*)carve(p, sizes[22]) : nullptr;
  m->moe_pos = sizes[23] ? (int32_t*)carve(p, sizes[23]) : nullptr;
  m->moe_cnt = sizes[24] ? (int32_t*)carve(p, sizes[24]) : nullptr;
  m->sk_f = sizes[25] ? (float*)carve(p, sizes[25]) : nullptr;
  m->sk_n = sizes[25] ? (int)sk_n : 0;
  m->sk_xs = sizes[26] ? carve(p, sizes[26]) : nullptr;
  m->rope_cnt = (unsigned int*)carve(p, sizes[27]);
  m->gemv_part = (float*)carve(p, sizes[28]);
  m->sk_xs_stride = sizes[26] ? sk_xs : 0;
  if (m->sk_f && !m->sk_fork) {
    M5_CUDA(cudaEventCreateWithFlags(&m->sk_fork, cudaEventDisableTiming));
    for (int i = 0; i < Model::kSplitK; ++i) {
      M5_CUDA(cudaStreamCreateWithFlags(&m->sk_st[i], cudaStreamNonBlocking));
      M5_CUDA(cudaEventCreateWithFlags(&m->sk_join[i], cudaEventDisableTiming));
    }
  }
  if (moe_pre && !m->h_moe_cnt) {
    M5_CUDA(cudaMallocHost(&m->h_moe_cnt, size_t(m->E_local) * sizeof(int32_t)));
    M5_CUDA(cudaEventCreateWithFlags(&m->moe_fork, cudaEventDisableTiming));
    for (int i = 0; i < Model::kMoeStreams; ++i) {
      M5_CUDA(cudaStreamCreateWithFlags(&m->moe_st[i], cudaStreamNonBlocking));
      M5_CUDA(cudaEventCreateWithFlags(&m->moe_join[i], cudaEventDisableTiming));
    }
  }
  m->max_tokens = max_tokens;
  return M5_OK;
}

static int check_forward(Model* m, const m5_layer_kv* kv, int rows, int logits_mode, void* logits,
                         const char* who) {
  const std::string w(who);
  M5_CHECK_ARG(logits_mode >= M5_LOGITS_NONE && logits_mode <= M5_LOGITS_ALL, w + ": logits_mode");
  M5_CHECK_ARG(logits_mode == M5_LOGITS_NONE || logits, w + ": logits buffer required");
  if (rows > m->max_tokens) return fail(M5_ERR_STATE, w + ": tokens exceed the m5_model_reserve size");
  std::string miss = missing(m);
  if (!miss.empty()) return fail(M5_ERR_STATE, "model tensor not bound: " + miss);
  if (!m->rope_set) return fail(M5_ERR_STATE, "model RoPE table not set");
  if ((m->cfg.tp_size > 1 || m->cfg.ep_size > 1) && !m->comm)
    return fail(M5_ERR_STATE, "multi-rank model has no communicator (m5_model_set_comm)");
  for (int i = 0; i < m->cfg.num_layers; ++i) {
    const m5_layer_kv& l = kv[i];
    if (!l.k || !l.v || l.capacity <= 0) return fail(M5_ERR_INVALID, w + ": cache layer " + std::to_string(i));
    if (l.bits != 0 && l.bits != 4 && l.bits != 8) return fail(M5_ERR_INVALID, w + ": cache bits");
    if (l.bits && (!l.k_scales || !l.k_biases || !l.v_scales || !l.v_biases || l.group_size != 64))
      return fail(M5_ERR_INVALID, w + ": packed cache needs scales/biases and group 64");
  }
  return M5_OK;
}

extern "C" int m5_forward(void* model, const m5_layer_kv* kv, int32_t* d_len, const int32_t* d_tokens, int L,
                          void* logits, int logits_mode, int32_t* d_argmax, void* stream) {
  M5_CHECK_ARG(model && kv && d_len && d_tokens, "m5_forward: null argument");
  M5_CHECK_ARG(L > 0, "m5_forward: L must be positive");
  Model* m = (Model*)model;
  if (int rc = check_forward(m, kv, L, logits_mode, logits, "m5_forward")) return rc;
  return forward(m, kv, d_len, d_tokens, L, logits, logits_mode, d_argmax, (cudaStream_t)stream);
}

extern "C" int m5_forward_batch(void* model, const m5_layer_kv* kv, int32_t* d_len, const int32_t* d_tokens, int B,
                                void* logits, int logits_mode, int32_t* d_argmax, void* stream) {
  M5_CHECK_ARG(model && kv && d_len && d_tokens, "m5_forward_batch: null argument");
  M5_CHECK_ARG(B > 0, "m5_forward_batch: B must be positive");
  M5_CHECK_ARG(!d_argmax || logits_mode != M5_LOGITS_NONE, "m5_forward_batch: argmax needs logits");
  Model* m = (Model*)model;
  if (int rc = check_forward(m, kv, B, logits_mode, logits, "m5_forward_batch")) return rc;
  return forward(m, kv, d_len, d_tokens, 1, logits, logits_mode, d_argmax, (cudaStream_t)stream, B);
}
