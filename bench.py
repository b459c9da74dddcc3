"""Batch-1 greedy decode and chunked prefill of a Qwen3-family 4-bit model on B200.

`python bench.py [--gpus N] [--steps K] [--warmup W] [--impl m5|reference]
                 [--config qwen3-32b|qwen3-30b-a3b|qwen3-235b-a22b|qwen3-0.6b] [--ctx T] [--kv-bits 8|4]`

The default is the headline workload, Qwen3-32B shape with a 32K-token prompt
and 8-bit KV; the MoE configs default to their BASELINE prompts and KV bits
(30B-A3B: 4K, 8-bit; 235B-A22B: 8K, 4-bit).  A step is one decode token: one
full forward of the model at the current context with greedy argmax, replayed
from a CUDA graph.  Before the timed decode the prompt (seeded random ids,
`--ctx` tokens) is prefilled in chunks of 2048 through the same model and
cache (timed too: `prefill` in the JSON line).  Weights are seeded random MLX
4-bit g64 tensors resident in HBM; every decode step streams more than L2
(~22.6 GB for the 32B shape).  With N > 1 (torchrun) a dense model runs tensor
parallel and a MoE model expert parallel over the N GPUs (one sequence, so
`value` is that sequence's tokens/s and scaling is strong).

Printed JSON (rank 0): value = decode tokens/s; hbm = algorithmic bytes per
token against the measured copy bandwidth; roofline = the dominant kernel
(w4 dequant-GEMV) timed alone with CUDA events; cpu_baseline = the CPU
oracle on a bounded sample of the same step.  `--impl reference` times the
CPU restatement of the reference path (MLX is not installable here) and
prints the same line shape.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "qwen3-32b": dict(model_type="qwen3", hidden_size=5120, num_hidden_layers=64, num_attention_heads=64,
                      num_key_value_heads=8, head_dim=128, intermediate_size=25600, vocab_size=151936,
                      tie_word_embeddings=False, max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6),
    "qwen3-0.6b": dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=151936,
                       tie_word_embeddings=True, max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6),
    "qwen3-30b-a3b": dict(model_type="qwen3_moe", hidden_size=2048, num_hidden_layers=48, num_attention_heads=32,
                          num_key_value_heads=4, head_dim=128, intermediate_size=6144, moe_intermediate_size=768,
                          num_experts=128, num_experts_per_tok=8, norm_topk_prob=True, vocab_size=151936,
                          tie_word_embeddings=False, max_position_embeddings=40960, rms_norm_eps=1e-6,
                          rope_theta=1e6),
    "qwen3-235b-a22b": dict(model_type="qwen3_moe", hidden_size=4096, num_hidden_layers=94, num_attention_heads=64,
                            num_key_value_heads=4, head_dim=128, intermediate_size=12288, moe_intermediate_size=1536,
                            num_experts=128, num_experts_per_tok=8, norm_topk_prob=True, vocab_size=151936,
                            tie_word_embeddings=False, max_position_embeddings=40960, rms_norm_eps=1e-6,
                            rope_theta=1e6),
}
# prompt length and KV bits each config is quoted with
DEFAULTS = {"qwen3-32b": (32768, 8), "qwen3-0.6b": (512, 8), "qwen3-30b-a3b": (4096, 8), "qwen3-235b-a22b": (8192, 4)}
NAMES = {"qwen3-32b": "Qwen3-32B", "qwen3-0.6b": "Qwen3-0.6B", "qwen3-30b-a3b": "Qwen3-30B-A3B",
         "qwen3-235b-a22b": "Qwen3-235B-A22B"}


def weight_bytes_per_token(cfg: dict) -> int:
    """Packed weight bytes one decode token streams (0.5625 B per weight + norms);
    for MoE the router and the k routed experts of every layer."""
    H, L, D = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    Hq, Hkv, I, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["intermediate_size"], cfg["vocab_size"]
    if cfg.get("num_experts", 0):
        mlp = cfg["num_experts"] * H + cfg["num_experts_per_tok"] * 3 * cfg["moe_intermediate_size"] * H
    else:
        mlp = 3 * I * H
    per_layer = (Hq * D * H + 2 * Hkv * D * H + H * Hq * D + mlp) * 0.5625 + (2 * H + 2 * D) * 2
    head = V * H * 0.5625
    return int(L * per_layer + head + H * 2)


def kv_bytes_per_token(cfg: dict, ctx: int, bits: int = 8, kv_heads: int = 0) -> int:
    per_elem = bits / 8 + 4 / 64
    n = kv_heads or cfg["num_key_value_heads"]
    return int(2 * cfg["num_hidden_layers"] * n * cfg["head_dim"] * per_elem * ctx)


def moe_bytes_per_rank(cfg: dict, world: int, ctx: int, bits: int) -> int:
    """Bytes one rank streams for a batch-1 MoE decode token with the heads
    sharded over `world` ranks (kv heads replicated where there are fewer
    than ranks), the router replicated, the lm_head split by rows and the k
    routed experts spread evenly (their expected share)."""
    from myinfer_b200.distributed import kv_heads_local
    H, L, D = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    Hq, V, E = cfg["num_attention_heads"], cfg["vocab_size"], cfg["num_experts"]
    hkv = kv_heads_local(cfg["num_key_value_heads"], world)
    attn = (2 * (Hq // world) * D * H + 2 * hkv * D * H) * 0.5625
    experts = cfg["num_experts_per_tok"] * 3 * cfg["moe_intermediate_size"] * H * 0.5625 / world
    per_layer = attn + E * H * 0.5625 + experts + (2 * H + 2 * D) * 2
    return int(L * per_layer + V // world * H * 0.5625 + H * 2 + kv_bytes_per_token(cfg, ctx, bits, hkv))


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        def run():
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            try:
                p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                      "-lms", "200"], stdout=subprocess.PIPE, text=True)
            except Exception:
                return
            while not self._stop.is_set():
                line = p.stdout.readline()
                if not line:
                    break
                self.samples.append([s.strip() for s in line.split(",")])
            p.terminate()
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        sm = [float(s[0]) for s in self.samples if s and s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if len(s) > 1 and s[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 3 + i and s[3 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def attention_block() -> list:
    """The attention op alone: 64 q / 8 kv heads, D 128,
    bf16 q, K/V N(0, 1) quantized to 8 and 4 bits, at 4K / 32K / 128K keys;
    decode (one query) against HBM, a causal 2048-query prefill chunk against
    bf16 tensor throughput.  Device time per call, graph-replayed; several
    KV sets rotate where they fit so the decode reads come from HBM."""
    from myinfer_b200.microbench import bench_attention
    peaks = measured_peaks()
    out = []
    for s in (4096, 32768, 131072):
        for bits in (8, 4):
            for l in (1, 2048):
                r = bench_attention(s, l, bits, 64, 8, 20 if l == 1 else 3)
                row = {"keys": s, "queries": l, "kv_bits": bits, "us": r["us"]}
                if l == 1:
                    row.update(gbs=r["gbs"], hbm_frac_of_measured=round(r["gbs"] / peaks["hbm_gbs"], 4))
                else:
                    row.update(tflops=r["tflops"], tensor_frac_of_measured=round(r["tflops"] / peaks["bf16_tflops"], 4))
                out.append(row)
    return out


# ----------------------------------------------------------------- CPU legs
def cpu_decode_sample(cfg: dict, ctx: int, kv_bits: int = 8, threads: int = 0, budget_s: float = 20.0) -> dict:
    """The CPU oracle's decode step at the stated context, on a bounded sample.

    Times whole decoder layers of the config (attention over `ctx` cached
    positions in the packed KV layout, the MLP or the routed experts) with the
    oracle's real per-call work: every call dequantizes the packed weights it
    multiplies by (as a quantized matmul does) and the KV it attends over, then
    multiplies in fp32.  Packed codes, scales and biases are random (their
    values do not change the work).  Layers repeat until `budget_s` is spent
    (at least one); the lm_head (vocab x hidden, dequantized per call) is
    timed on a slice of its rows.  One token = layers x the mean layer time +
    the full lm_head."""
    import numpy as np
    import torch

    from oracle import model as om

    if threads:
        torch.set_num_threads(threads)
    c = om.Config.from_dict(dict(cfg, num_hidden_layers=1, vocab_size=16384))
    rng = np.random.default_rng(1)
    w = {}
    for name, shape, kind in om.weight_specs(c):
        if kind == "norm":
            w[name + ".weight"] = np.full(shape, 0x3F80, dtype=np.uint16)
            continue
        K = shape[-1]
        w[name + ".weight"] = rng.integers(0, 2 ** 32, shape[:-1] + (K // 8,), dtype=np.uint32)
        for suf in (".scales", ".biases"):
            w[name + suf] = om.f32_to_bf16_bits((0.01 * rng.standard_normal(shape[:-1] + (K // 64,))).astype(np.float32))
    m = om.Model(c, w)
    words = c.head_dim * kv_bits // 32

    def kv_part():
        return (rng.integers(0, 2 ** 32, (c.num_key_value_heads, ctx, words), dtype=np.uint32),
                om.f32_to_bf16_bits((0.05 * rng.standard_normal((c.num_key_value_heads, ctx, 2))).astype(np.float32)),
                om.f32_to_bf16_bits((0.05 * rng.standard_normal((c.num_key_value_heads, ctx, 2))).astype(np.float32)))
    qc = om.QuantizedKVCache(64, kv_bits)
    qc.k_parts.append(kv_part())
    qc.v_parts.append(kv_part())
    qc.offset = ctx
    x = om.rb(torch.randn(1, cfg["hidden_size"]))
    p = "model.layers.0."
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start < budget_s and len(times) < cfg["num_hidden_layers"]):
        m._deq.clear()  # a quantized matmul dequantizes on every call
        t0 = time.perf_counter()
        r = m.attention(0, om.rms_norm(x, m.norm_w(p + "input_layernorm"), c.rms_norm_eps), qc)
        h = om.rb(x + r)
        r = m.mlp(0, om.rms_norm(h, m.norm_w(p + "post_attention_layernorm"), c.rms_norm_eps))
        h = om.rb(h + r)
        times.append(time.perf_counter() - t0)
        qc.k_parts, qc.v_parts, qc.offset = qc.k_parts[:1], qc.v_parts[:1], ctx  # every layer sees ctx keys
    layer_s = sum(times) / len(times)
    rows = 16384
    m._deq.clear()
    t1 = time.perf_counter()
    _ = m.lm_head(m.final_hidden(h))
    head_s = (time.perf_counter() - t1) * cfg["vocab_size"] / rows
    tok_s = cfg["num_hidden_layers"] * layer_s + head_s
    return {"value": round(1.0 / tok_s, 6), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} decoder-layer call(s) of the {cfg['num_hidden_layers']}-layer model at context "
                      f"{ctx} ({kv_bits}-bit KV), weights and KV dequantized on every call, timed and scaled by the "
                      f"layer count; lm_head timed on {rows} of {cfg['vocab_size']} rows and scaled to all rows"}


# ----------------------------------------------------------------- GPU leg
def gemv_roofline(model, cfg, peak_gbs, peak_src="measured", proj="mlp.up_proj") -> dict:
    """Dominant kernel: the decode dequant-GEMV, timed alone with CUDA events on
    one projection of every layer (dense: up_proj; MoE: q_proj)."""
    import torch

    from myinfer_b200 import ops
    H = cfg["hidden_size"]
    L = cfg["num_hidden_layers"]
    x = torch.randn(1, H, device=model.device).to(torch.bfloat16)
    names = [f"model.layers.{i}.{proj}" for i in range(L)]
    w = model.weights
    for _ in range(2):
        for n in names[:4]:
            ops.quantized_matmul(x, w[n + ".weight"], w[n + ".scales"], w[n + ".biases"])
    torch.cuda.synchronize()
    # all layers' projections back to back (distinct weights, no L2 reuse),
    # captured in one CUDA graph so host launch overhead is not timed
    s = torch.cuda.Stream(device=model.device)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    N = w[names[0] + ".weight"].shape[0]  # this rank's rows (intermediate_size / tp under tensor parallelism)
    outs = [torch.empty(1, N, dtype=torch.bfloat16, device=model.device) for _ in names]
    with torch.cuda.stream(s):
        graph.capture_begin()
        for n, o in zip(names, outs):
            ops.quantized_matmul(x, w[n + ".weight"], w[n + ".scales"], w[n + ".biases"], out=o)
        graph.capture_end()
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / len(names)
    K = H
    alg = N * K * 0.5625 + K * 2 + N * 2
    ach = alg / (ms * 1e-3) / 1e9
    # `traffic` (DRAM bytes per launch) comes from an ncu capture, which this
    # run does not make: null here, the captured figure is in the profiles
    return {"bound": "hbm", "kernel": f"gemv_tmap_kernel<1,EPI_STORE> ({proj.split('.')[-1]} {N}x{K} w4g64, 1 token)",
            "achieved": round(ach, 1), "peak": peak_gbs, "peak_source": peak_src,
            "unit": "GB/s", "frac": round(ach / peak_gbs, 4), "traffic": None,
            "alg_bytes_per_launch": int(alg), "avg_launch_us": round(ms * 1e3, 2)}


def prefill(model, cache, ids, chunk: int):
    """Chunked prefill of `ids` (device int32) into `cache`, like generate_step's prompt loop."""
    for pos in range(0, ids.numel(), chunk):
        model.forward(ids[pos:pos + chunk], cache)
    return cache


class BatchDecodeGraph:
    """One captured batched decode step: tokens [B] in, greedy tokens into the
    same buffer (logits [B, V] kept on the device)."""

    def __init__(self, model, cache):
        import torch
        self.model, self.cache = model, cache
        B = cache.batch
        dev = model.device
        self.tok = torch.ones(B, dtype=torch.int32, device=dev)
        self.logits = torch.empty(B, model.args.vocab_size, dtype=torch.bfloat16, device=dev)
        cache.d_len.fill_(cache.offset)
        model.forward_batch(self.tok, cache, logits=self.logits, argmax_out=self.tok, sync_len=False)  # eager warm
        torch.cuda.synchronize()
        offsets = [c.offset for c in cache]
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self.graph.capture_begin()
            try:
                model.forward_batch(self.tok, cache, logits=self.logits, argmax_out=self.tok, sync_len=False)
            finally:
                self.graph.capture_end()
        torch.cuda.current_stream(dev).wait_stream(s)
        for c, o in zip(cache, offsets):  # capture ran nothing
            c.offset = o

    def step(self) -> None:
        self.graph.replay()
        for c in self.cache:
            c.offset += 1


class Ctx:
    """Rank, device and communicator of this process (torchrun env)."""

    def __init__(self):
        import datetime

        import torch
        self.rank = int(os.environ.get("RANK", 0))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.comm = None
        if self.world > 1:
            import torch.distributed as dist

            from myinfer_b200.distributed import Communicator
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
            self.comm = Communicator(self.world, self.rank)

    def barrier(self):
        import torch
        if self.world > 1:
            torch.distributed.barrier()

    def max_over_ranks(self, v: float) -> float:
        import torch
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t)


def build_model(cx: Ctx, cfg: dict, seed: int, chunk: int, sharded: bool = True):
    """This rank's shard of the seeded random model (dense: tensor parallel;
    MoE: expert parallel over all ranks with the attention heads sharded over
    the same ranks), or the whole model on this GPU."""
    import torch

    from myinfer_b200.distributed import shard_weights
    from myinfer_b200.model import Model, ModelArgs, random_weights
    a = ModelArgs.from_dict(cfg)
    world = cx.world if sharded else 1
    par = {}
    if world > 1 and a.num_experts:
        El = a.num_experts // world
        w = random_weights(a, seed=seed, device=cx.dev, experts=(cx.rank * El, El))  # this rank's experts only
        par = dict(ep_size=world, ep_rank=cx.rank, tp_size=world, tp_rank=cx.rank)
        w = shard_weights(w, a, experts_local=True, **par)
        torch.cuda.empty_cache()
    else:
        w = random_weights(a, seed=seed, device=cx.dev)
        if world > 1:
            par = dict(tp_size=world, tp_rank=cx.rank)
            w = shard_weights(w, a, **par)
            torch.cuda.empty_cache()
    model = Model(a, w, cx.dev, max_tokens=chunk, comm=cx.comm if world > 1 else None, **par)
    torch.cuda.synchronize()
    return model


def new_cache(model, cap: int, kv_bits: int, batch: int = 1):
    from myinfer_b200.cache import PromptCache, QuantizedKVCache
    a = model.args
    return PromptCache([QuantizedKVCache(model.n_kv_heads_local, a.head_dim, model.device, 64, kv_bits, capacity=cap,
                                         batch=batch) for _ in range(a.num_hidden_layers)], model.device)


def greedy_tokens(model, ids, n: int, kv_bits: int, chunk: int, feed=None):
    """Eager greedy decode: prefill ids[:-1], then n tokens.  Returns the
    greedy tokens, their top-2 margins and the per-step logits (host fp32);
    with `feed` (teacher forcing) step i + 1 is fed feed[i] instead."""
    import torch

    from myinfer_b200 import _lib
    cache = new_cache(model, ids.numel() + n + 8, kv_bits)
    prefill(model, cache, ids[:-1], chunk)
    tok = ids[-1:].clone()
    out, margins, logits = [], [], []
    lg = torch.empty(model.args.vocab_size, dtype=torch.bfloat16, device=model.device)
    for i in range(n):
        model.forward(tok, cache, _lib.M5_LOGITS_LAST, lg, tok)
        top = lg.float().topk(2).values
        margins.append(float(top[0] - top[1]))
        logits.append(lg.float().cpu())
        out.append(int(tok.item()))
        if feed is not None:
            tok.fill_(int(feed[i]))
    return out, margins, torch.stack(logits)


N1_COS_FLOOR = 0.995  # teacher-forced logits cosine, N GPUs vs one (see n1_token_check)


def n1_token_check(cx: Ctx, model, cfg: dict, seed: int, kv_bits: int, chunk: int, n: int = 16) -> dict:
    """The N-GPU model against the same seeded model on one GPU (rank 0), at a
    64-token prompt: the 1-GPU greedy tokens, the N-GPU greedy tokens (how
    long they agree), and the N-GPU logits teacher-forced on the 1-GPU tokens
    (per-step cosine and max-abs).  The ranks add their fp32 partial sums in
    another order than one GPU, so over dozens of layers the logits drift by
    bf16 rounding and a close top two may swap.  How far such a change moves
    this random-weight model was measured on one GPU: the 64-layer 32B shape
    run with the GEMV's fp16 consumer instead of its int8 one (both valid,
    both within one bf16 step per projection) gives a teacher-forced logits
    cosine of 0.9975 (max-abs 0.48) against the default, and the same run
    twice gives identical logits.  `pass` asks for a cosine >= 0.995 at every
    step; a missing or doubled rank partial in any layer falls far below it."""
    import torch
    g = torch.Generator(device=cx.dev).manual_seed(seed + 11)
    ids = torch.randint(0, cfg["vocab_size"], (64,), generator=g, device=cx.dev, dtype=torch.int32)
    ref_t = torch.zeros(n, dtype=torch.int32, device=cx.dev)
    ref = margins = ref_logits = None
    if cx.rank == 0:
        full = build_model(cx, cfg, seed, chunk, sharded=False)
        ref, margins, ref_logits = greedy_tokens(full, ids, n, kv_bits, chunk)
        del full
        torch.cuda.empty_cache()
        ref_t.copy_(torch.tensor(ref, dtype=torch.int32))
    if cx.world > 1:
        torch.distributed.broadcast(ref_t, src=0)
    # every rank takes the same collective steps: a free run, then a forced one
    got, _, _ = greedy_tokens(model, ids, n, kv_bits, chunk)
    _, _, forced = greedy_tokens(model, ids, n, kv_bits, chunk, feed=ref_t.tolist())
    res = None
    if cx.rank == 0:
        cos = torch.nn.functional.cosine_similarity(forced, ref_logits, dim=-1)
        k = next((i for i, (x, y) in enumerate(zip(got, ref)) if x != y), n)
        res = {"tokens": n, "equal_prefix": k, "match": k == n,
               "first_diff_margin": None if k == n else round(margins[k], 4),
               "forced_logits_cos_min": round(cos.min().item(), 6),
               "forced_logits_max_abs": round((forced - ref_logits).abs().max().item(), 4),
               "pass": cos.min().item() >= N1_COS_FLOOR}
    cx.barrier()
    return res


def decode_bench(cx: Ctx, model, cfg: dict, ctx: int, kv_bits: int, batch: int, steps: int, warmup: int,
                 chunk: int, seed: int, clocks: bool = False, e2e: bool = False) -> dict:
    """Timed prefill of a `ctx`-token prompt, then `steps` graph-replayed
    decode steps after `warmup` untimed ones (device time, max over ranks)."""
    import torch

    from myinfer_b200 import _lib
    from myinfer_b200.generate import DecodeGraph
    B = batch
    g = torch.Generator(device=cx.dev).manual_seed(seed + 7)
    ids = torch.randint(0, cfg["vocab_size"], (ctx,), generator=g, device=cx.dev, dtype=torch.int32)
    prefill(model, new_cache(model, chunk, kv_bits), ids[:chunk], chunk)  # warm the prefill kernels
    cache = new_cache(model, ctx + warmup + steps * 2 + 8, kv_bits, B)
    torch.cuda.synchronize()
    cx.barrier()
    ps, pe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ps.record()
    if B == 1:
        prefill(model, cache, ids, chunk)
    else:  # the timed prompt fills sequence 0; the other sequences get copies of its KV
        model.prefill_sequence(ids, cache, 0, chunk)
    pe.record()
    torch.cuda.synchronize()
    prefill_ms = cx.max_over_ranks(ps.elapsed_time(pe))
    if B > 1:
        for c in cache:
            for t in c._tensors():
                t[1:].copy_(t[:1].expand_as(t[1:]))
            c.offset = ctx
    if B == 1:
        tok = torch.tensor([1], dtype=torch.int32, device=cx.dev)
        model.forward(tok, cache, _lib.M5_LOGITS_NONE, None, tok)
        graph = DecodeGraph(model, cache, with_logits=False)
        graph.tok.copy_(tok)
    else:
        graph = BatchDecodeGraph(model, cache)
    for _ in range(warmup):
        graph.step()
    torch.cuda.synchronize()
    cx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(cx.local) if clocks else None
    if clk:
        clk.__enter__()
    start.record()
    for _ in range(steps):
        graph.step()
    end.record()
    torch.cuda.synchronize()
    if clk:
        clk.__exit__()
    ms_step = cx.max_over_ranks(start.elapsed_time(end)) / steps
    out = {"ms_step": ms_step, "prefill_ms": prefill_ms, "mean_ctx": ctx + 1 + warmup + steps / 2,
           "clocks": clk.summary() if clk else None}
    if e2e:  # the public decode step with pinned host tokens in and out, every step
        host = torch.ones(B, dtype=torch.int32, pin_memory=True)
        torch.cuda.synchronize()
        cx.barrier()
        e_steps = max(4, steps // 2)
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        for _ in range(e_steps):
            graph.tok.copy_(host, non_blocking=True)
            graph.step()
            host.copy_(graph.tok, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        ee.record()
        torch.cuda.synchronize()
        out["e2e_ms"] = cx.max_over_ranks(es.elapsed_time(ee)) / e_steps
    del graph, cache
    torch.cuda.empty_cache()
    return out


def moe_block(cx: Ctx, name: str, args, steps: int) -> dict:
    """Batch-1 decode of a MoE config at its BASELINE prompt and KV bits,
    expert parallel over all ranks with the attention heads, their KV and the
    lm_head rows sharded over the same ranks (router replicated; each rank
    streams its own routed experts)."""
    import torch
    cfg = CONFIGS[name]
    ctx, kv_bits = DEFAULTS[name]
    t0 = time.perf_counter()
    model = build_model(cx, cfg, args.seed, args.chunk)
    load_s = time.perf_counter() - t0
    r = decode_bench(cx, model, cfg, ctx, kv_bits, 1, steps, 3, args.chunk, args.seed)
    check = n1_token_check(cx, model, cfg, args.seed, kv_bits, args.chunk) \
        if cx.world > 1 and name != "qwen3-235b-a22b" else None
    del model
    torch.cuda.empty_cache()
    per_rank = moe_bytes_per_rank(cfg, cx.world, int(r["mean_ctx"]), kv_bits)
    peaks = measured_peaks()
    return {"model": name, "parallelism": f"ep{cx.world}+tp{cx.world}-attention" if cx.world > 1 else "single", "prompt_tokens": ctx,
            "kv_bits": kv_bits, "value": round(1000.0 / r["ms_step"], 2), "unit": "tok/s",
            "ms_per_step": round(r["ms_step"], 4), "steps": steps,
            "prefill_tok_s": round(ctx / (r["prefill_ms"] * 1e-3), 1),
            "bytes_per_token_per_rank": int(per_rank),
            "hbm_frac_of_measured": round(per_rank / (r["ms_step"] * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
            "tokens_match_n1": check, "load_seconds": round(load_s, 1)}


def run_gpu(args) -> dict:
    import torch
    cx = Ctx()
    cfg = CONFIGS[args.config]
    t0 = time.perf_counter()
    model = build_model(cx, cfg, args.seed, args.chunk)
    load_s = time.perf_counter() - t0
    a = model.args
    B, ctx, world = args.batch, args.ctx, cx.world
    r = decode_bench(cx, model, cfg, ctx, args.kv_bits, B, args.steps, args.warmup, args.chunk, args.seed,
                     clocks=True, e2e=True)
    ms_step = r["ms_step"]
    # bytes one step streams: the weights once, the KV of every sequence
    bytes_step = weight_bytes_per_token(cfg) + B * kv_bytes_per_token(cfg, int(r["mean_ctx"]), args.kv_bits)
    peaks = measured_peaks()
    tok_s = B * 1000.0 / ms_step  # every rank works on the same B tokens
    roof = gemv_roofline(model, cfg, peaks["hbm_gbs"], peaks["source"],
                         "mlp.up_proj" if not a.num_experts else "self_attn.q_proj")
    check = n1_token_check(cx, model, cfg, args.seed, args.kv_bits, args.chunk) if world > 1 else None
    per_rank = bytes_step / world
    par_name = f"tp{world}" if world > 1 and not a.num_experts else (f"ep{world}+tp{world}-attention" if world > 1 else "single")
    prefill_flops = 2.0 * ctx * (weight_bytes_per_token(cfg) / 0.5625) + 4.0 * a.num_hidden_layers * \
        a.num_attention_heads * a.head_dim * ctx * ctx / 2
    prefill_ms = r["prefill_ms"]
    out = {
        "metric": f"batch-{B} decode tok/s ({NAMES[args.config]}-shaped, w4g64, {args.kv_bits}-bit KV) + HBM TB/s "
                  "vs peak; prefill tok/s",
        "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": f"w4a16 (bf16 activations, fp32 accumulate), {args.kv_bits}-bit KV",
        "data": "synthetic (seeded random weights and prompt ids)",
        "config": {"workload": f"{args.config} batch-{B} decode after a {ctx}-token prefill"
                               + (" (one prompt prefilled, its KV copied to every sequence)" if B > 1 else ""),
                   "model": args.config, "global_batch": B, "seq_len": ctx, "parallelism": par_name,
                   "prefill_chunk": args.chunk, "kv_bits": args.kv_bits,
                   "l2": f"inputs larger than L2 ({bytes_step / 1e9:.1f} GB streamed per decode step)"},
        "hbm": {"bytes_per_step": bytes_step, "bytes_per_token": round(bytes_step / B),
                "achieved_gbs": round(bytes_step / (ms_step * 1e-3) / 1e9, 1),
                "achieved_gbs_per_gpu": round(per_rank / (ms_step * 1e-3) / 1e9, 1), "peak_gbs": peaks["hbm_gbs"],
                "frac_of_measured": round(per_rank / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                "frac_of_8tbs_nominal": round(per_rank / (ms_step * 1e-3) / 8e12, 4)},
        "prefill": {"value": round(ctx / (prefill_ms * 1e-3), 1), "unit": "tok/s", "prompt_tokens": ctx,
                    "ms": round(prefill_ms, 1), "flops": prefill_flops,
                    "tflops": round(prefill_flops / (prefill_ms * 1e-3) / 1e12, 1)},
        "roofline": roof,
        "e2e": {"value": round(B * 1000.0 / r["e2e_ms"], 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": None,
        "clocks": r["clocks"],
        "tokens_match_n1": check,
        "load_seconds": round(load_s, 1),
    }
    # kernels per decode step: per layer q|k|v (QK-norm, RoPE and KV append in its
    # epilogue), attention, combine, o, gate/up, down (+ 2 peer all-reduces under
    # tensor parallelism); embed, lm_head, argmax, length update.
    # MoE: q|k|v, attention, combine, o, router + top-k, expert gate/up, expert down
    # (+ the o_proj and expert all-reduces when sharded)
    per_layer = (7 + (2 if world > 1 else 0)) if a.num_experts else (6 + (2 if world > 1 else 0))
    out["gpu_launches"] = args.steps * (a.num_hidden_layers * per_layer + 4)
    del model
    torch.cuda.empty_cache()
    if not args.no_moe and args.config == "qwen3-32b" and B == 1:
        out["moe"] = [moe_block(cx, "qwen3-30b-a3b", args, min(args.steps, 32))]
        if world >= 4:  # 132 GB of weights: 33 GB per rank at EP4
            out["moe"].append(moe_block(cx, "qwen3-235b-a22b", args, min(args.steps, 16)))
    if world == 1 and not args.no_attention:
        out["attention_op"] = attention_block()
    if cx.rank == 0 and not args.no_cpu:
        out["cpu_baseline"] = cpu_decode_sample(cfg, ctx, args.kv_bits, threads=os.cpu_count() or 1, budget_s=15.0)
    if world > 1:
        cx.barrier()
        cx.comm.close()
        torch.distributed.destroy_process_group()
    return out if cx.rank == 0 else None


def run_reference(args) -> dict:
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return None
    cfg = CONFIGS[args.config]
    vals = []
    base = None
    for _ in range(max(1, args.steps // 10) if args.steps else 1):
        base = cpu_decode_sample(cfg, args.ctx, args.kv_bits, threads=os.cpu_count() or 1, budget_s=10.0)
        vals.append(base["value"])
    v = statistics.mean(vals)
    return {"impl": "reference",
            "metric": f"batch-1 decode tok/s ({NAMES[args.config]}-shaped, w4g64, {args.kv_bits}-bit KV) + HBM TB/s "
                      "vs peak; prefill tok/s",
            "value": round(v, 6), "unit": "tok/s", "n_gpus": int(os.environ.get("WORLD_SIZE", 1)),
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (CPU oracle)",
            "data": "synthetic (seeded random weights and KV)",
            "config": {"workload": f"{args.config} batch-1 decode after a {args.ctx}-token prefill",
                       "model": args.config, "global_batch": 1, "seq_len": args.ctx, "kv_bits": args.kv_bits},
            "cpu_baseline": dict(base, value=round(v, 6)),
            "e2e": {"value": round(v, 6), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "MLX/mlx-lm (the reference's own CPU path) is not installable here; the CPU restatement "
                    "in oracle/ stands in for it, sampled at the stated context (see cpu_baseline.sample)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="m5", choices=["m5", "reference"])
    ap.add_argument("--config", default="qwen3-32b", choices=sorted(CONFIGS))
    ap.add_argument("--ctx", type=int, default=None, help="prompt tokens (default: the config's)")
    ap.add_argument("--kv-bits", type=int, default=None, choices=[4, 8], help="KV cache bits (default: the config's)")
    ap.add_argument("--batch", type=int, default=1, help="sequences decoded together (m5_forward_batch when > 1)")
    ap.add_argument("--chunk", type=int, default=2048, help="prefill chunk (prefill_step_size)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-moe", action="store_true", help="skip the expert-parallel MoE block")
    ap.add_argument("--no-attention", action="store_true", help="skip the attention-op block (1 GPU)")
    args = ap.parse_args()
    if args.ctx is None:
        args.ctx = DEFAULTS[args.config][0]
    if args.kv_bits is None:
        args.kv_bits = DEFAULTS[args.config][1]
    if args.warmup < 3:
        args.warmup = 3
    out = run_reference(args) if args.impl == "reference" else run_gpu(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
