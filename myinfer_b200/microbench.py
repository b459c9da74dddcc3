"""Kernel microbenchmarks (CUDA-event timed) for the token loop's hot kernels.

    python -m myinfer_b200.microbench gemv --n 25600 --k 5120 [--m 1] [--iters 20]
    python -m myinfer_b200.microbench attention --s 32768 --l 1 --bits 8 [--hq 64 --hkv 8]
    python -m myinfer_b200.microbench gemm --m 2048 --n 8192 --k 5120
    python -m myinfer_b200.microbench step --ctx 32768 --steps 2 [--config qwen3-30b-a3b] [--batch 16]   # decode steps
    python -m myinfer_b200.microbench sample [--rows 1] [--vocab 151936]   # device sampler vs torch ops

``gemv`` cycles over enough distinct weight matrices that every launch reads
from HBM (more than L2 in total); ``attention`` is the standalone
attention.py-op microbench of the BASELINE config (B=1, 64 q / 8 kv heads,
D=128, bf16 Q, N(0,1) K/V quantized 8/4-bit g64).  One JSON line per run.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch


def _timed(fn, iters: int) -> float:
    """Mean device microseconds per call.  The `iters` calls are captured once
    into a CUDA graph and the graph is replayed, so host-side launch overhead
    (Python, ctypes, descriptor setup) is not part of the measurement."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        fn(0)  # warm (lazy module load, attribute setup) outside the capture
        torch.cuda.synchronize()
        g.capture_begin()
        for i in range(iters):
            fn(i)
        g.capture_end()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    g.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / iters


def bench_gemv(n: int, k: int, m: int, iters: int) -> dict:
    from myinfer_b200 import ops
    per = n * k // 2 + n * k // 32
    copies = max(2, (3 << 28) // per + 1)  # > 768 MB of weights in rotation (L2 is 126 MB)
    g = torch.Generator(device="cuda").manual_seed(0)
    mats = []
    for _ in range(copies):
        w = (0.02 * torch.randn(n, k, generator=g, device="cuda")).to(torch.bfloat16)
        mats.append(ops.quantize(w, 64, 4))
        del w
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    for i in range(3):
        ops.quantized_matmul(x, *mats[i % copies])
    torch.cuda.synchronize()
    us = _timed(lambda i: ops.quantized_matmul(x, *mats[i % copies]), iters)
    alg = n * k * 0.5625 + m * k * 2 + m * n * 2
    return {"kernel": "gemv", "n": n, "k": k, "m": m, "us": round(us, 2), "alg_bytes": int(alg),
            "gbs": round(alg / us / 1e3, 1)}


def bench_gemm(m: int, n: int, k: int, iters: int) -> dict:
    """Prefill dequant-GEMM (tensor cores): M tokens x N weight rows x K."""
    from myinfer_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (0.02 * torch.randn(n, k, generator=g, device="cuda")).to(torch.bfloat16)
    mat = ops.quantize(w, 64, 4)
    del w
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ops.quantized_matmul(x, *mat, out=y)
    torch.cuda.synchronize()
    us = _timed(lambda i: ops.quantized_matmul(x, *mat, out=y), iters)
    flops = 2.0 * m * n * k
    return {"kernel": "gemm", "m": m, "n": n, "k": k, "us": round(us, 2), "tflops": round(flops / us / 1e6, 1)}


def bench_step(ctx: int, steps: int, config: str = "qwen3-32b", batch: int = 1) -> dict:
    """Decode steps of a Qwen3-32B- or Qwen3-30B-A3B-shaped model over a synthetic 8-bit KV
    cache of `ctx` positions (`batch` > 1: that many sequences per step through
    m5_forward_batch); only the timed steps run inside a CUDA profiler range
    (cudaProfilerStart/Stop), so `ncu --profile-from-start off` lists exactly
    the kernels of `steps` decode steps."""
    from myinfer_b200 import _lib, ops
    from myinfer_b200.cache import PromptCache, QuantizedKVCache
    from myinfer_b200.model import Model, ModelArgs, random_weights
    presets = {"qwen3-32b": dict(model_type="qwen3", hidden_size=5120, num_hidden_layers=64,
                                 num_attention_heads=64, num_key_value_heads=8, head_dim=128,
                                 intermediate_size=25600, vocab_size=151936, tie_word_embeddings=False),
               "qwen3-30b-a3b": dict(model_type="qwen3_moe", hidden_size=2048, num_hidden_layers=48,
                                     num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                                     intermediate_size=6144, moe_intermediate_size=768, num_experts=128,
                                     num_experts_per_tok=8, norm_topk_prob=True, vocab_size=151936,
                                     tie_word_embeddings=False)}
    a = ModelArgs.from_dict(presets[config])
    dev = torch.device("cuda")
    model = Model(a, random_weights(a, 0, dev), dev, max_tokens=8)
    cache = PromptCache([QuantizedKVCache(a.num_key_value_heads, a.head_dim, dev, 64, 8, capacity=ctx + steps + 8,
                                          batch=batch) for _ in range(a.num_hidden_layers)], dev)
    g = torch.Generator(device=dev).manual_seed(1)
    for c in cache:  # random N(0,1) K/V at positions [0, ctx) of every sequence
        for which in ("k", "v"):
            tq, ts, tb = (c._kq, c._ks, c._kb) if which == "k" else (c._vq, c._vs, c._vb)
            for bi in range(batch):
                x = torch.randn(c.n_kv_heads, ctx, a.head_dim, generator=g, device=dev).to(torch.bfloat16)
                q, sc, b = ops.quantize(x, 64, 8)
                tq[bi, :, :ctx].copy_(q)
                ts[bi, :, :ctx].copy_(sc)
                tb[bi, :, :ctx].copy_(b)
        c.offset = ctx
    tok = torch.ones(batch, dtype=torch.int32, device=dev)
    logits = torch.empty(batch, a.vocab_size, dtype=torch.bfloat16, device=dev) if batch > 1 else None

    def step():
        if batch > 1:
            model.forward_batch(tok, cache, logits=logits, argmax_out=tok)
        else:
            model.forward(tok, cache, _lib.M5_LOGITS_NONE, None, tok)

    for _ in range(2):  # warm: configures every kernel, then rewinds the cache
        step()
        for c in cache:
            c.offset -= 1
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = start.elapsed_time(end) / steps
    return {"kernel": "decode_step", "config": config, "ctx": ctx, "batch": batch, "steps": steps,
            "ms_per_step_eager": round(ms, 3), "tok_s_eager": round(batch * 1e3 / ms, 1)}


def bench_attention(s: int, l: int, bits: int, hq: int, hkv: int, iters: int) -> dict:
    from myinfer_b200 import ops
    from myinfer_b200.attention import blocked_quantized_sdpa
    D = 128
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(1, hq, l, D, generator=g, device="cuda").to(torch.bfloat16)
    reps = max(1, min(8, (1 << 29) // max(1, 2 * hkv * s * D)))
    kvs = []
    for _ in range(reps):
        k = torch.randn(1, hkv, s, D, generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn(1, hkv, s, D, generator=g, device="cuda").to(torch.bfloat16)
        kvs.append((ops.quantize(k, 64, bits), ops.quantize(v, 64, bits)) if bits else (k, v))
        del k, v
    mask = "causal" if l > 1 else None
    for i in range(2):
        blocked_quantized_sdpa(q, *kvs[i % reps], D ** -0.5, mask, 64, bits)
    torch.cuda.synchronize()
    us = _timed(lambda i: blocked_quantized_sdpa(q, *kvs[i % reps], D ** -0.5, mask, 64, bits), iters)
    per_elem = bits / 8 + 4 / 64 if bits else 2
    kv_bytes = 2 * hkv * D * s * per_elem
    alg = kv_bytes + 2 * hq * l * D * 2
    flops = 4 * hq * D * (l * s - (l * (l - 1) // 2 if l > 1 else 0))
    return {"kernel": "attention", "s": s, "l": l, "bits": bits, "hq": hq, "hkv": hkv, "us": round(us, 2),
            "alg_bytes": int(alg), "gbs": round(alg / us / 1e3, 1), "tflops": round(flops / us / 1e6, 2)}


def bench_sample(rows: int, vocab: int, iters: int) -> dict:
    """The device sampler on bf16 logits [rows, vocab], graph replayed, on a
    flat row (N(0, 2): top-p's cut lies in the bulk, so the threshold search
    runs over the whole row) and a peaked one (the same plus 64 tokens lifted
    by 12..20, as a language model's next-token row usually is: the cut lies
    in a narrow band under the max).  Settings: "full" = temperature 0.7,
    top-p 0.9, top-k 50, repetition penalty 1.1 over 20 tokens; "top_p" =
    temperature 0.7, top-p 0.9; "temp" = temperature only; "greedy".  Beside
    them the same filters as a chain of torch ops on the GPU (topk, softmax,
    sort, cumsum, scatter, multinomial), timed eagerly with CUDA events
    because multinomial does not capture."""
    from myinfer_b200.sample import DeviceSampler, make_logits_processors
    g = torch.Generator(device="cuda").manual_seed(0)
    flat = (2 * torch.randn(rows, vocab, generator=g, device="cuda")).to(torch.bfloat16)
    peaked = flat.float()
    idx = torch.randint(0, vocab, (rows, 64), generator=g, device="cuda")
    peaked.scatter_add_(1, idx, 12 + 8 * torch.rand(rows, 64, generator=g, device="cuda"))
    peaked = peaked.to(torch.bfloat16)
    hist = torch.randint(0, vocab, (rows, 20), generator=g, device="cuda", dtype=torch.int32)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    pen = make_logits_processors(repetition_penalty=1.1)
    settings = {"full": (DeviceSampler(0.7, top_p=0.9, top_k=50, processors=pen, seed=1), hist),
                "top_p": (DeviceSampler(0.7, top_p=0.9, seed=1), None),
                "temp": (DeviceSampler(0.7, seed=1), None),
                "greedy": (DeviceSampler(0.0), None)}
    res = {"kernel": "sample", "rows": rows, "vocab": vocab}
    for name, x in (("flat", flat), ("peaked", peaked)):
        for key, (smp, h) in settings.items():
            smp.state("cuda")
            xs = x.clone()
            res[f"{name}_{key}_us"] = round(_timed(lambda i: smp(xs, history=h, out=out), iters), 2)

    def torch_chain(lg):
        z = lg.float() / 0.7
        kth = torch.topk(z, 50, dim=-1).values[..., -1:]
        z = torch.where(z < kth, torch.full_like(z, -float("inf")), z)
        probs = torch.softmax(z, dim=-1)
        sp, si = torch.sort(probs, descending=True, dim=-1)
        keep = torch.cumsum(sp, dim=-1) - sp < 0.9
        probs = torch.zeros_like(probs).scatter(-1, si, sp * keep)
        return torch.multinomial(probs / probs.sum(dim=-1, keepdim=True), 1)

    for _ in range(3):
        torch_chain(flat)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        torch_chain(flat)
    t1.record()
    torch.cuda.synchronize()
    res["torch_ops_us"] = round(t0.elapsed_time(t1) * 1e3 / iters, 2)
    return res


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemv")
    g.add_argument("--n", type=int, default=25600)
    g.add_argument("--k", type=int, default=5120)
    g.add_argument("--m", type=int, default=1)
    g.add_argument("--iters", type=int, default=20)
    st = sub.add_parser("step")
    st.add_argument("--ctx", type=int, default=32768)
    st.add_argument("--steps", type=int, default=2)
    st.add_argument("--config", default="qwen3-32b", choices=["qwen3-32b", "qwen3-30b-a3b"])
    st.add_argument("--batch", type=int, default=1)
    gm = sub.add_parser("gemm")
    gm.add_argument("--m", type=int, default=2048)
    gm.add_argument("--n", type=int, default=8192)
    gm.add_argument("--k", type=int, default=5120)
    gm.add_argument("--iters", type=int, default=20)
    a = sub.add_parser("attention")
    a.add_argument("--s", type=int, default=32768)
    a.add_argument("--l", type=int, default=1)
    a.add_argument("--bits", type=int, default=8)
    a.add_argument("--hq", type=int, default=64)
    a.add_argument("--hkv", type=int, default=8)
    a.add_argument("--iters", type=int, default=20)
    sm = sub.add_parser("sample")
    sm.add_argument("--rows", type=int, default=1)
    sm.add_argument("--vocab", type=int, default=151936)
    sm.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    if args.cmd == "gemv":
        r = bench_gemv(args.n, args.k, args.m, args.iters)
    elif args.cmd == "gemm":
        r = bench_gemm(args.m, args.n, args.k, args.iters)
    elif args.cmd == "sample":
        r = bench_sample(args.rows, args.vocab, args.iters)
    elif args.cmd == "step":
        r = bench_step(args.ctx, args.steps, args.config, args.batch)
    else:
        r = bench_attention(args.s, args.l, args.bits, args.hq, args.hkv, args.iters)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
