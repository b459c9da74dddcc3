"""The token loop: chunked prefill + greedy decode on the device.

Replaces mlx-lm ``stream_generate`` / ``generate_step`` as the reference calls
them at m5engine/engine.py:396-423: the prompt minus its last token runs in
chunks of ``prefill_step_size``; after every model call the cache is
quantized once ``offset >= quantized_kv_start`` (m5engine/attention.py:106-112);
the last prompt token produces the first sampled token; then every decode step
feeds the previous token.  Like ``generate_step`` the next step is computed
before the current token is yielded, so the cache ends holding prompt +
max_tokens positions.

Decode steps run as one replayed CUDA graph per cache layout: the graph
reads the previous token and the cache length from device memory and writes
the next token back (the argmax, or the device sampler's draw, which also
applies the logits processors and rolls their token window on the device), so
the host only copies 4 bytes per token out.

Every kernel wait is bounded: a wait that runs out (a copy that never landed,
a peer rank that never arrived) records a device error word instead of
hanging.  The loop reads those words after the prompt, every
``STATUS_EVERY`` decode steps and at the end, and raises ``M5CudaError``
(M5_ERR_TIMEOUT) so a failed step never passes silently as tokens.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Iterator, List, Optional

import torch

from . import _lib
from .attention import safe_maybe_quantize_kv_cache
from .cache import PromptCache, make_prompt_cache, trim_prompt_cache
from .sample import DeviceSampler, with_processors

STATUS_EVERY = 64  # decode steps between reads of the device error words


@dataclass
class GenerationResponse:
    """Fields the reference reads from mlx-lm responses (m5engine/engine.py:424-432)."""
    text: str
    token: int
    logprobs: Optional[torch.Tensor]
    from_draft: bool
    prompt_tokens: int
    prompt_tps: float
    generation_tokens: int
    generation_tps: float
    peak_memory: float
    finish_reason: Optional[str] = None


class DecodeGraph:
    """One captured L=1 forward: token buffer in, next token (argmax, or the
    device sampler's draw with its penalty window rolled) into the same buffer."""

    def __init__(self, model, cache: PromptCache, with_logits: bool, sampler: Optional[DeviceSampler] = None,
                 history: Optional[torch.Tensor] = None):
        self.model, self.cache = model, cache
        dev = model.device
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        with_logits = with_logits or sampler is not None
        self.logits = torch.empty(model.args.vocab_size, dtype=torch.bfloat16, device=dev) if with_logits else None
        if sampler is not None:
            sampler.state(dev)  # the draw counter must exist before the capture
        self.sig = cache.signature()
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        offsets = [c.offset for c in cache]
        with torch.cuda.stream(s):
            self.graph.capture_begin()
            try:
                model.forward(self.tok, cache, _lib.M5_LOGITS_LAST if with_logits else _lib.M5_LOGITS_NONE,
                              self.logits, None if sampler is not None else self.tok, sync_len=False)
                if sampler is not None:
                    sampler(self.logits, history=history, out=self.tok, append=history is not None)
            finally:
                self.graph.capture_end()
        torch.cuda.current_stream(dev).wait_stream(s)
        for c, o in zip(cache, offsets):  # capture did not run anything
            c.offset = o

    def valid_for(self, cache: PromptCache) -> bool:
        return cache is self.cache and cache.signature() == self.sig

    def step(self) -> None:
        self.graph.replay()
        for c in self.cache:
            c.offset += 1


def _step_eager(model, cache: PromptCache, tokens: torch.Tensor, want_logits: bool):
    out_tok = torch.empty(1, dtype=torch.int32, device=model.device)
    logits = torch.empty(model.args.vocab_size, dtype=torch.bfloat16, device=model.device) if want_logits else None
    model.forward(tokens, cache, _lib.M5_LOGITS_LAST if want_logits else _lib.M5_LOGITS_NONE, logits, out_tok)
    return out_tok, logits


def generate_step(prompt: List[int], model, max_tokens: int = 256, sampler: Optional[Callable] = None,
                  logits_processors: Optional[list] = None,
                  prompt_cache: Optional[PromptCache] = None, prefill_step_size: int = 2048,
                  kv_bits: Optional[int] = None, kv_group_size: int = 64, quantized_kv_start: int = 0,
                  use_graph: bool = True, return_logits: bool = False,
                  stats: Optional[dict] = None, feed: Optional[List[int]] = None) -> Iterator[tuple]:
    """Yields (token, logits-or-None) pairs; ``sampler`` None means greedy on the
    device, a ``DeviceSampler`` (``sample.make_sampler``) samples on the device
    inside the decode graph, any other callable gets fp32 logits [1, V] eagerly.
    ``logits_processors`` (``sample.make_logits_processors``) fold into the
    device sampler.  Yielded logits are the processed ones.

    ``feed`` (testing, greedy) replaces the token fed at decode step i with
    feed[i] while the yielded tokens stay the device's own choice."""
    if not prompt:
        raise ValueError("empty prompt")
    V = model.args.vocab_size
    if min(prompt) < 0 or max(prompt) >= V:
        raise ValueError(f"token id out of range [0, {V})")
    dev = model.device
    cache = prompt_cache if prompt_cache is not None else make_prompt_cache(model)
    total = cache.offset + len(prompt) + max_tokens
    prompt_t = torch.as_tensor(prompt, dtype=torch.int32).to(dev, non_blocking=True)
    model.reserve(min(prefill_step_size, max(1, len(prompt) - 1)))

    def maybe_quantize():
        safe_maybe_quantize_kv_cache(cache, quantized_kv_start, kv_group_size, kv_bits)
        for c in cache:  # pre-size so decode never reallocates under a captured graph
            if c.capacity < total:
                c.reserve(total)

    t0 = time.perf_counter()
    pos = 0
    n = len(prompt)
    while n - pos > 1:
        m = min(prefill_step_size, n - pos - 1)
        model.forward(prompt_t[pos:pos + m], cache)
        maybe_quantize()
        pos += m
    sampler = with_processors(sampler, logits_processors)
    greedy = sampler is None
    dev_sampler = isinstance(sampler, DeviceSampler)
    # penalty window: the tokens that pass through the sampling step (mlx-lm generate_step)
    hist = sampler.history(prompt[-1:], dev) if dev_sampler else None
    tok, logits = _step_eager(model, cache, prompt_t[pos:], return_logits or not greedy)
    maybe_quantize()
    if dev_sampler:
        tok = sampler(logits, history=hist, out=tok, append=hist is not None)
    elif not greedy:
        tok = sampler(logits.float()[None]).to(torch.int32).reshape(1)
    host = torch.empty(2, dtype=torch.int32, pin_memory=True)
    host[0:1].copy_(tok, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record()
    ev.synchronize()
    if stats is not None:
        stats["prompt_time"] = time.perf_counter() - t0
        stats["prompt_tokens"] = n
    _lib.device_check()
    y = int(host[0])
    y_logits = logits
    graph: Optional[DecodeGraph] = None
    feed_t = None if feed is None else torch.as_tensor(feed, dtype=torch.int32).to(dev)
    t1 = time.perf_counter()
    for i in range(max_tokens):
        # compute the next step before yielding y (mlx-lm generate_step order)
        if feed_t is not None:
            tok = feed_t[i:i + 1]
            y_in = int(feed[i])
        else:
            y_in = y
        if (greedy or dev_sampler) and use_graph:
            if graph is None or not graph.valid_for(cache):
                graph = DecodeGraph(model, cache, return_logits, sampler if dev_sampler else None, hist)
            if tok is not graph.tok:
                graph.tok.copy_(tok)
            graph.step()
            tok = graph.tok
            nxt_logits = graph.logits.clone() if return_logits else None
        else:
            tok_in = torch.tensor([y_in], dtype=torch.int32, device=dev)
            tok, nxt_logits = _step_eager(model, cache, tok_in, return_logits or not greedy)
            if dev_sampler:
                tok = sampler(nxt_logits, history=hist, out=tok, append=hist is not None)
            elif not greedy:
                tok = sampler(nxt_logits.float()[None]).to(torch.int32).reshape(1)
            maybe_quantize()
        slot = (i + 1) & 1
        host[slot:slot + 1].copy_(tok, non_blocking=True)
        ev.record()
        yield y, y_logits
        ev.synchronize()
        if (i + 1) % STATUS_EVERY == 0:
            _lib.device_check()
        y, y_logits = int(host[slot]), nxt_logits
    _lib.device_check()
    if stats is not None:
        stats["decode_time"] = time.perf_counter() - t1


def penalty_windows(prefix: torch.Tensor, fed: torch.Tensor) -> torch.Tensor:
    """[L, W] int32 penalty windows for L logits rows that follow the tokens
    ``fed`` [L]: row i holds the last W of ``prefix`` [W] (the window before
    fed[0], -1 where empty) + fed[:i + 1]."""
    W = prefix.numel()
    seq = torch.cat([prefix.to(torch.int32), fed.to(torch.int32)])
    return seq.unfold(0, W, 1)[1:1 + fed.numel()].contiguous()


def speculative_generate_step(prompt: List[int], model, draft_model, num_draft_tokens: int = 2,
                              max_tokens: int = 256, sampler: Optional[Callable] = None,
                              logits_processors: Optional[list] = None,
                              prompt_cache: Optional[PromptCache] = None, draft_cache: Optional[PromptCache] = None,
                              prefill_step_size: int = 2048, kv_bits: Optional[int] = None,
                              kv_group_size: int = 64, quantized_kv_start: int = 0,
                              stats: Optional[dict] = None) -> Iterator[tuple]:
    """Speculative decoding with a draft model (the algorithm of mlx-lm's
    ``speculative_generate_step``, which the reference reaches through
    ``stream_generate(..., draft_model=...)`` at m5engine/engine.py:420-423):
    each round the draft model proposes up to ``num_draft_tokens`` tokens one at
    a time, the main model scores the pending token plus all proposals in one
    call, the longest prefix of proposals equal to the main model's own choices
    is accepted, and the main model's choice after it is emitted too.  Yields
    (token, from_draft).  Both caches are trimmed back to the accepted context
    (move-not-copy); when every proposal was accepted, the last one is fed to the
    draft model at the start of the next round.  With a greedy sampler the
    tokens equal the main model's greedy decode."""
    if not prompt:
        raise ValueError("empty prompt")
    if draft_model.args.vocab_size != model.args.vocab_size:
        raise ValueError("draft model vocabulary differs from the main model's")
    dev = model.device
    mcache = prompt_cache if prompt_cache is not None else make_prompt_cache(model)
    dcache = draft_cache if draft_cache is not None else make_prompt_cache(draft_model)
    prompt_t = torch.as_tensor(prompt, dtype=torch.int32).to(dev, non_blocking=True)
    sampler = with_processors(sampler, logits_processors)
    greedy = sampler is None
    dev_sampler = isinstance(sampler, DeviceSampler)
    k_max = max(1, num_draft_tokens)
    total = max(mcache.offset, dcache.offset) + len(prompt) + max_tokens + k_max + 1
    model.reserve(max(k_max + 1, min(prefill_step_size, max(1, len(prompt) - 1))))
    draft_model.reserve(min(prefill_step_size, max(1, len(prompt) - 1)))

    def maybe_quantize(cache):
        safe_maybe_quantize_kv_cache(cache, quantized_kv_start, kv_group_size, kv_bits)
        for c in cache:
            if c.capacity < total:
                c.reserve(total)

    def prefill(m, cache, ids):
        for p0 in range(0, ids.numel(), prefill_step_size):
            m.forward(ids[p0:p0 + prefill_step_size], cache)
            maybe_quantize(cache)

    ctx: List[int] = []  # sampled-through tokens before the pending one (the penalty window)

    def windows(fed: torch.Tensor) -> Optional[torch.Tensor]:
        """Penalty window of each row whose logits follow the tokens ``fed``."""
        if not dev_sampler or sampler.window == 0:
            return None
        return penalty_windows(sampler.history(ctx, dev)[0], fed)

    def pick(logits, fed):  # logits [L, V] after the last L tokens of ``fed`` -> int32 [L] on the device
        if greedy:
            return logits.float().argmax(dim=-1).to(torch.int32)
        if dev_sampler:
            w = windows(fed)
            return sampler(logits, history=None if w is None else w[-logits.shape[0]:].contiguous())
        return sampler(logits.float()).to(torch.int32).reshape(-1)

    t0 = time.perf_counter()
    prefill(model, mcache, prompt_t[:-1])
    prefill(draft_model, dcache, prompt_t[:-1])
    if stats is not None:
        stats["prompt_time"] = time.perf_counter() - t0
        stats["prompt_tokens"] = len(prompt)
    V = model.args.vocab_size
    y = prompt_t[-1:].clone()          # pending token: in neither cache yet
    y_host = int(prompt[-1])
    backlog = None                     # draft token the draft cache still lacks
    ntoks = 0
    t1 = time.perf_counter()
    while ntoks < max_tokens:
        nd = min(max_tokens - ntoks, k_max)
        if backlog is not None:
            draft_model.forward(backlog, dcache)
            maybe_quantize(dcache)
            backlog = None
        drafts = []
        t = y
        for _ in range(nd):
            lg = torch.empty(1, V, dtype=torch.bfloat16, device=dev)
            draft_model.forward(t, dcache, _lib.M5_LOGITS_LAST, lg)
            maybe_quantize(dcache)
            t = pick(lg, torch.cat([y] + drafts))
            drafts.append(t)
        d = torch.cat(drafts)
        vlog = torch.empty(nd + 1, V, dtype=torch.bfloat16, device=dev)
        model.forward(torch.cat([y, d]), mcache, _lib.M5_LOGITS_ALL, vlog)
        maybe_quantize(mcache)
        v = pick(vlog, torch.cat([y, d]))
        dh, vh = d.tolist(), v.tolist()  # one host sync per round
        n = 0
        while n < nd and vh[n] == dh[n]:
            n += 1
        for i in range(n):
            ntoks += 1
            yield dh[i], True
            if ntoks == max_tokens:
                break
        if ntoks == max_tokens:
            break
        ntoks += 1
        yield vh[n], False
        # keep y + the n accepted proposals in both caches
        trim_prompt_cache(mcache, nd - n)
        if n < nd:
            trim_prompt_cache(dcache, nd - n - 1)
        else:
            backlog = d[nd - 1:nd]
        ctx.extend([y_host] + dh[:n])
        y = v[n:n + 1].clone()
        y_host = vh[n]
    if stats is not None:
        stats["decode_time"] = time.perf_counter() - t1


def stream_generate(model, tokenizer, prompt, max_tokens: int = 256, draft_model=None,
                    **kwargs) -> Iterator[GenerationResponse]:
    """mlx-lm ``stream_generate`` surface used by the engine (greedy or sampler;
    speculative decoding when ``draft_model`` is given: ``num_draft_tokens`` and
    ``draft_cache`` are then read from the keyword arguments)."""
    if isinstance(prompt, str):
        prompt = tokenizer.encode(prompt)
    prompt = [int(t) for t in (prompt.tolist() if hasattr(prompt, "tolist") else prompt)]
    eos = set(getattr(tokenizer, "eos_token_ids", []) or [])
    stats: dict = {}
    t_start = time.perf_counter()
    n = 0
    if draft_model is not None:
        kwargs.pop("use_graph", None)
        steps = speculative_generate_step(prompt, model, draft_model, max_tokens=max_tokens, stats=stats, **kwargs)
    else:
        kwargs.pop("num_draft_tokens", None)
        kwargs.pop("draft_cache", None)
        steps = ((t, False) for t, _ in generate_step(prompt, model, max_tokens, stats=stats, **kwargs))
    for token, from_draft in steps:
        n += 1
        prompt_tps = stats.get("prompt_tokens", len(prompt)) / max(stats.get("prompt_time", 1e-9), 1e-9)
        gen_time = time.perf_counter() - t_start - stats.get("prompt_time", 0.0)
        finish = None
        if token in eos:
            finish = "stop"
        elif n == max_tokens:
            finish = "length"
        yield GenerationResponse(
            text="" if finish == "stop" else tokenizer.decode([token]), token=token, logprobs=None,
            from_draft=from_draft, prompt_tokens=len(prompt), prompt_tps=prompt_tps, generation_tokens=n,
            generation_tps=n / max(gen_time, 1e-9),
            peak_memory=torch.cuda.max_memory_allocated(model.device) / 1e9, finish_reason=finish)
        if finish:
            break
