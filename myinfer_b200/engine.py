"""Engine: model lifecycle, context planning and generation on the device.

Keeps the host API of m5engine/engine.py (EngineError :47-56, LoadOptions
:59-84, GenerationParams :87-100, Chunk :103-107, RequestMetrics :110-121,
Engine.load :192-205, generate :351-362, _generate :364-461, benchmark
:464-513, info :516-553) and drives the libm5cuda token loop
(``generate.stream_generate``) instead of mlx-lm.  What changes underneath:

* weights live in HBM (MLX safetensors layout or seeded random init), so
  expert streaming (m5engine/expert_stream.py) has no role: MoE experts are
  resident (and sharded over ranks when expert-parallel);
* the memory budget comes from ``cudaMemGetInfo`` instead of macOS sysctl;
* prefix caches are device caches whose trim moves the offset back.
"""

from __future__ import annotations

import gc
import json
import logging
import threading
import time
import warnings
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional

import torch

from . import sample
from .cache import PromptCache, make_prompt_cache
from .context import (GB, MAX_YARN_FACTOR, ContextPlan, KVFootprint, apply_yarn, kv_estimate_per_token,
                      measure_kv_footprint, native_context, plan_context, reserve_bytes, yarn_capable,
                      yarn_factor_for)
from .generate import stream_generate
from .prefix_cache import PrefixCache

log = logging.getLogger("myinfer_b200")


class EngineError(Exception):
    status = 400


class ContextOverflow(EngineError):
    pass


class NotLoaded(EngineError):
    status = 503


@dataclass
class LoadOptions:
    model: str
    kv_bits: int = 8  # 0 = keep KV in bf16
    kv_group_size: int = 64
    quantized_kv_start: int = 4096
    max_context: Optional[int] = None
    rope_scaling: str = "auto"  # auto | off | 2 | 4
    stream_experts: str = "auto"  # kept for API compatibility: experts are HBM-resident here
    expert_cache_gb: Optional[float] = None
    io_threads: int = 8
    prefetch_experts: bool = True
    draft_model: Optional[str] = None
    num_draft_tokens: int = 3
    prefill_step: int = 2048
    memory_budget_gb: Optional[float] = None
    prefix_cache: bool = True
    prefix_cache_entries: int = 4
    trust_remote_code: bool = False
    device: str = "cuda"
    seed: int = 0  # random-init models ("random:<config.json path or preset>")

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "LoadOptions":
        known = {k: v for k, v in d.items() if k in cls.__dataclass_fields__ and v is not None}
        if "model" not in known:
            raise EngineError("'model' is required (local path or random:<preset>)")
        return cls(**known)


@dataclass
class GenerationParams:
    max_tokens: int = 1024
    temperature: float = 0.7
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: Optional[float] = None
    presence_penalty: Optional[float] = None
    frequency_penalty: Optional[float] = None
    stop: List[str] = field(default_factory=list)
    seed: Optional[int] = None
    use_prefix_cache: bool = True
    use_draft: bool = True


@dataclass
class Chunk:
    text: str
    finish_reason: Optional[str] = None
    metrics: Optional["RequestMetrics"] = None


@dataclass
class RequestMetrics:
    prompt_tokens: int = 0
    cached_tokens: int = 0
    completion_tokens: int = 0
    ttft_ms: float = 0.0
    prompt_tps: float = 0.0
    decode_tps: float = 0.0
    draft_accepted: int = 0
    yarn_factor: float = 1.0
    peak_memory_gb: float = 0.0
    finish_reason: str = ""


class ByteTokenizer:
    """Tokenizer for random-init models: UTF-8 bytes offset by 3 (0 pad, 1 bos, 2 eos)."""

    eos_token_ids = [2]
    bos_token_id = 1
    chat_template = None

    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids: List[int]) -> str:
        return bytes([(i - 3) % 256 for i in ids if i >= 3]).decode("utf-8", errors="replace")


PRESETS = {
    "qwen3-0.6b": dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=151936,
                       tie_word_embeddings=True, max_position_embeddings=40960, rms_norm_eps=1e-6,
                       rope_theta=1e6),
    "qwen3-32b": dict(model_type="qwen3", hidden_size=5120, num_hidden_layers=64, num_attention_heads=64,
                      num_key_value_heads=8, head_dim=128, intermediate_size=25600, vocab_size=151936,
                      tie_word_embeddings=False, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      rope_theta=1e6),
    "qwen3-30b-a3b": dict(model_type="qwen3_moe", hidden_size=2048, num_hidden_layers=48,
                          num_attention_heads=32, num_key_value_heads=4, head_dim=128, intermediate_size=6144,
                          moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
                          norm_topk_prob=True, vocab_size=151936, tie_word_embeddings=False,
                          max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6),
    "qwen3-235b-a22b": dict(model_type="qwen3_moe", hidden_size=4096, num_hidden_layers=94,
                            num_attention_heads=64, num_key_value_heads=4, head_dim=128, intermediate_size=12288,
                            moe_intermediate_size=1536, num_experts=128, num_experts_per_tok=8,
                            norm_topk_prob=True, vocab_size=151936, tie_word_embeddings=False,
                            max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6),
}


def _load_model(opts: LoadOptions):
    """(model, tokenizer, config) from a directory or a random:<preset|config.json> spec."""
    from .model import Model, ModelArgs, random_weights
    dev = torch.device(opts.device)
    if opts.model.startswith("random:"):
        spec = opts.model[len("random:"):]
        config = dict(PRESETS[spec]) if spec in PRESETS else json.loads(Path(spec).read_text())
        args = ModelArgs.from_dict(config)
        weights = random_weights(args, opts.seed, dev)
        return Model(args, weights, dev, max_tokens=min(opts.prefill_step, 2048)), ByteTokenizer(args.vocab_size), config
    path = Path(opts.model)
    if not path.is_dir():
        raise EngineError(f"model path {path} not found (no network: pass a local MLX checkpoint directory)")
    config = json.loads((path / "config.json").read_text())
    args = ModelArgs.from_dict(config)
    from .loader import load_mlx_checkpoint
    weights = load_mlx_checkpoint(path, dev, tie_word_embeddings=args.tie_word_embeddings)
    model = Model(args, weights, dev, max_tokens=min(opts.prefill_step, 2048))
    tok_files = [f for f in ("tokenizer.json", "tokenizer_config.json", "tokenizer.model", "vocab.json")
                 if (path / f).exists()]
    if not tok_files:  # weights only: ids in, ids out, text as raw bytes
        warnings.warn(f"{path} has no tokenizer files; using the byte tokenizer")
        return model, ByteTokenizer(args.vocab_size), config
    try:
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(str(path), local_files_only=True,
                                            trust_remote_code=opts.trust_remote_code)
    except Exception as e:  # a checkpoint's own tokenizer that fails to load is an error, not a fallback
        raise EngineError(f"tokenizer in {path} ({', '.join(tok_files)}) failed to load: {e}") from e
    tok.eos_token_ids = [config.get("eos_token_id")] if isinstance(config.get("eos_token_id"), int) \
        else list(config.get("eos_token_id") or [])
    return model, tok, config


class Engine:
    def __init__(self):
        self._lock = threading.RLock()
        self._gen_lock = threading.Lock()
        self.model = None
        self.draft_model = None
        self.tokenizer = None
        self.config: dict = {}
        self.options: Optional[LoadOptions] = None
        self.plan: Optional[ContextPlan] = None
        self.footprint: Optional[KVFootprint] = None
        self.prefix = PrefixCache()
        self.resident_bytes = 0
        self.load_seconds = 0.0
        self.state = "empty"
        self.error: Optional[str] = None
        self.last: RequestMetrics = RequestMetrics()
        self.last_tokens: List[int] = []  # token ids the last request generated
        self.totals = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0, "cached_tokens": 0}
        self._native = 0
        self._plain_limit = 0
        self._yarn_now = 1.0

    # ------------------------------------------------------------------ load
    @property
    def loaded(self) -> bool:
        return self.model is not None

    def budget_bytes(self, opts: Optional[LoadOptions] = None) -> int:
        opts = opts or self.options
        if opts and opts.memory_budget_gb:
            return int(opts.memory_budget_gb * GB)
        free, total = torch.cuda.mem_get_info(torch.device(opts.device if opts else "cuda"))
        return int(total)

    def unload(self) -> None:
        with self._gen_lock, self._lock:
            self._unload()

    def _unload(self) -> None:
        self.model = self.draft_model = self.tokenizer = None
        self.plan = None
        self.footprint = None
        self.prefix.clear()
        self.config = {}
        self.state = "empty"
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    def load(self, opts: LoadOptions) -> dict:
        with self._gen_lock, self._lock:
            self._unload()
            self.state = "loading"
            self.error = None
            try:
                self._load(opts)
            except Exception as e:
                self._unload()
                self.state = "error"
                self.error = str(e)
                raise
            self.state = "ready"
            return self.info()

    def _load(self, opts: LoadOptions) -> None:
        t0 = time.perf_counter()
        if opts.kv_bits not in (0, 4, 8):
            raise EngineError("kv_bits must be 0 (bf16), 4 or 8")
        model, tokenizer, config = _load_model(opts)
        draft, draft_yarn = None, False
        if opts.draft_model:  # engine.py:223-228: a second, smaller model for speculative decoding
            draft, _, dconfig = _load_model(replace(opts, model=opts.draft_model))
            if draft.args.vocab_size != model.args.vocab_size:
                raise EngineError("draft model vocabulary differs from the main model's")
            draft_yarn = yarn_capable(dconfig)
        budget = self.budget_bytes(opts)
        native, plain_limit = native_context(config)
        resident = model.nbytes + (draft.nbytes if draft is not None else 0)
        hidden = int(config.get("hidden_size") or 4096)
        if resident + reserve_bytes(budget, hidden, opts.prefill_step) > budget:
            raise EngineError(f"Model needs {resident / GB:.1f} GB but the GPU budget is {budget / GB:.1f} GB.")
        fp = measure_kv_footprint(model, opts.kv_bits, opts.kv_group_size)
        if opts.kv_bits and opts.quantized_kv_start:
            dense_fp = measure_kv_footprint(model, 0)
            extra = max(0.0, dense_fp.bytes_per_token - fp.bytes_per_token) * opts.quantized_kv_start
            fp = KVFootprint(fp.bytes_per_token, int(fp.fixed_bytes + extra), fp.kv_bits)
        if draft is not None:  # the draft's cache grows with the same tokens (engine.py:276-277)
            dfp = measure_kv_footprint(draft, opts.kv_bits, opts.kv_group_size)
            fp = KVFootprint(fp.bytes_per_token + dfp.bytes_per_token, fp.fixed_bytes + dfp.fixed_bytes, fp.kv_bits)
        plan = plan_context(config=config, footprint=fp, budget_bytes=budget, resident_weight_bytes=resident,
                            expert_cache_bytes=0, prefill_step=opts.prefill_step, rope_scaling=opts.rope_scaling,
                            requested_context=opts.max_context)
        if plan.max_context < 512:
            raise EngineError(f"Only {plan.max_context} tokens of KV cache fit in memory; "
                              "use kv_bits=4 or a smaller model.")
        self.model, self.tokenizer = model, tokenizer
        self.draft_model, self._draft_yarn = draft, draft_yarn
        self.config, self.options = config, opts
        self.plan, self.footprint = plan, fp
        self.resident_bytes = resident
        self.prefix = PrefixCache(max_entries=opts.prefix_cache_entries)
        self._native, self._plain_limit = native, plain_limit
        self._yarn_now = 1.0
        if opts.rope_scaling not in ("auto", "off") and plan.yarn_factor > 1:
            self._set_yarn(plan.yarn_factor)
        self.load_seconds = time.perf_counter() - t0
        self.last = RequestMetrics()
        log.info("Loaded %s in %.1fs: resident %.1f GB, max context %d (%s)", opts.model, self.load_seconds,
                 resident / GB, plan.max_context, plan.limited_by)

    def _set_yarn(self, factor: float) -> None:
        if factor == self._yarn_now:
            return
        apply_yarn(self.model, factor, self._native)
        if self.draft_model is not None and self._draft_yarn:
            apply_yarn(self.draft_model, factor, self._native)
        self._yarn_now = factor

    def _yarn_for_request(self, tokens: int) -> float:
        opts, plan = self.options, self.plan
        if plan.yarn_factor <= 1:
            return 1.0
        if opts.rope_scaling != "auto":
            return plan.yarn_factor
        if tokens <= self._plain_limit:
            return 1.0
        return yarn_factor_for(tokens, self._native, min(plan.yarn_factor, MAX_YARN_FACTOR))

    # ------------------------------------------------------------- generate
    def encode_chat(self, messages: List[dict], chat_template_kwargs: Optional[dict] = None,
                    tools: Optional[list] = None) -> List[int]:
        tok = self.tokenizer
        msgs = []
        for m in messages:
            content = m.get("content")
            if isinstance(content, list):
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            msgs.append({**m, "content": content or ""})
        if getattr(tok, "chat_template", None):
            kwargs = dict(chat_template_kwargs or {})
            if tools:
                kwargs["tools"] = tools
            text = tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True, **kwargs)
            return list(tok.encode(text, add_special_tokens=False))
        text = "\n".join(f"{m['role']}: {m['content']}" for m in msgs) + "\nassistant:"
        return list(tok.encode(text))

    def encode_text(self, prompt: str) -> List[int]:
        return list(self.tokenizer.encode(prompt))

    def generate(self, tokens: List[int], params: GenerationParams) -> Iterator[Chunk]:
        if not self.loaded:
            raise NotLoaded("No model loaded")
        n_prompt = len(tokens)
        if n_prompt >= self.plan.max_context:
            raise ContextOverflow(f"Prompt is {n_prompt} tokens but the maximum context is "
                                  f"{self.plan.max_context} (limited by {self.plan.limited_by}).")
        max_tokens = max(1, min(params.max_tokens, self.plan.max_context - n_prompt))
        return self._generate(tokens, max_tokens, params)

    def _generate(self, tokens: List[int], max_tokens: int, params: GenerationParams) -> Iterator[Chunk]:
        with self._gen_lock:
            if not self.loaded:
                raise NotLoaded("No model loaded")
            opts = self.options
            factor = self._yarn_for_request(len(tokens) + max_tokens)
            self._set_yarn(factor)
            key = f"yarn={factor}"
            use_prefix = opts.prefix_cache and params.use_prefix_cache
            draft = self.draft_model if params.use_draft else None
            # with a draft model the cached context covers both models' layers
            # (engine.py:373-377); a request without it keeps the main layers only
            # and does not return them to the prefix cache (engine.py:393-395, 459)
            if self.draft_model is not None and draft is None:
                use_prefix = False
            cache, hit = (self.prefix.take(key, tokens) if use_prefix else (None, 0))
            if cache is None:
                cache = make_prompt_cache(self.model)
                if draft is not None:
                    cache = PromptCache(list(cache) + list(make_prompt_cache(draft)), self.model.device)
                hit = 0
            n_main = self.model.args.num_hidden_layers
            main_cache = cache if draft is None else PromptCache(list(cache)[:n_main], self.model.device)
            need = self.footprint.bytes_for(len(tokens) + max_tokens)
            self.prefix.evict_to(self.plan.kv_budget_bytes - need)
            if params.seed is not None:
                sample.seed(params.seed)
            sampler = sample.make_sampler(temp=params.temperature, top_p=params.top_p if params.top_p < 1 else 0.0,
                                          min_p=params.min_p, top_k=params.top_k)
            processors = sample.make_logits_processors(repetition_penalty=params.repetition_penalty,
                                                       presence_penalty=params.presence_penalty,
                                                       frequency_penalty=params.frequency_penalty)
            kwargs = dict(sampler=sampler, logits_processors=processors, prompt_cache=main_cache,
                          prefill_step_size=opts.prefill_step,
                          kv_bits=opts.kv_bits or None, kv_group_size=opts.kv_group_size,
                          quantized_kv_start=opts.quantized_kv_start)
            if draft is not None:
                kwargs.update(draft_model=draft, num_draft_tokens=opts.num_draft_tokens,
                              draft_cache=PromptCache(list(cache)[n_main:], self.model.device))
            m = RequestMetrics(prompt_tokens=len(tokens), cached_tokens=hit, yarn_factor=factor)
            torch.cuda.reset_peak_memory_stats(self.model.device)
            generated: List[int] = []
            text = ""
            emitted = 0
            finish = "length"
            t0 = time.perf_counter()
            t_first = None
            stop = [s for s in params.stop if s]
            hold = max((len(s) for s in stop), default=1) - 1
            stopped = False
            eos = set(getattr(self.tokenizer, "eos_token_ids", []) or [])
            try:
                for resp in stream_generate(self.model, self.tokenizer, tokens[hit:], max_tokens, **kwargs):
                    if t_first is None:
                        t_first = time.perf_counter()
                        m.ttft_ms = (t_first - t0) * 1000
                        m.prompt_tps = resp.prompt_tps
                    if not (resp.finish_reason == "stop" and resp.token in eos):
                        generated.append(resp.token)
                    m.draft_accepted += int(resp.from_draft)
                    m.decode_tps = resp.generation_tps
                    text += resp.text
                    if resp.finish_reason:
                        finish = resp.finish_reason
                    safe = len(text)
                    if stop:
                        hits = [i for i in (text.find(s, max(0, emitted - hold)) for s in stop) if i >= 0]
                        if hits:
                            safe, finish, stopped = min(hits), "stop", True
                        else:
                            safe = max(emitted, len(text) - hold)
                    if safe > emitted:
                        yield Chunk(text[emitted:safe])
                        emitted = safe
                    if stopped:
                        break
                if not stopped and emitted < len(text):
                    yield Chunk(text[emitted:])
                    emitted = len(text)
            finally:
                m.completion_tokens = len(generated)
                m.finish_reason = finish
                m.peak_memory_gb = round(torch.cuda.max_memory_allocated(self.model.device) / GB, 2)
                self.last = m
                self.last_tokens = list(generated)
                self.totals["requests"] += 1
                self.totals["prompt_tokens"] += m.prompt_tokens
                self.totals["completion_tokens"] += m.completion_tokens
                self.totals["cached_tokens"] += m.cached_tokens
                if use_prefix:
                    context = tokens + generated
                    if draft is not None:  # the sub-lists may have swapped layers when quantizing
                        cache = PromptCache(list(main_cache) + list(kwargs["draft_cache"]), self.model.device)
                        # The draft cache lags one position after a fully accepted round and the main
                        # cache may hold verified positions past the last yielded token: cut every layer
                        # to the context both models hold, so the entry is reusable.
                        common = min([c.offset for c in cache] + [len(context)])
                        for c in cache:
                            if c.offset > common:
                                c.trim(c.offset - common)
                    self.prefix.put(key, context, cache)
            yield Chunk("", finish, m)

    # ------------------------------------------------------------ benchmark
    def benchmark(self, prompt_tokens: int = 1024, gen_tokens: int = 128, use_draft: bool = True) -> dict:
        """Fresh-cache prefill + greedy decode of a fixed workload."""
        if not self.loaded:
            raise NotLoaded("No model loaded")
        prompt_tokens = max(16, min(int(prompt_tokens), self.plan.max_context - gen_tokens - 64))
        unit = self.encode_text("Decode speed is mostly limited by how many bytes of weights and cache "
                                "must be streamed for every generated token. ")
        tokens = (unit * (prompt_tokens // max(1, len(unit)) + 1))[:prompt_tokens]
        params = GenerationParams(max_tokens=gen_tokens, temperature=0.0, use_prefix_cache=False,
                                  use_draft=use_draft)
        m = None
        for chunk in self.generate(tokens, params):
            m = chunk.metrics or m
        return {"time": time.time(), "model": self.options.model, "prompt_tokens": m.prompt_tokens,
                "completion_tokens": m.completion_tokens, "ttft_ms": round(m.ttft_ms, 1),
                "prompt_tps": round(m.prompt_tps, 1), "decode_tps": round(m.decode_tps, 2),
                "peak_memory_gb": m.peak_memory_gb,
                "draft_model": self.options.draft_model if use_draft and self.draft_model is not None else None,
                "draft_accepted": m.draft_accepted,
                "kv_bits": self.options.kv_bits, "max_context": self.plan.max_context,
                "expert_streaming": False, "expert_hit_rate": None, "device": torch.cuda.get_device_name(),
                "chip": torch.cuda.get_device_name()}

    # ---------------------------------------------------------------- info
    def info(self) -> dict:
        d: Dict[str, Any] = {"state": self.state, "error": self.error}
        if torch.cuda.is_available():
            free, total = torch.cuda.mem_get_info()
            d["hardware"] = {"device": torch.cuda.get_device_name(), "memory_gb": round(total / GB, 2),
                             "free_gb": round(free / GB, 2)}
        if not self.loaded:
            return d
        opts = self.options
        d["model"] = {"id": opts.model, "type": self.config.get("model_type"),
                      "moe": bool(self.config.get("num_experts")), "resident_gb": round(self.resident_bytes / GB, 2),
                      "load_seconds": round(self.load_seconds, 1), "quantization": self.config.get("quantization")}
        d["options"] = asdict(opts)
        d["context"] = {**self.plan.to_dict(), "current_yarn_factor": self._yarn_now}
        d["expert_streaming"] = None
        d["prefix_cache"] = {"entries": len(self.prefix), "gb": round(self.prefix.nbytes / GB, 2),
                             "hit_tokens": self.prefix.total_hit_tokens,
                             "prompt_tokens": self.prefix.total_prompt_tokens}
        d["last_request"] = asdict(self.last)
        d["totals"] = dict(self.totals)
        return d
