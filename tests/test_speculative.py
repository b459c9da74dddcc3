"""Speculative decoding bookkeeping on the CPU with fake models.

The fake models see exactly the tokens their cache holds plus the tokens of
the call, and pick the next token as a fixed function of that context, so any
slip in acceptance, cache trimming or the draft's backlog shows up as a token
that differs from the main model's plain greedy continuation."""

import torch

from myinfer_b200 import _lib
from myinfer_b200.generate import speculative_generate_step

V = 97


class FakeLayer:
    def __init__(self):
        self.tokens = []
        self.capacity = 1 << 20

    @property
    def offset(self):
        return len(self.tokens)

    def is_trimmable(self):
        return True

    def trim(self, n):
        n = min(n, len(self.tokens))
        del self.tokens[len(self.tokens) - n:]
        return n

    def reserve(self, n):
        pass


class FakeCache(list):
    @property
    def offset(self):
        return self[0].offset


class Args:
    vocab_size = V


class FakeModel:
    """next token = rule(context); logits are one-hot rows."""

    def __init__(self, rule):
        self.rule = rule
        self.args = Args()
        self.device = torch.device("cpu")
        self.calls = 0

    def reserve(self, n):
        pass

    def forward(self, tokens, cache, logits_mode=_lib.M5_LOGITS_NONE, logits=None, argmax_out=None,
                sync_len=True):
        self.calls += 1
        ctx = list(cache[0].tokens)
        rows = []
        for t in tokens.tolist():
            ctx.append(t)
            rows.append(self.rule(ctx))
        cache[0].tokens = ctx
        if logits is not None:
            out = torch.full((len(rows), V), -1.0)
            for i, r in enumerate(rows):
                out[i, r] = 1.0
            if logits_mode == _lib.M5_LOGITS_LAST:
                logits.copy_(out[-1:].reshape(logits.shape).to(logits.dtype))
            else:
                logits.copy_(out.reshape(logits.shape).to(logits.dtype))


def main_rule(ctx):
    return (sum(ctx) * 31 + len(ctx) * 7) % V


def draft_rule(ctx):  # agrees with the main model about two times in three
    r = main_rule(ctx)
    return r if (sum(ctx) % 3) else (r + 1) % V


def greedy(rule, prompt, n):
    ctx, out = list(prompt), []
    for _ in range(n):
        t = rule(ctx)
        out.append(t)
        ctx.append(t)
    return out


def run(prompt, n, k, draft_rule_=draft_rule):
    main, draft = FakeModel(main_rule), FakeModel(draft_rule_)
    mc, dc = FakeCache([FakeLayer()]), FakeCache([FakeLayer()])
    got = list(speculative_generate_step(prompt, main, draft, num_draft_tokens=k, max_tokens=n, prompt_cache=mc,
                                         draft_cache=dc, prefill_step_size=5))
    return got, mc, dc, main


def test_tokens_equal_plain_greedy():
    prompt = [3, 14, 15, 92, 65, 35, 8]
    for k in (1, 2, 3, 5):
        for n in (1, 7, 30):
            got, _, _, _ = run(prompt, n, k)
            assert [t for t, _ in got] == greedy(main_rule, prompt, n), (k, n)


def test_from_draft_flags_and_caches():
    prompt = [1, 2, 3]
    got, mc, dc, main = run(prompt, 40, 3)
    # every from-draft token is the draft rule's choice at that point, all are the main rule's
    ctx = list(prompt)
    for t, fd in got:
        assert t == main_rule(ctx)
        if fd:
            assert t == draft_rule(ctx)
        ctx.append(t)
    assert 0 < sum(fd for _, fd in got) < len(got)
    # fewer main-model calls than tokens: the verify calls score several at once
    assert main.calls < len(got)
    # both caches stay on the accepted context (a prefix of prompt + tokens)
    full = prompt + [t for t, _ in got]
    assert full[:mc[0].offset] == mc[0].tokens
    assert full[:dc[0].offset] == dc[0].tokens


def test_self_draft_accepts_all():
    prompt = [5, 6, 7, 8]
    n, k = 24, 4
    got, _, _, _ = run(prompt, n, k, draft_rule_=main_rule)
    assert [t for t, _ in got] == greedy(main_rule, prompt, n)
    assert sum(fd for _, fd in got) == n - n // (k + 1)
