"""The sampler on the CPU: the oracle's restatement of mlx-lm's sampler and
processors (m5engine/engine.py:384-392 builds them), the host side of the
device sampler, and the C struct layout the ctypes binding assumes."""

import ctypes
import shutil
import subprocess

import numpy as np
import pytest
import torch

from myinfer_b200 import _lib
from myinfer_b200.sample import DeviceSampler, LogitsPenalty, make_logits_processors, make_sampler, with_processors
from oracle import sample as osmp


def test_splitmix64_published_sequence():
    # SplitMix64 from state 0: the generator's published first outputs
    assert [osmp.splitmix64(0, i) for i in range(3)] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4,
                                                       0x06C45D188009454F]
    u = [osmp.uniform(123, i) for i in range(1000)]
    assert min(u) >= 0.0 and max(u) < 1.0 and abs(np.mean(u) - 0.5) < 0.03


def test_bf16_round_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 37
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(osmp.bf16_round(x), ref)


@pytest.mark.parametrize("top_p,min_p,top_k", [(0.9, 0, 0), (0.5, 0, 0), (0, 0.05, 0), (0, 0, 40), (0.8, 0.02, 25),
                                               (0.95, 0.001, 300), (0.3, 0.5, 3)])
def test_threshold_form_equals_mlx_steps(top_p, min_p, top_k):
    """On rows without ties the composed threshold keeps exactly what mlx-lm's
    sort / cumsum / argpartition steps keep."""
    rng = np.random.default_rng(7)
    for r in range(6):
        v = (rng.standard_normal(3000) * (1 + r)).astype(np.float32)
        while np.unique(v).size != v.size:  # redraw until no two values tie
            v = (rng.standard_normal(3000) * (1 + r)).astype(np.float32)
        lit = osmp.mlx_kept(v, top_p, min_p, top_k)
        thr = osmp.kept_mask(v, top_p, min_p, top_k)
        assert np.array_equal(lit, thr), (r, int(lit.sum()), int(thr.sum()))


def test_ties_at_threshold_are_kept():
    v = np.array([3.0, 2.0, 2.0, 2.0, 1.0], dtype=np.float32)
    assert osmp.kept_mask(v, top_k=2).tolist() == [True, True, True, True, False]


def test_penalties_known_answer():
    row = np.array([2.0, -2.0, 1.0, 0.5, -1.0], dtype=np.float32)
    win = [0, 1, 0, 4, -1, 99]
    v = osmp.apply_penalties(row, win, repetition=2.0)
    assert v.tolist() == [1.0, -4.0, 1.0, 0.5, -2.0]
    v = osmp.apply_penalties(row, win, presence=0.5, frequency=0.25)
    # token 0: 2 - 0.5 - 0.25*2; token 1: -2 - 0.5 - 0.25; token 4: -1 - 0.5 - 0.25
    assert v.tolist() == [1.0, -2.75, 1.0, 0.5, -1.75]


def test_draw_inverse_cdf():
    v = np.log(np.array([0.1, 0.2, 0.3, 0.4], dtype=np.float64)).astype(np.float32)
    keep = np.ones(4, dtype=bool)
    for u, want in [(0.0, 0), (0.05, 0), (0.11, 1), (0.35, 2), (0.65, 3), (0.999, 3)]:
        assert osmp.draw(v, keep, 1.0, u)[0] == want


def test_processor_and_sampler_surface():
    assert make_sampler(0.0) is None
    assert make_logits_processors() == []
    assert make_logits_processors(repetition_penalty=0.0, presence_penalty=None) == []
    p = make_logits_processors(repetition_penalty=1.3, frequency_penalty=0.2)
    assert p == [LogitsPenalty("repetition", 1.3, 20), LogitsPenalty("frequency", 0.2, 20)]
    with pytest.raises(ValueError):
        make_logits_processors(repetition_penalty=-1.0)
    with pytest.raises(ValueError):
        DeviceSampler(0.7, min_p=1.5)
    with pytest.raises(ValueError):
        DeviceSampler(0.7, processors=[LogitsPenalty("repetition", 1.1, 20), LogitsPenalty("presence", 0.1, 10)])
    s = make_sampler(0.7, top_p=0.9, seed=5)
    assert s.seed == 5 and s.window == 0 and s.history([1, 2], "cpu") is None
    g = with_processors(None, p)
    assert isinstance(g, DeviceSampler) and g.greedy and g.window == 20 and g.repetition == 1.3
    s2 = with_processors(s, p)
    assert s2.temp == 0.7 and s2.top_p == 0.9 and s2.seed == 5 and s2.frequency == 0.2
    h = s2.history(list(range(30)), "cpu", rows=2)
    assert h.shape == (2, 20) and h[0].tolist() == list(range(10, 30))
    assert s2.history([7], "cpu")[0].tolist() == [-1] * 19 + [7]
    with pytest.raises(ValueError):
        with_processors(lambda x: x, p)


def test_seeded_samplers_repeat():
    from myinfer_b200 import sample
    sample.seed(11)
    a = [DeviceSampler(1.0).seed for _ in range(3)]
    sample.seed(11)
    b = [DeviceSampler(1.0).seed for _ in range(3)]
    assert a == b and len(set(a)) == 3


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "l.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "m5cuda.h"\nint main(void){'
                   'printf("%zu %zu %zu %zu\\n", sizeof(m5_sample_params), offsetof(m5_sample_params, flags),'
                   ' offsetof(m5_sample_params, seed), offsetof(m5_sample_params, offset)); return 0;}\n')
    exe = tmp_path / "l"
    subprocess.run(["gcc", f"-I{_lib.HEADER_PATH.parent}", str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    S = _lib.M5SampleParams
    assert got == [ctypes.sizeof(S), S.flags.offset, S.seed.offset, S.offset.offset]


def test_sample_argument_checks():
    p = _lib.M5SampleParams(temperature=1.0, top_k=0, repetition_penalty=1.0)
    dummy = ctypes.c_void_p(16)
    L = _lib.lib()
    assert L.m5_sample_bf16(dummy, 1, 1 << 20, 1 << 20, None, 0, 0, p, None, dummy, None) == _lib.M5_ERR_INVALID
    assert "vocab" in _lib.last_error()
    assert L.m5_sample_bf16(dummy, 1, 100, 50, None, 0, 0, p, None, dummy, None) == _lib.M5_ERR_INVALID
    assert L.m5_sample_bf16(dummy, 1, 100, 100, None, 2000, 2000, p, None, dummy, None) == _lib.M5_ERR_INVALID
    p.flags = _lib.M5_SAMPLE_APPEND_HISTORY
    assert L.m5_sample_bf16(dummy, 1, 100, 100, None, 0, 0, p, None, dummy, None) == _lib.M5_ERR_INVALID
    assert "append" in _lib.last_error()
    p.flags = 0
    p.min_p = 2.0
    assert L.m5_sample_bf16(dummy, 1, 100, 100, None, 0, 0, p, None, dummy, None) == _lib.M5_ERR_INVALID


def test_penalty_windows_of_verify_rows():
    """The speculative loop's per-row windows: row i = last W of the context
    before the pending token + the pending token and the first i proposals."""
    from myinfer_b200.generate import penalty_windows
    W = 5
    for ctx in ([], [7], [1, 2, 3, 4, 5, 6, 7, 8]):
        s = DeviceSampler(0.0, processors=[LogitsPenalty("repetition", 1.2, W)])
        prefix = s.history(ctx, "cpu")[0]
        fed = torch.tensor([40, 41, 42, 43], dtype=torch.int32)
        rows = penalty_windows(prefix, fed)
        assert rows.shape == (4, W) and rows.dtype == torch.int32 and rows.is_contiguous()
        for i in range(4):
            full = [-1] * W + list(ctx) + fed[:i + 1].tolist()
            assert rows[i].tolist() == full[-W:], (ctx, i)
