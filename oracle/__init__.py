"""CPU oracle for the M5Engine token loop.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker.

What it restates (numpy for the integer/byte work, torch-CPU fp32 for the
float work):

* ``quant``  - MLX affine group quantization (``mx.quantize`` /
  ``mx.dequantize``, bits 4 and 8, group 64, bf16 scale + bias, values packed
  low-bits-first into uint32).  The reference calls it for the KV cache at
  m5engine/attention.py:111-112 (``to_quantized``) and for every weight via
  mlx-lm ``QuantizedLinear``; the packed layout is also spelled out at
  native/include/tensor.hpp:76-86 and native/src/memory_arena.mm:229-238.
* ``rope``   - plain split-half RoPE and the YaRN frequency table / mscale that
  m5engine/context.py:94-121 swaps in through mlx-lm ``initialize_rope``.
* ``sdpa``   - m5engine/attention.py:29-103 (``blocked_quantized_sdpa``) op for
  op, and the mlx-lm dense quantized SDPA it falls back to (attention.py:42-45).
* ``model``  - the mlx-lm Qwen3 / Qwen3-MoE decoder, its KV caches and the
  chunked-prefill + greedy-decode loop that m5engine/engine.py:420-423 drives.

Parity status: the arithmetic lives in the third-party packages ``mlx>=0.32.4``
and ``mlx-lm==0.31.3`` (requirements.txt:3-4), which are not vendored under
the reference and cannot be installed here.  Against MLX itself the float path
is therefore "parity unpinned"; the restatement is pinned against (a) the
reference's own known-answer tests for the host logic, (b) the dense
dequantized-attention check of tests/test_core.py:16-40, and (c) the
HF ``transformers`` Qwen3 architecture on dequantized weights.
"""
