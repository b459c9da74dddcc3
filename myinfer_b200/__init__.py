"""myinfer_b200 - B200-native (sm_100a) token loop of M5Engine.

The product path is libm5cuda.so (hand-written CUDA kernels behind a C ABI,
``include/m5cuda.h``) driven from Python through ctypes; torch tensors only
carry device memory and streams.  Modules:

* ``_lib``          ctypes binding of the C ABI (no fallback: errors raise)
* ``ops``           mx.quantize / dequantize / quantized_matmul / rms_norm ...
* ``attention``     blocked_quantized_sdpa / safe_maybe_quantize_kv_cache
* ``cache``         device KVCache / QuantizedKVCache / make_prompt_cache
* ``model``         Qwen3 / Qwen3-MoE model handle, random-init weights
* ``generate``      chunked prefill + CUDA-graph greedy decode loop
* ``context``, ``prefix_cache``, ``engine``  the reference's host policy
"""

__version__ = "0.1.0"
