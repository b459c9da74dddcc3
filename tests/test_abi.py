"""The C ABI library loads on a machine without a GPU, exports every symbol the
public header declares, and rejects bad arguments with a status (never a
crash) before touching the device."""

import ctypes

import pytest

from myinfer_b200 import _lib


def test_exports_every_header_symbol():
    lib = _lib.lib()
    names = _lib.header_symbols()
    assert len(names) >= 17
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(_lib._SIGS), "ctypes signatures and header disagree"


def test_version_and_error_text():
    assert _lib.lib().m5_version() >= 100
    rc = _lib.lib().m5_affine_quantize(None, 0, 1, 64, 64, 64, 4, None, None, None, None)
    assert rc == _lib.M5_ERR_INVALID
    assert "null pointer" in _lib.last_error()


@pytest.mark.parametrize("bits,gs,cols", [(3, 64, 64), (4, 32, 64), (8, 64, 100)])
def test_quantize_argument_checks(bits, gs, cols):
    dummy = ctypes.c_void_p(16)
    rc = _lib.lib().m5_affine_quantize(dummy, 0, 1, cols, cols, gs, bits, dummy, dummy, dummy, None)
    assert rc == _lib.M5_ERR_INVALID


def test_model_config_checks():
    cfg = _lib.M5ModelCfg(hidden_size=1024, num_layers=2, num_heads=16, num_kv_heads=8, head_dim=64,
                          intermediate_size=3072, vocab_size=1000, rms_norm_eps=1e-6, group_size=64, bits=4,
                          tp_size=1, ep_size=1)
    h = ctypes.c_void_p()
    assert _lib.lib().m5_model_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.M5_ERR_INVALID
    assert "head_dim" in _lib.last_error()
    cfg.head_dim = 128
    assert _lib.lib().m5_model_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.M5_OK
    assert _lib.lib().m5_model_bind(h, b"model.layers.9.self_attn.q_proj.weight", ctypes.c_void_p(16)) == \
        _lib.M5_ERR_INVALID
    assert _lib.lib().m5_model_bind(h, b"model.layers.1.self_attn.q_proj.weight", ctypes.c_void_p(16)) == _lib.M5_OK
    assert _lib.lib().m5_model_check(h) == _lib.M5_ERR_STATE
    assert "model.embed_tokens" in _lib.last_error()
    assert _lib.lib().m5_model_destroy(h) == _lib.M5_OK


def test_sdpa_argument_checks():
    v = _lib.M5KvView(16, 16, 16, 0, 100)
    rc = _lib.lib().m5_quantized_sdpa(ctypes.c_void_p(16), 1, 6, 1, 128, v, v, 4, 100, 1.0, 0, None, None, 64, 8,
                                      ctypes.c_void_p(16), None)
    assert rc == _lib.M5_ERR_INVALID and "multiple" in _lib.last_error()
    rc = _lib.lib().m5_quantized_sdpa(ctypes.c_void_p(16), 1, 8, 1, 96, v, v, 4, 100, 1.0, 0, None, None, 64, 8,
                                      ctypes.c_void_p(16), None)
    assert rc == _lib.M5_ERR_INVALID and "head_dim" in _lib.last_error()
