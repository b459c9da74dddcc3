"""Failure detection without a GPU fault: a bounded device wait that runs out
returns an error status the host reads, and the context stays usable.

The peer all-reduce (one kernel per residual add under tensor / expert
parallelism) waits for every rank's flag with a wall-clock bound.  Here it
runs on one GPU against a stand-in second rank that never arrives, with a
short bound: the call must return after about that bound, leave the device
error word set (read through m5_device_status by the token loop), leave the
residual stream unchanged, and the GPU must take new work afterwards."""

import ctypes

import pytest
import torch

from myinfer_b200 import _lib

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_reports():
    code, ms, same = ctypes.c_int(0), ctypes.c_double(0), ctypes.c_int(0)
    _lib.call("m5_comm_peer_wait_selftest", 200, ctypes.byref(code), ctypes.byref(ms), ctypes.byref(same))
    assert code.value == 1, code.value
    assert 150 <= ms.value < 5000, ms.value
    assert same.value == 1
    # the selftest cleared the word it read: the device reports clean, and works
    _lib.device_check()
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_device_check_raises_on_recorded_error():
    """The token loop's check turns a recorded wait failure into M5CudaError."""
    code, ms, same = ctypes.c_int(0), ctypes.c_double(0), ctypes.c_int(0)
    _lib.call("m5_comm_peer_wait_selftest", 100, ctypes.byref(code), ctypes.byref(ms), ctypes.byref(same))
    assert code.value == 1
    _lib.device_check()  # already cleared by the selftest
