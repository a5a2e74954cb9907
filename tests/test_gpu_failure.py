"""Failure paths on the GPU, without faulting it.

Every spin in the library's kernels is an mbarrier wait bounded in wall-clock
time (q38_device.cuh: mbar_wait_bounded); when it runs out the kernel records
the wait-timeout status, drains what it has in flight and returns, so the
context stays usable.  q38cu_debug_wait_probe runs that same wait with a short
limit on a barrier nothing completes; the status must come back once, and
ordinary work must run correctly right after it.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from q38b200 import synth

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1  # kStatusWaitTimeout


def _probe(q38):
    fn = q38.lib().q38cu_debug_wait_probe
    fn.argtypes = [ctypes.c_uint64, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def test_bounded_wait_runs_out_and_reports(q38, oracle):
    import torch
    assert q38.device_status() == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _probe(q38)(1_000_000, stream) == 1, q38.last_error()  # 1 ms limit
    assert q38.device_status() == WAIT_TIMEOUT
    assert q38.device_status() == 0, "the status is cleared once read"
    # the context is still usable: a GEMV right after matches the oracle
    rows, width = 64, 512
    w = synth.quant_tensor(O.Q4_K, rows, width, seed=11)
    x = synth.activations(1, width, seed=12)
    t = q38.DeviceTensor(O.Q4_K, width, rows, w, layout=q38.LAYOUT_TILED)
    act = q38.quantize_q8_k(torch.from_numpy(x).cuda())
    got = q38.gemm_q8_k(t, act, 1).cpu().numpy().reshape(-1)
    want = oracle.gemm_q8_k(O.Q4_K, w, rows, width, oracle.quantize_q8_k(x)).reshape(-1)
    assert np.allclose(got, want, rtol=1e-3, atol=1e-3 * np.abs(want).max())
    assert q38.device_status() == 0


def test_wait_probe_rejects_bad_limits(q38):
    fn = _probe(q38)
    assert fn(0, None) == 0
    assert fn(2_000_000_000, None) == 0
