"""q38cu_tensor_gemm_q8_k_noalloc: the GEMM entry point for callers that cannot
allocate device memory (an engine whose device memory comes only from its own
pre-planned arena, since cudaMalloc/cudaFree synchronize the whole device; or
a tiled tensor placed without its scratch buffer).  It must give the same
results as q38cu_tensor_gemm_q8_k, call after call, while using only the
library's one fixed scratch array.

This file is collected last on purpose (a failure here leaves every other
test already run), and passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from q38b200 import synth

pytestmark = pytest.mark.gpu

REL = 1e-3  # the fp32 tolerance used by every GEMM parity test


def _noalloc(q38):
    lib = q38.lib()
    fn = lib.q38cu_tensor_gemm_q8_k_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64,
                   ctypes.POINTER(q38.CuTensor), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    floor = 1e-2 * np.sqrt(np.mean(b * b)) + 1e-30
    return bool(np.all(np.abs(a - b) <= REL * np.maximum(np.abs(b), floor)))


@pytest.mark.parametrize("qtype,rows,width,batch", [
    (O.Q4_K, 17408, 5120, 1),     # one whole tile per CTA
    (O.Q6_K, 40000, 5120, 3),     # more tiles than SMs: tiles shared between CTAs (uses the scratch)
    (O.Q4_K, 5120, 17408, 2),
    # more tokens than one launch takes (8 at width 5120, 4 at 17408): the
    # counters are cleared again before the second launch on the same array
    (O.Q6_K, 40000, 5120, 12),
    (O.Q4_K, 5120, 17408, 6),
])
def test_noalloc_matches_regular_entry_point(q38, oracle, qtype, rows, width, batch):
    import torch
    fn = _noalloc(q38)
    weights = synth.quant_tensor(qtype, rows, width, seed=rows + batch)
    t = q38.DeviceTensor(qtype, width, rows, weights, layout=q38.LAYOUT_TILED)
    act = torch.from_numpy(oracle.quantize_q8_k(synth.activations(batch, width, seed=7))
                           .view(np.uint8).reshape(-1).copy()).cuda()
    expect = q38.gemm_q8_k(t, act, batch).cpu().numpy()

    # the tensor's own scratch is not used: hand over a copy of the
    # descriptor without it
    desc = q38.CuTensor()
    ctypes.memmove(ctypes.byref(desc), ctypes.byref(t.desc), ctypes.sizeof(q38.CuTensor))
    desc.scratch = None
    desc.scratch_bytes = 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # two calls in a row: the shared array keeps the last call's contents
        out = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
        ok = fn(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(act.data_ptr()), batch, width,
                ctypes.byref(desc), stream)
        assert ok == 1, q38.last_error()
        got = out.cpu().numpy()
        assert _close(got, expect), f"call {call}"
    assert q38.device_status() == 0


def test_noalloc_rejects_oversized_scratch(q38):
    """A shape whose scratch exceeds the fixed maximum is refused up front
    (nothing is launched, so the descriptor's data is never read)."""
    fn = _noalloc(q38)
    desc = q38.CuTensor()
    desc.type, desc.n_dims = O.Q6_K, 2
    desc.shape[0], desc.shape[1] = 5120, 8_000_000
    desc.layout, desc.tile_rows = q38.LAYOUT_TILED, 256
    desc.nbytes = 20 * 210 * 8_000_000
    desc.data = 256  # never dereferenced: the call is rejected before any launch
    buf = ctypes.c_void_p(256)
    assert fn(buf, buf, 8, 5120, ctypes.byref(desc), None) == 0
    assert "no-allocation maximum" in q38.last_error()
