"""Parity of the tensor-core batch GEMM (q38cu_tensor_gemm_q8_k_tc: fp16
dequant-staged operands, tcgen05.mma, fp32 accumulation) with the upstream
integer path on the same Q8_K inputs.

Small shapes are checked against the CPU oracle (the restatement of
qwen38_quant.c); the full model shapes against the device's integer path,
which the kernel-level parity tests pin bit-exactly to the oracle.  The bar
is the north-star's fp32 output bar: 1e-3 relative, with a floor of 1e-2 of
the output RMS for outputs that cancel to near zero.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from q38b200 import synth

pytestmark = pytest.mark.gpu

REL = 1e-3


def _tc(q38):
    lib = q38.lib()
    ws = lib.q38cu_tensor_gemm_q8_k_tc_workspace
    ws.argtypes = [ctypes.c_uint32, ctypes.c_uint64, ctypes.POINTER(q38.CuTensor)]
    ws.restype = ctypes.c_uint64
    fn = lib.q38cu_tensor_gemm_q8_k_tc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64,
                   ctypes.POINTER(q38.CuTensor), ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return ws, fn


def tc_gemm(q38, t, act, batch):
    import torch
    ws_fn, fn = _tc(q38)
    need = ws_fn(batch, t.width, ctypes.byref(t.desc))
    assert need > 0
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 255) // 256 * 256
    out = torch.full((batch, t.rows), float("nan"), dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ok = fn(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(act.data_ptr()), batch, t.width,
            ctypes.byref(t.desc), ctypes.c_void_p(base), need, stream)
    assert ok == 1, q38.last_error()
    got = out.cpu().numpy()
    assert q38.device_status() == 0
    return got


def close(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    floor = 1e-2 * np.sqrt(np.mean(want * want)) + 1e-30
    err = np.abs(got - want) / np.maximum(np.abs(want), floor)
    return float(err.max())


@pytest.mark.parametrize("qtype,rows,width,batch,layout", [
    (O.Q4_K, 256, 512, 256, 0),      # one 128x256 tile pair, GGUF layout
    (O.Q4_K, 384, 1024, 100, 1),     # 128-token tiles, ragged M, tiled layout
    (O.Q6_K, 200, 768, 300, 1),      # ragged rows and tokens, Q6_K
    (O.Q6_K, 128, 256, 1, 0),        # a single token
])
def test_tc_gemm_matches_oracle(q38, oracle, qtype, rows, width, batch, layout):
    import torch
    w = synth.quant_tensor(qtype, rows, width, seed=rows * 7 + batch)
    x = synth.activations(batch, width, seed=batch)
    q8 = oracle.quantize_q8_k(x)
    t = q38.DeviceTensor(qtype, width, rows, w, layout=layout)
    act = torch.from_numpy(q8.view(np.uint8).reshape(-1).copy()).cuda()
    got = tc_gemm(q38, t, act, batch)
    want = oracle.gemm_q8_k(qtype, w, rows, width, q8)
    assert np.all(np.isfinite(got))
    err = close(got, want)
    assert err <= REL, f"max relative error {err:.2e}"


@pytest.mark.parametrize("qtype,rows,width,batch", [
    (O.Q4_K, 17408, 5120, 512),      # ffn_gate / ffn_up at a 512-token chunk
    (O.Q6_K, 5120, 17408, 256),      # ffn_down (Q6_K half of the layers)
    (O.Q4_K, 5120, 6144, 333),       # ssm_out / attn_output, ragged chunk
])
def test_tc_gemm_matches_integer_path_at_model_shapes(q38, qtype, rows, width, batch):
    import torch
    w = synth.quant_tensor(qtype, rows, width, seed=rows + width)
    t = q38.DeviceTensor(qtype, width, rows, w, layout=q38.LAYOUT_TILED)
    x = torch.from_numpy(synth.activations(batch, width, seed=5)).cuda()
    act = q38.quantize_q8_k(x)
    want = q38.gemm_q8_k(t, act, batch).cpu().numpy()
    got = tc_gemm(q38, t, act, batch)
    err = close(got, want)
    assert err <= REL, f"max relative error {err:.2e}"


def test_tc_gemm_rejects_bad_arguments(q38):
    _, fn = _tc(q38)
    desc = q38.CuTensor()
    desc.type, desc.n_dims = O.IQ1_M, 2
    desc.shape[0], desc.shape[1] = 256, 8
    desc.data, desc.nbytes = 256, 8 * 56
    buf = ctypes.c_void_p(256)
    assert fn(buf, buf, 4, 256, ctypes.byref(desc), buf, 1 << 20, None) == 0
    assert "Q4_K and Q6_K" in q38.last_error()
