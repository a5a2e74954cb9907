"""CPU tests of the C ABI: the library loads without a GPU, exports every
symbol include/q38cuda.h and include/q38cuda_model.h declare, and rejects bad
arguments with the upstream return convention (0) before touching the
device."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "q38cuda.h")
MODEL_HEADER = os.path.join(ROOT, "include", "q38cuda_model.h")
# include/qwen38/qwen38_model.h of the upstream engine: the model entry points
# the device model must provide under the same names.
UPSTREAM_MODEL_API = [
    "q38_model_open_gguf", "q38_model_attach_mtp_gguf", "q38_model_close", "q38_model_reset",
    "q38_model_forward_token", "q38_model_prefill", "q38_model_enable_mtp", "q38_model_mtp_forward",
    "q38_model_speculative_greedy", "q38_model_forward_token_layers", "q38_model_vocab_size",
    "q38_model_position", "q38_model_context_length",
]


def declared_functions(path=HEADER, prefix="q38cu_"):
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(" + prefix + r"\w+)\s*\(", text)))


def test_library_exports_header(q38):
    lib = q38.lib()
    names = declared_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name


def test_library_exports_model_api(q38):
    lib = q38.lib()
    names = declared_functions(MODEL_HEADER, prefix="q38(?:cu)?_model_")
    assert set(UPSTREAM_MODEL_API) <= set(names)
    for name in names:
        assert hasattr(lib, name), name


def test_model_rejects_bad_arguments_without_device(q38):
    """Argument checks happen before any device work, as upstream
    (qwen38_model.c:1372, 1497-1498)."""
    from q38b200 import model as M
    lib = M._bind()
    assert not lib.q38_model_open_gguf(None, 16)
    assert not lib.q38_model_open_gguf(b"model.gguf", 0)
    assert lib.q38_model_forward_token(None, 1, None) == 0
    assert lib.q38_model_vocab_size(None) == 0
    assert lib.q38_model_position(None) == 0


def test_host_helpers(q38):
    lib = q38.lib()
    assert lib.q38cu_f16_to_f32(0x3C00) == 1.0
    assert lib.q38cu_f16_to_f32(0x0001) == 2.0 ** -24
    assert lib.q38cu_f16_to_f32(0xC000) == -2.0
    # GGUF block geometry (upstream src/io/qwen38_gguf.c:130-185)
    expect = {12: (256, 144), 14: (256, 210), 8: (32, 34), 19: (256, 50), 29: (256, 56), 22: (256, 82),
              0: (1, 4), 1: (1, 2), 20: (32, 18)}
    for t, (e, b) in expect.items():
        assert lib.q38cu_block_elements(t) == e and lib.q38cu_block_bytes(t) == b
    assert lib.q38cu_block_bytes(2) == 0  # Q4_0 is not part of this engine's formats


def test_rejects_bad_arguments_without_device(q38):
    lib = q38.lib()
    null = ctypes.c_void_p()
    assert lib.q38cu_quantize_q8_k(null, null, 256, null) == 0
    assert "required" in q38.last_error()
    t = q38.CuTensor()
    t.type, t.n_dims, t.shape[0], t.shape[1], t.nbytes = 12, 2, 512, 4, 4 * 288
    t.data = 16
    buf = ctypes.c_void_p(64)
    # width mismatch
    assert lib.q38cu_tensor_gemv_q8_k(buf, buf, 256, ctypes.byref(t), null) == 0
    assert "shape[0]" in q38.last_error()
    # misaligned data
    t.data = 18
    assert lib.q38cu_tensor_gemv_q8_k(buf, buf, 512, ctypes.byref(t), null) == 0
    assert "aligned" in q38.last_error()
    # too few bytes
    t.data, t.nbytes = 16, 100
    assert lib.q38cu_tensor_gemv_q8_k(buf, buf, 512, ctypes.byref(t), null) == 0
    # float-path type on the integer path
    t.type, t.nbytes = 8, 10 ** 6
    assert lib.q38cu_tensor_gemv_q8_k(buf, buf, 512, ctypes.byref(t), null) == 0
    assert "Q8_K" in q38.last_error()
    # zero batch
    t.type = 12
    assert lib.q38cu_tensor_gemm_q8_k(buf, buf, 0, 512, ctypes.byref(t), null) == 0


def test_stream_unit_ownership_formula():
    """The streaming kernel gives CTA c the units [floor(U c / G), floor(U (c+1) / G))
    and finds a unit's owner with ((u + 1) G - 1) // U (q38_stream.cu)."""
    for units in (1, 2, 7, 20, 136, 1360, 19400):
        for grid in range(1, min(units, 300) + 1):
            owner = [((u + 1) * grid - 1) // units for u in range(units)]
            for c in range(grid):
                for u in range(units * c // grid, units * (c + 1) // grid):
                    assert owner[u] == c
