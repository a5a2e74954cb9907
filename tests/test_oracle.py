"""CPU tests: the oracle restatement pinned against the upstream engine.

Pins, in order of strength:
  * golden fixtures produced by the upstream library (tests/golden/), which
    also hold per-superblock integer sums read out of the upstream kernels;
  * the known-answer blocks of the upstream unit tests
    (tests/unit/test_qwen38_quant.c:763-883), restated here;
  * a live comparison against the upstream library when it was built here.
"""
import glob
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN
from q38b200 import synth

Q8K_NAMES = [O.TYPE_NAMES[t] for t in O.Q8K_TYPES]
NAME_TO_TYPE = {v: k for k, v in O.TYPE_NAMES.items()}


def rel_close(actual, expected, rel=1e-5):
    """|a - e| <= rel * max(1, |e|), the upstream test's close_to
    (tests/unit/test_qwen38_quant.c:28-31)."""
    return np.all(np.abs(actual - expected) <= rel * np.maximum(1.0, np.abs(expected)))


def test_f16_edges(oracle):
    # tests/unit/test_qwen38_quant.c:765-769
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xC000) == -2.0
    assert oracle.f16_to_f32(0x0001) == 2.0 ** -24
    assert oracle.f16_to_f32(0x7C00) == float("inf")
    for bits in range(0, 0x10000, 97):
        expect = np.array([bits], np.uint16).view(np.float16).astype(np.float32)[0]
        got = oracle.f16_to_f32(bits)
        assert (np.isnan(expect) and np.isnan(got)) or got == expect


def test_q8k_signed_range(oracle):
    # tests/unit/test_qwen38_quant.c:771-776
    x = ((np.arange(256) - 128) / 128.0).astype(np.float32)
    q = oracle.quantize_q8_k(x)
    assert q["quants"][0, 0] == -127 and q["quants"][0, 128] == 0


def test_quantize_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "quantize_edges.npz"))
    got = oracle.quantize_q8_k(g["x"]).view(np.uint8).reshape(g["q8k"].shape)
    assert np.array_equal(got, g["q8k"])


@pytest.mark.parametrize("name", Q8K_NAMES)
def test_q8k_golden(oracle, name):
    g = np.load(os.path.join(GOLDEN, f"q8k_{name}.npz"))
    qtype = NAME_TO_TYPE[name]
    rows, width = g["weights"].shape[0], g["x"].shape[1]
    q8k = oracle.quantize_q8_k(g["x"])
    assert np.array_equal(q8k.view(np.uint8).reshape(g["q8k"].shape), g["q8k"])
    out = oracle.gemm_q8_k(qtype, g["weights"], rows, width, q8k)
    scale = np.abs(g["out"]).max()
    assert np.max(np.abs(out - g["out"])) <= 1e-5 * scale
    if "block_w" in g:
        w, x = oracle.gemm_q8_k_sums(qtype, g["weights"], rows, width, q8k)
        if qtype == O.IQ1_M:
            assert np.array_equal(8 * w.astype(np.int64) + x, g["block_w"])
        else:
            assert np.array_equal(w, g["block_w"]) and np.array_equal(x, g["block_x"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "f32_*.npz"))), ids=os.path.basename)
def test_f32_golden(oracle, path):
    g = np.load(path)
    qtype = NAME_TO_TYPE[os.path.basename(path)[4:-4]]
    rows, width = g["weights"].shape[0], g["x"].shape[1]
    out = oracle.gemm_f32(qtype, g["weights"], rows, width, g["x"])
    assert np.array_equal(out, g["out"])
    for r in range(rows):
        assert np.array_equal(oracle.row_f32(qtype, g["weights"], rows, width, r), g["rows"][r])


def _half(block, off, value):
    block[off] = value & 0xFF
    block[off + 1] = value >> 8


def known_blocks():
    """Known-answer blocks of tests/unit/test_qwen38_quant.c:778-883 with
    all-ones activations: (type, bytes, expected)."""
    out = []
    q2 = np.zeros(84, np.uint8); q2[:16] = 0x01; q2[16:80] = 0x55; _half(q2, 80, 0x3C00)
    out.append((O.Q2_K, q2, 256.0))
    q3 = np.zeros(110, np.uint8); q3[:32] = 0xFF; q3[32:96] = 0x55; q3[96:104] = 0x11
    q3[104:108] = 0xAA; _half(q3, 108, 0x3C00)
    out.append((O.Q3_K, q3, 256.0))
    q4 = np.zeros(144, np.uint8); _half(q4, 0, 0x3C00); _half(q4, 2, 0x3800)
    q4[4:8] = 1; q4[8:12] = 2; q4[16:] = 0x21
    out.append((O.Q4_K, q4, 64.0))
    q5 = np.zeros(176, np.uint8); _half(q5, 0, 0x3C00); _half(q5, 2, 0x3800)
    q5[4:8] = 1; q5[8:12] = 2; q5[48:] = 0x21
    out.append((O.Q5_K, q5, 64.0))
    q6 = np.zeros(210, np.uint8); q6[192:208] = 1; _half(q6, 208, 0x3C00)
    out.append((O.Q6_K, q6, -8192.0))
    for qtype, nbytes, expected in ((O.IQ2_XXS, 66, 256.0), (O.IQ2_XS, 74, 256.0),
                                    (O.IQ3_XXS, 98, 256.0), (O.IQ3_S, 110, 256.0),
                                    (O.IQ4_XS, 136, 1040384.0), (O.IQ4_NL, 144, -32512.0),
                                    (O.IQ1_S, 50, -224.0), (O.IQ1_M, 56, -224.0),
                                    (O.IQ2_S, 82, 256.0)):
        b = np.zeros(nbytes, np.uint8)
        if qtype == O.IQ4_NL:
            for g in range(8):
                _half(b, 18 * g, 0x3C00)
        elif qtype == O.IQ1_M:
            _half(b, 54, 0x3000)  # fp16 1.0 spread over the top nibbles: 0x3C00 -> 0,0,C,3
            _half(b, 52, 0xC000)
        else:
            _half(b, 0, 0x3C00)
        out.append((qtype, b, expected))
    return out


@pytest.mark.parametrize("qtype,block,expected", known_blocks(),
                         ids=lambda v: O.TYPE_NAMES.get(v, "") if isinstance(v, int) else None)
def test_known_blocks(oracle, qtype, block, expected):
    ones = np.ones(256, np.float32)
    act = oracle.quantize_q8_k(ones)
    if qtype in O.Q8K_TYPES:
        got = oracle.gemm_q8_k(qtype, block[None, :], 1, 256, act)[0, 0]
        assert rel_close(got, expected)
    if qtype in (O.Q2_K, O.Q3_K, O.Q4_K, O.Q5_K, O.Q6_K):
        got = oracle.gemm_f32(qtype, block[None, :], 1, 256, ones[None])[0, 0]
        assert rel_close(got, expected)


def test_q8_0_known_block(oracle):
    b = np.zeros(34, np.uint8); _half(b, 0, 0x3800); b[2:] = 2
    got = oracle.gemm_f32(O.Q8_0, b[None, :], 1, 32, np.ones((1, 32), np.float32))[0, 0]
    assert got == 32.0


def test_batch_major_layout(oracle):
    # tests/unit/test_qwen38_quant.c:802-829
    q4 = known_blocks()[2][1]
    data = np.stack([q4, q4])
    x = np.concatenate([np.ones(256), np.full(256, 2.0)]).astype(np.float32).reshape(2, 256)
    out = oracle.gemm_q8_k(O.Q4_K, data, 2, 256, oracle.quantize_q8_k(x))
    assert rel_close(out.ravel(), np.array([64, 64, 128, 128], np.float32))


@pytest.mark.parametrize("qtype", O.Q8K_TYPES, ids=lambda t: O.TYPE_NAMES[t])
def test_live_against_upstream(oracle, reference, qtype):
    rows, width = 7, 1024
    data = synth.quant_tensor(qtype, rows, width, seed=qtype + 17)
    x = synth.activations(5, width, seed=qtype + 29)
    qo, qr = oracle.quantize_q8_k(x), reference.quantize_q8_k(x)
    assert qo.tobytes() == qr.tobytes()
    a = oracle.gemm_q8_k(qtype, data, rows, width, qo)
    b = reference.gemm_q8_k(qtype, data, rows, width, qr)
    assert np.max(np.abs(a - b)) <= 1e-5 * np.abs(b).max()
