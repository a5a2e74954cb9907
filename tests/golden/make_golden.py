#!/usr/bin/env python3
"""Generate tests/golden/*.npz from the upstream engine's own kernels.

Run in a checkout where the upstream sources were available so that
oracle/_ref/libq38ref.so exists (`make -C oracle`).  The fixtures are small
seeded cases; tests compare both the CPU oracle and the CUDA kernels against
them, so parity stays pinned on machines without the upstream tree.

Per-superblock integer sums are read out of the upstream kernels by running
one-superblock tensors with unit scales: with the fp16 super-scale set so the
float multiplier is 1.0 and the Q8_K block scale set to 1.0, the upstream
float result is exactly the integer sum (all magnitudes stay far below 2^24).
"""
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "qwen3.8-27b-in-c_b200", "python"))

import oracle as O  # noqa: E402
from q38b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
ONE, EIGHT, FOUR = 0x3C00, 0x4800, 0x4400


def set_half(block, offset, value):
    block[offset] = value & 0xFF
    block[offset + 1] = value >> 8


def set_iq1m_scale(block, value):
    words = block[48:56].copy().view(np.uint16)
    for k in range(4):
        words[k] = (words[k] & 0x0FFF) | (((value >> (4 * k)) & 0xF) << 12)
    block[48:56] = words.view(np.uint8)


def unit_blocks(qtype, block):
    """Return (block scaled so v = w, block scaled so v = -x or None)."""
    w_blk = block.copy()
    x_blk = None
    if qtype in (O.Q4_K, O.Q5_K):
        set_half(w_blk, 0, ONE); set_half(w_blk, 2, 0)
        x_blk = block.copy(); set_half(x_blk, 0, 0); set_half(x_blk, 2, ONE)
    elif qtype == O.Q2_K:
        set_half(w_blk, 80, ONE); set_half(w_blk, 82, 0)
        x_blk = block.copy(); set_half(x_blk, 80, 0); set_half(x_blk, 82, ONE)
    elif qtype == O.Q3_K:
        set_half(w_blk, 108, ONE)
    elif qtype == O.Q6_K:
        set_half(w_blk, 208, ONE)
    elif qtype in (O.IQ2_XXS, O.IQ2_XS, O.IQ2_S):
        set_half(w_blk, 0, EIGHT)
    elif qtype == O.IQ3_XXS:
        set_half(w_blk, 0, FOUR)
    elif qtype in (O.IQ3_S, O.IQ4_XS, O.IQ1_S):
        set_half(w_blk, 0, ONE)
    elif qtype == O.IQ1_M:
        set_iq1m_scale(w_blk, ONE)
    return w_blk, x_blk


def ref_block_sums(ref, qtype, block, act_block):
    """Integer sums of one superblock, read from the upstream kernel.

    Returns (w, x); for IQ1_M the upstream folds x into the float result
    alongside w, so the pinned value is 8*w + x (returned as (8*w + x, None))."""
    a = act_block.copy()
    a["scale"] = 1.0
    w_blk, x_blk = unit_blocks(qtype, block)
    if qtype == O.IQ1_M:
        v = ref.gemm_q8_k(qtype, w_blk[None, :], 1, 256, a[None])[0, 0]
        return int(round(v * 8)), None
    if qtype == O.IQ1_S:
        z = a.copy()
        z["sums"] = 0
        w = ref.gemm_q8_k(qtype, w_blk[None, :], 1, 256, z[None])[0, 0]
        full = ref.gemm_q8_k(qtype, w_blk[None, :], 1, 256, a[None])[0, 0]
        return int(w), int(round((full - w) * 8))
    w = ref.gemm_q8_k(qtype, w_blk[None, :], 1, 256, a[None])[0, 0]
    x = 0
    if x_blk is not None:
        x = -ref.gemm_q8_k(qtype, x_blk[None, :], 1, 256, a[None])[0, 0]
    return int(w), int(x)


def main():
    ref = O.Reference()
    cases = {}
    rows, width, batch = 6, 512, 3
    for qtype in O.Q8K_TYPES:
        name = O.TYPE_NAMES[qtype]
        weights = synth.quant_tensor(qtype, rows, width, seed=1000 + qtype)
        x = synth.activations(batch, width, seed=2000 + qtype)
        q8k = ref.quantize_q8_k(x)
        out = ref.gemm_q8_k(qtype, weights, rows, width, q8k)
        gemv = np.stack([ref.gemm_q8_k(qtype, weights, rows, width, q8k[t:t + 1])[0] for t in range(batch)])
        entry = dict(weights=weights, x=x, q8k=q8k.view(np.uint8).reshape(batch, -1), out=out, gemv=gemv)
        if qtype != O.IQ4_NL:
            nb = width // 256
            bb = O.BLOCK[qtype][1]
            ws = np.zeros((batch, rows, nb), np.int64)
            xs = np.zeros((batch, rows, nb), np.int64)
            for t in range(batch):
                for r in range(rows):
                    for b in range(nb):
                        blk = weights[r, b * bb:(b + 1) * bb]
                        w, xx = ref_block_sums(ref, qtype, blk, q8k[t, b])
                        ws[t, r, b] = w
                        xs[t, r, b] = 0 if xx is None else xx
            entry["block_w"] = ws
            entry["block_x"] = xs
        cases[name] = entry
        np.savez_compressed(os.path.join(OUT, f"q8k_{name}.npz"), **entry)

    # Float-activation path and row dequantization.
    for qtype in (O.Q8_0, O.F32, O.F16, O.Q4_K, O.Q6_K, O.Q2_K, O.Q3_K, O.Q5_K, O.IQ4_NL):
        name = O.TYPE_NAMES[qtype]
        weights = synth.quant_tensor(qtype, 5, 512, seed=3000 + qtype)
        x = synth.activations(2, 512, seed=4000 + qtype)
        out = ref.gemm_f32(qtype, weights, 5, 512, x)
        rows_f32 = np.stack([ref.row_f32(qtype, weights, 5, 512, r) for r in range(5)])
        np.savez_compressed(os.path.join(OUT, f"f32_{name}.npz"), weights=weights, x=x, out=out, rows=rows_f32)

    # Q8_K quantizer edge cases.
    rng = np.random.default_rng(77)
    blocks = [
        np.zeros(256, np.float32),                                     # all zero -> scale 0
        np.linspace(-1.0, 1.0, 256, dtype=np.float32),                 # negative extreme first
        np.concatenate([np.full(128, 3.0), np.full(128, -3.0)]).astype(np.float32),  # tie: first wins
        np.concatenate([np.full(128, -3.0), np.full(128, 3.0)]).astype(np.float32),
        (rng.standard_normal(256) * 1e-30).astype(np.float32),         # tiny magnitudes
        (rng.standard_normal(256) * 1e30).astype(np.float32),          # huge magnitudes
        (np.arange(256, dtype=np.float32) - 127.5) / 127.0,            # exact .5 rounding cases
        rng.standard_normal(256).astype(np.float32),
    ]
    xq = np.stack(blocks)
    q = ref.quantize_q8_k(xq)
    np.savez_compressed(os.path.join(OUT, "quantize_edges.npz"), x=xq, q8k=q.view(np.uint8).reshape(len(blocks), -1))
    print("wrote", len(os.listdir(OUT)) - 1, "fixtures to", OUT)


if __name__ == "__main__":
    main()
