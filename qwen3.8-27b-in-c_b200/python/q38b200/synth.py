"""Seeded synthetic GGUF-layout tensors with the value distributions of the
benchmark configurations (no checkpoint or dataset is available offline).

* K-quants (Q4_K, Q5_K, Q2_K): fp16 d and dmin ~ |N(0, 0.01)|, packed 6-bit
  scale/min bytes uniform, quant bytes uniform.  With centered=True, Q4_K
  sub-block mins equal their scales and dmin = 7.5 d, so every sub-block is
  d*sc*(q - 7.5): zero-mean weights, as trained checkpoints have (the uniform
  draw gives every row a positive mean, and a random model built from it
  answers every token with the same logits).
* Q6_K / Q3_K: quant and high-bit bytes uniform, int8 scales uniform, fp16
  d ~ |N(0, 0.01)|.
* Q8_0: fp16 d ~ |N(0, 0.01)|, int8 quants uniform.
* IQ types: every index, sign and scale field uniform over its bit range
  (hence uniform over the codebooks), fp16 super-scales ~ |N(0, 0.01)|.

All generators return a uint8 array of shape [rows, row_bytes].
"""
import numpy as np

F32, F16, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 0, 1, 8, 10, 11, 12, 13, 14
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS, IQ1_M, BF16 = (
    16, 17, 18, 19, 20, 21, 22, 23, 29, 30)

BLOCK = {
    F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), IQ4_NL: (32, 18),
    Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176),
    Q6_K: (256, 210), IQ2_XXS: (256, 66), IQ2_XS: (256, 74), IQ3_XXS: (256, 98),
    IQ1_S: (256, 50), IQ3_S: (256, 110), IQ2_S: (256, 82), IQ4_XS: (256, 136),
    IQ1_M: (256, 56),
}

# Byte offset of the fp16 super-scale(s) inside a block.
_SCALE_OFFSETS = {
    Q4_K: (0, 2), Q5_K: (0, 2), Q2_K: (80, 82), Q3_K: (108,), Q6_K: (208,),
    Q8_0: (0,), IQ2_XXS: (0,), IQ2_XS: (0,), IQ2_S: (0,), IQ3_XXS: (0,),
    IQ3_S: (0,), IQ4_XS: (0,), IQ1_S: (0,), IQ4_NL: (0,),
}


def row_bytes(qtype, width):
    elements, nbytes = BLOCK[qtype]
    assert width % elements == 0, (qtype, width)
    return width // elements * nbytes


def half_scales(rng, shape, sigma=0.01):
    """fp16 bit patterns of |N(0, sigma)|."""
    return np.abs(rng.normal(0.0, sigma, size=shape)).astype(np.float16).view(np.uint16)


def _center_q4_k(rng, data, sigma):
    """Q4_K blocks with min_j = scale_j and dmin = 7.5 d (packing as
    ggml-common.h block_q4_K / get_scale_min_k4)."""
    rows, nblocks = data.shape[:2]
    d = np.abs(rng.normal(0.0, sigma, size=(rows, nblocks))).astype(np.float16)
    dmin = (d.astype(np.float32) * 7.5).astype(np.float16)
    sc = rng.integers(0, 64, size=(rows, nblocks, 8), dtype=np.uint8)
    packed = np.empty((rows, nblocks, 12), np.uint8)
    for j in range(4):
        packed[:, :, j] = sc[:, :, j] | ((sc[:, :, j + 4] >> 4) << 6)
        packed[:, :, j + 4] = sc[:, :, j] | ((sc[:, :, j + 4] >> 4) << 6)
        packed[:, :, j + 8] = (sc[:, :, j + 4] & 0xF) | ((sc[:, :, j + 4] & 0xF) << 4)
    data[:, :, 0:2] = d.view(np.uint8).reshape(rows, nblocks, 2)
    data[:, :, 2:4] = dmin.view(np.uint8).reshape(rows, nblocks, 2)
    data[:, :, 4:16] = packed


def quant_tensor(qtype, rows, width, seed, sigma=0.01, centered=False):
    """Random GGUF-layout bytes for a [rows x width] matrix of type qtype."""
    rng = np.random.default_rng(seed)
    elements, nbytes = BLOCK[qtype]
    if qtype == F32:
        return rng.normal(0.0, sigma, size=(rows, width)).astype(np.float32).view(np.uint8).reshape(rows, -1)
    if qtype == F16:
        return rng.normal(0.0, sigma, size=(rows, width)).astype(np.float16).view(np.uint8).reshape(rows, -1)
    nblocks = width // elements
    data = rng.integers(0, 256, size=(rows, nblocks, nbytes), dtype=np.uint8)
    if qtype == IQ1_M:
        # fp16 super-scale spread over the top nibbles of the four scale words.
        bits = half_scales(rng, (rows, nblocks), sigma).astype(np.uint32)
        words = data[:, :, 48:56].copy().view(np.uint16).astype(np.uint32)
        for k in range(4):
            nib = (bits >> (4 * k)) & 0xF
            words[:, :, k] = (words[:, :, k] & 0x0FFF) | (nib << 12)
        data[:, :, 48:56] = words.astype(np.uint16).view(np.uint8).reshape(rows, nblocks, 8)
    elif centered and qtype == Q4_K:
        _center_q4_k(rng, data, sigma)
    else:
        for off in _SCALE_OFFSETS[qtype]:
            h = half_scales(rng, (rows, nblocks), sigma)
            data[:, :, off] = (h & 0xFF).astype(np.uint8)
            data[:, :, off + 1] = (h >> 8).astype(np.uint8)
    return data.reshape(rows, nblocks * nbytes)


def activations(batch, width, seed):
    """fp32 activations ~ N(0, 1)."""
    return np.random.default_rng(seed).standard_normal((batch, width)).astype(np.float32)
