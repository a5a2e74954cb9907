"""Seeded synthetic GGUF files with the upstream engine's model contract.

The upstream loader accepts exactly one architecture (src/qwen38/
qwen38_model.c:19-39, 209-320): `general.architecture = "qwen35"`, 64 blocks
(65 with the one-layer MTP head), hidden 5120, FFN 17408, 24 query / 4 KV
heads of 256, full attention every 4th block, Gated-DeltaNet blocks with 16
key heads / 48 value heads of 128, vocabulary 248320.  This writer produces a
GGUF v3 file with those tensor names, shapes and metadata and a Q4_K_M-style
type mix (Q6_K for output.weight, every attn_v and ffn_down of even blocks;
Q8_0 for ssm_alpha / ssm_beta; Q4_K for the other matrices, token_embd
included; F32 for norms and the DeltaNet vectors).  Quantized weights follow
the benchmark distributions (see synth.py).  mix="IQ1_M" gives the IQ1_M-typed
variant: every Q4_K matrix but token_embd in IQ1_M, the rest unchanged.

With alias=True the tensors of one role (the name without its "blk.N."
prefix) and one (type, shape) point at a single shared data region across
layers (the upstream reader only bounds-checks offsets,
src/io/qwen38_gguf.c:401-411), which keeps the file near 2 GB; loaders still
see separate tensors, and a device loader uploads each one separately.
Different roles never share bytes (ffn_gate and ffn_up differ, as do
ssm_alpha and ssm_beta), so an exchanged pair shows up in the results.
"""
import struct

import numpy as np

from . import synth

HIDDEN, FFN, LAYERS, VOCAB = 5120, 17408, 64, 248320
ATTN_HEADS, ATTN_KV_HEADS, ATTN_HEAD_DIM = 24, 4, 256
LIN_QK_HEADS, LIN_V_HEADS, LIN_HEAD_DIM = 16, 48, 128
LIN_QKV, LIN_V = 10240, 6144
ATTN_QG, ATTN_Q, ATTN_KV = 12288, 6144, 1024

GGUF_UINT32, GGUF_STRING = 4, 8
ALIGN = 32


MIXES = ("Q4_K_M", "IQ1_M")


def tensor_specs(mtp=False, ffn_down_q6k_every=2, mix="Q4_K_M"):
    """[(name, shape (GGUF order: width first), type)] of the model."""
    assert mix in MIXES, mix
    F32, Q6_K, Q8_0 = synth.F32, synth.Q6_K, synth.Q8_0
    Q4_K = synth.IQ1_M if mix == "IQ1_M" else synth.Q4_K  # the mix's main matrix type
    specs = [("token_embd.weight", (HIDDEN, VOCAB), synth.Q4_K),
             ("output_norm.weight", (HIDDEN,), F32),
             ("output.weight", (HIDDEN, VOCAB), Q6_K)]
    for layer in range(LAYERS + (1 if mtp else 0)):
        p = f"blk.{layer}."
        full = (layer + 1) % 4 == 0 or layer == LAYERS
        down_type = Q6_K if layer % ffn_down_q6k_every == 0 else Q4_K
        specs += [(p + "attn_norm.weight", (HIDDEN,), F32),
                  (p + "post_attention_norm.weight", (HIDDEN,), F32),
                  (p + "ffn_gate.weight", (HIDDEN, FFN), Q4_K),
                  (p + "ffn_up.weight", (HIDDEN, FFN), Q4_K),
                  (p + "ffn_down.weight", (FFN, HIDDEN), down_type)]
        if full:
            specs += [(p + "attn_q.weight", (HIDDEN, ATTN_QG), Q4_K),
                      (p + "attn_k.weight", (HIDDEN, ATTN_KV), Q4_K),
                      (p + "attn_v.weight", (HIDDEN, ATTN_KV), Q6_K),
                      (p + "attn_output.weight", (ATTN_Q, HIDDEN), Q4_K),
                      (p + "attn_q_norm.weight", (ATTN_HEAD_DIM,), F32),
                      (p + "attn_k_norm.weight", (ATTN_HEAD_DIM,), F32)]
        else:
            specs += [(p + "attn_qkv.weight", (HIDDEN, LIN_QKV), Q4_K),
                      (p + "attn_gate.weight", (HIDDEN, LIN_V), Q4_K),
                      (p + "ssm_alpha.weight", (HIDDEN, LIN_V_HEADS), Q8_0),
                      (p + "ssm_beta.weight", (HIDDEN, LIN_V_HEADS), Q8_0),
                      (p + "ssm_conv1d.weight", (4, LIN_QKV), F32),
                      (p + "ssm_dt.bias", (LIN_V_HEADS,), F32),
                      (p + "ssm_a", (LIN_V_HEADS,), F32),
                      (p + "ssm_norm.weight", (LIN_HEAD_DIM,), F32),
                      (p + "ssm_out.weight", (LIN_V, HIDDEN), Q4_K)]
        if layer == LAYERS:
            specs += [(p + "nextn.eh_proj.weight", (2 * HIDDEN, HIDDEN), Q4_K),
                      (p + "nextn.enorm.weight", (HIDDEN,), F32),
                      (p + "nextn.hnorm.weight", (HIDDEN,), F32),
                      (p + "nextn.shared_head_norm.weight", (HIDDEN,), F32)]
    return specs


def _vector_values(name, count, rng):
    """Float vectors: norm weights ~ 1 + N(0, 0.05); ssm_a negative (decay <= 1,
    qwen38_model.c:751-771); dt bias and conv taps small."""
    if name.endswith("ssm_a"):
        return -rng.uniform(0.05, 0.5, count).astype(np.float32)
    if name.endswith("ssm_dt.bias"):
        return rng.normal(0.0, 0.5, count).astype(np.float32)
    if "ssm_conv1d" in name:
        return rng.normal(0.0, 0.3, count).astype(np.float32)
    return (1.0 + rng.normal(0.0, 0.05, count)).astype(np.float32)


# RMS of (scale x quant) for one unit of the fp16 super-scale d, per type, as
# synth.quant_tensor draws them: Q4_K centered sqrt(E[sc^2] E[(q - 7.5)^2]) =
# 36.5 * 4.61; Q6_K sqrt(E[sc^2] E[(q - 32)^2]) = 73.9 * 18.5 (int8 scales);
# Q8_0 sqrt(E[q^2]) = 73.9.
_WEIGHT_RMS_PER_D = {synth.Q4_K: 168.3, synth.Q6_K: 1367.0, synth.Q8_0: 73.9}

DISTRIBUTIONS = ("config0", "centered", "conditioned", "robust")

# "robust": the residual branches' output projections are damped by this
# factor and ROBUST_FAVORED rows of the LM head get ROBUST_FAVOR_SCALE times
# the scale (see _tensor_bytes).
ROBUST_DAMP = 1.0 / 256.0
ROBUST_FAVOR_SCALE = 4.0
ROBUST_FAVORED = tuple(17 + 3880 * k for k in range(64))
_BRANCH_OUTPUTS = ("ssm_out.weight", "attn_output.weight", "ffn_down.weight")


def _tensor_bytes(name, shape, qtype, seed, dist):
    """config0: the single-matvec benchmark draw (fp16 d ~ |N(0, 0.01)|, all
    fields uniform).  centered: the same with zero-mean Q4_K sub-blocks.
    conditioned: centered, with d ~ |N(0, s)| and s chosen per tensor so that
    weights have RMS 1 / sqrt(width): every projection then roughly keeps the
    norm of its input, like a trained checkpoint, instead of multiplying it by
    ~100 per layer.
    robust: conditioned, with the output projections of the residual
    branches (ssm_out, attn_output, ffn_down) damped by ROBUST_DAMP, so a
    perturbation of the residual stream grows by about (1 + damp^2) per
    branch instead of doubling (the 64 conditioned layers amplify a one-ulp
    difference chaotically), and 64 LM-head rows whose scales are
    ROBUST_FAVOR_SCALE times larger, so the greedy choice falls among them
    with top-2 margins of about 15 % of the top logit instead of about 4 %
    for 248,320 equal rows: a random-init model whose greedy tokens are
    stable under the legal evaluation-order differences between correct
    implementations."""
    rng = np.random.default_rng(seed)
    if qtype == synth.F32:
        return _vector_values(name, int(np.prod(shape)), rng).tobytes()
    width, rows = shape
    sigma = 0.01
    if dist in ("conditioned", "robust"):
        sigma = 1.0 / (_WEIGHT_RMS_PER_D[qtype] * np.sqrt(width))
    if dist == "robust" and name.endswith(_BRANCH_OUTPUTS):
        sigma *= ROBUST_DAMP
    data = synth.quant_tensor(qtype, rows, width, seed=seed, sigma=sigma, centered=dist != "config0")
    if dist == "robust" and name == "output.weight":
        assert qtype == synth.Q6_K
        blocks = data.reshape(rows, width // 256, 210)
        for r in ROBUST_FAVORED:
            d = blocks[r, :, 208:210].copy().view(np.float16).astype(np.float32) * ROBUST_FAVOR_SCALE
            blocks[r, :, 208:210] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    return data.tobytes()


def _pack_string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_model_gguf(path, seed=0, mtp=False, alias=True, dist="config0", mix="Q4_K_M"):
    """Write the synthetic model; returns the list of tensor specs.  `dist`
    is one of DISTRIBUTIONS (see _tensor_bytes), `mix` one of MIXES."""
    assert dist in DISTRIBUTIONS, dist
    assert mix == "Q4_K_M" or dist == "config0", "the conditioned and robust draws are defined for Q4_K_M"
    specs = tensor_specs(mtp=mtp, mix=mix)
    meta = [("general.architecture", GGUF_STRING, "qwen35"),
            ("general.alignment", GGUF_UINT32, ALIGN),
            ("qwen35.block_count", GGUF_UINT32, LAYERS + (1 if mtp else 0)),
            ("qwen35.nextn_predict_layers", GGUF_UINT32, 1 if mtp else 0),
            ("qwen35.embedding_length", GGUF_UINT32, HIDDEN),
            ("qwen35.feed_forward_length", GGUF_UINT32, FFN),
            ("qwen35.attention.head_count", GGUF_UINT32, ATTN_HEADS),
            ("qwen35.attention.head_count_kv", GGUF_UINT32, ATTN_KV_HEADS),
            ("qwen35.full_attention_interval", GGUF_UINT32, 4),
            ("qwen35.ssm.state_size", GGUF_UINT32, LIN_HEAD_DIM),
            ("qwen35.ssm.group_count", GGUF_UINT32, LIN_QK_HEADS),
            ("qwen35.ssm.time_step_rank", GGUF_UINT32, LIN_V_HEADS),
            ("qwen35.ssm.inner_size", GGUF_UINT32, LIN_V)]
    # data regions: one per tensor, or one per (type, shape) when aliased
    regions, offsets, region_of = [], [], {}
    cursor = 0
    for index, (name, shape, qtype) in enumerate(specs):
        role = name.split(".", 2)[2] if name.startswith("blk.") else name
        key = (qtype, shape, role) if alias else index
        if key not in region_of:
            nbytes = (np.prod(shape) // synth.BLOCK[qtype][0]) * synth.BLOCK[qtype][1]
            region_of[key] = (cursor, len(regions))
            regions.append((name, shape, qtype, seed * 1000003 + len(regions)))
            cursor += int(nbytes)
            cursor = (cursor + ALIGN - 1) // ALIGN * ALIGN
        offsets.append(region_of[key][0])
    header = struct.pack("<IIQQ", 0x46554747, 3, len(specs), len(meta))
    for key, kind, value in meta:
        header += _pack_string(key) + struct.pack("<I", kind)
        header += _pack_string(value) if kind == GGUF_STRING else struct.pack("<I", value)
    for (name, shape, qtype), offset in zip(specs, offsets):
        header += _pack_string(name) + struct.pack("<I", len(shape))
        header += b"".join(struct.pack("<Q", d) for d in shape)
        header += struct.pack("<IQ", qtype, offset)
    pad = (-len(header)) % ALIGN
    with open(path, "wb") as handle:
        handle.write(header + b"\0" * pad)
        written = 0
        for name, shape, qtype, region_seed in regions:
            data = _tensor_bytes(name, shape, qtype, region_seed, dist)
            handle.write(data)
            written += len(data)
            pad = (-written) % ALIGN
            handle.write(b"\0" * pad)
            written += pad
    return specs


def cached_model_path(seed=1, mtp=True, dist="conditioned", directory=None, mix="Q4_K_M"):
    """Path of the synthetic model for these parameters, written on first use
    (about 2 GB; a few tens of seconds)."""
    import os
    import tempfile
    directory = directory or os.environ.get("Q38_MODEL_DIR") or os.path.join(tempfile.gettempdir(), "q38b200")
    os.makedirs(directory, exist_ok=True)
    name = f"qwen38-synthetic-s{seed}{'-mtp' if mtp else ''}-{dist}{'' if mix == 'Q4_K_M' else '-' + mix}.gguf"
    path = os.path.join(directory, name)
    if not os.path.exists(path):
        partial = path + ".partial"
        write_model_gguf(partial, seed=seed, mtp=mtp, dist=dist, mix=mix)
        os.replace(partial, path)
    return path
