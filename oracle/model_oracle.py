"""CPU restatement of one Qwen3.8 decoder layer (TEST INFRASTRUCTURE ONLY).

Used to check the device model layer by layer with teacher forcing: the
device's own input to layer L goes through this restatement and the result is
compared with the device's output of layer L, so an error is located in the
layer that makes it instead of being amplified by the layers after it.

Projections use the upstream engine's own kernels (q38_quantize_q8_k and
q38_tensor_gemv_q8_k / q38_tensor_gemv_f32 from the compiled reference, or
this project's C restatement), so the Q8_K quantization of every projection
input is the upstream one; the rest follows src/qwen38/qwen38_model.c in
float32 numpy:

  q38_rmsnorm            qwen38_model.c:426-435
  q38_linear_core        qwen38_model.c:715-792 (conv, SiLU, L2 norm, delta rule)
  q38_full_core          qwen38_model.c:816-885 (q/k norms, RoPE, softmax)
  q38_layer_forward      qwen38_model.c:955-984
"""
import struct

import numpy as np

F32 = 0

_BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 8: (32, 34), 12: (256, 144), 14: (256, 210), 13: (256, 176),
          10: (256, 84), 11: (256, 110), 16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50),
          20: (32, 18), 21: (256, 110), 22: (256, 82), 23: (256, 136), 29: (256, 56)}


def read_gguf(path):
    """{name: (type, shape, bytes)} of a GGUF v2/v3 file (memory-mapped)."""
    data = np.memmap(path, dtype=np.uint8, mode="r")
    buf = memoryview(data)
    at = 0

    def take(fmt):
        nonlocal at
        v = struct.unpack_from(fmt, buf, at)
        at += struct.calcsize(fmt)
        return v

    def string():
        nonlocal at
        (n,) = take("<Q")
        s = bytes(buf[at:at + n]).decode()
        at += n
        return s

    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

    def skip(kind):
        nonlocal at
        if kind == 8:
            string()
        elif kind == 9:
            (sub,) = take("<I")
            (count,) = take("<Q")
            for _ in range(count):
                skip(sub)
        else:
            at += sizes[kind]

    magic, version, n_tensors, n_meta = take("<IIQQ")
    assert magic == 0x46554747 and version in (2, 3)
    alignment = 32
    for _ in range(n_meta):
        key = string()
        (kind,) = take("<I")
        if key == "general.alignment" and kind == 4:
            (alignment,) = take("<I")
        else:
            skip(kind)
    infos = []
    for _ in range(n_tensors):
        name = string()
        (dims,) = take("<I")
        shape = take("<" + "Q" * dims)
        qtype, offset = take("<IQ")
        infos.append((name, qtype, shape, offset))
    base = (at + alignment - 1) // alignment * alignment
    out = {}
    for name, qtype, shape, offset in infos:
        be, bb = _BLOCK[qtype]
        nbytes = int(np.prod(shape)) // be * bb
        out[name] = (qtype, shape, data[base + offset:base + offset + nbytes])
    return out


def rmsnorm(x, w, eps=1e-6):
    x = np.asarray(x, np.float32)
    mean = np.float32(np.sum(x.astype(np.float64) * x.astype(np.float64)) / x.size)
    scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(eps)))
    return (x * scale) * w


def silu(x):
    x = np.asarray(x, np.float32)
    return x / (np.float32(1) + np.exp(-x))


def sigmoid(x):
    return np.float32(1) / (np.float32(1) + np.exp(-np.asarray(x, np.float32)))


def softplus(x):
    x = np.float32(x)
    return x if x > 20 else np.float32(np.log(np.float32(1) + np.exp(x)))


class LayerOracle:
    """Layer-level restatement over the tensors of one synthetic GGUF.

    `kernels` provides quantize_q8_k(x) and gemm_q8_k(qtype, data, rows,
    width, act) / gemm_f32(qtype, data, rows, width, x) with upstream
    semantics (oracle.Reference or oracle.Oracle)."""

    Q8K_TYPES = {10, 11, 12, 13, 14, 16, 17, 18, 19, 20, 21, 22, 23, 29}

    def __init__(self, path, kernels):
        self.t = read_gguf(path)
        self.k = kernels

    def vec(self, name):
        qtype, shape, raw = self.t[name]
        assert qtype == F32
        return np.frombuffer(raw, np.float32, count=int(np.prod(shape)))

    def project(self, name, x, q8=None):
        """upstream q38_project (qwen38_model.c:599-606)"""
        qtype, shape, raw = self.t[name]
        width, rows = shape
        if qtype in self.Q8K_TYPES:
            q8 = self.k.quantize_q8_k(x) if q8 is None else q8
            return self.k.gemm_q8_k(qtype, raw, rows, width, q8)[0]
        return self.k.gemm_f32(qtype, raw, rows, width, x)[0]

    def deltanet_first_token(self, layer, x):
        """q38_linear_attention at the first position (zero conv and delta
        state) -> the mixer branch."""
        p = f"blk.{layer}."
        q8 = self.k.quantize_q8_k(x)
        qkv = self.project(p + "attn_qkv.weight", x, q8)
        z = self.project(p + "attn_gate.weight", x, q8)
        beta = self.project(p + "ssm_beta.weight", x, q8)
        alpha = self.project(p + "ssm_alpha.weight", x, q8)
        conv = self.vec(p + "ssm_conv1d.weight").reshape(10240, 4)
        qkv = silu(qkv * conv[:, 3])  # zero history: only the newest tap
        q, k, v = qkv[:2048].reshape(16, 128), qkv[2048:4096].reshape(16, 128), qkv[4096:].reshape(48, 128)

        def l2(u):
            s = np.float32(np.sqrt(np.float32(np.sum(u.astype(np.float64) ** 2))))
            return u * (np.float32(1) / max(s, np.float32(1e-6)))

        q = np.stack([l2(h) for h in q])
        k = np.stack([l2(h) for h in k])
        beta = sigmoid(beta)
        a, dt = self.vec(p + "ssm_a"), self.vec(p + "ssm_dt.bias")
        norm = self.vec(p + "ssm_norm.weight")
        out = np.zeros((48, 128), np.float32)
        qs = np.float32(1) / np.sqrt(np.float32(128))
        for vh in range(48):
            kh = vh % 16
            # state 0: prediction 0, delta = v * beta, state column = k * delta
            delta = v[vh] * beta[vh]
            dots = np.float32(k[kh] @ q[kh])
            res = delta * dots * qs
            o = rmsnorm(res, norm)
            out[vh] = o * silu(z[vh * 128:(vh + 1) * 128])
        attn = out.reshape(-1)
        return self.project(p + "ssm_out.weight", attn)

    def full_first_token(self, layer, x):
        """q38_full_attention at position 0: the softmax has one term, so the
        head output is v * sigmoid(gate)."""
        p = f"blk.{layer}."
        q8 = self.k.quantize_q8_k(x)
        qg = self.project(p + "attn_q.weight", x, q8).reshape(24, 512)
        v = self.project(p + "attn_v.weight", x, q8).reshape(4, 256)
        out = np.stack([v[h // 6] * sigmoid(qg[h, 256:]) for h in range(24)]).reshape(-1)
        return self.project(p + "attn_output.weight", out)

    def ffn(self, layer, h):
        p = f"blk.{layer}."
        x = rmsnorm(h, self.vec(p + "post_attention_norm.weight"))
        q8 = self.k.quantize_q8_k(x)
        g = self.project(p + "ffn_gate.weight", x, q8)
        u = self.project(p + "ffn_up.weight", x, q8)
        act = silu(g) * u
        return self.project(p + "ffn_down.weight", act)

    def layer_first_token(self, layer, hidden):
        """q38_layer_forward (qwen38_model.c:955-984) at position 0."""
        hidden = np.asarray(hidden, np.float32).copy()
        x = rmsnorm(hidden, self.vec(f"blk.{layer}.attn_norm.weight"))
        full = (layer + 1) % 4 == 0
        branch = self.full_first_token(layer, x) if full else self.deltanet_first_token(layer, x)
        hidden = hidden + branch
        return hidden + self.ffn(layer, hidden)


def rope(x, heads, position, theta_scale):
    """q38_rope (qwen38_model.c:697-713): first 64 dims of each 256-wide head,
    pairs (j, j + 32), angle position * theta_scale^j."""
    x = np.asarray(x, np.float32).reshape(heads, 256).copy()
    theta = np.float32(position)
    for j in range(32):
        c, s = np.float32(np.cos(theta)), np.float32(np.sin(theta))
        x0, x1 = x[:, j].copy(), x[:, j + 32].copy()
        x[:, j] = x0 * c - x1 * s
        x[:, j + 32] = x0 * s + x1 * c
        theta = np.float32(theta * theta_scale)
    return x


class StatefulLayer:
    """One layer with its recurrent state / KV cache, fed token by token with
    teacher-forced inputs (q38_layer_forward, qwen38_model.c:955-984)."""

    def __init__(self, lo, layer):
        self.lo, self.layer = lo, layer
        self.full = (layer + 1) % 4 == 0
        self.position = 0
        self.conv = np.zeros((10240, 3), np.float32)
        self.state = np.zeros((48, 128, 128), np.float32)  # [head][column][i]
        self.keys, self.values = [], []
        self.theta_scale = np.float32(np.power(np.float32(1e7), np.float32(-2.0 / 64.0)))

    def _deltanet(self, x):
        lo, p = self.lo, f"blk.{self.layer}."
        q8 = lo.k.quantize_q8_k(x)
        qkv = lo.project(p + "attn_qkv.weight", x, q8)
        z = lo.project(p + "attn_gate.weight", x, q8)
        beta = sigmoid(lo.project(p + "ssm_beta.weight", x, q8))
        alpha_raw = lo.project(p + "ssm_alpha.weight", x, q8)
        kern = lo.vec(p + "ssm_conv1d.weight").reshape(10240, 4)
        conv = (((self.conv[:, 0] * kern[:, 0]) + self.conv[:, 1] * kern[:, 1]) + self.conv[:, 2] * kern[:, 2]) \
            + qkv * kern[:, 3]
        self.conv = np.concatenate([self.conv[:, 1:], qkv[:, None]], axis=1)
        act = silu(conv)
        q, k, v = act[:2048].reshape(16, 128), act[2048:4096].reshape(16, 128), act[4096:].reshape(48, 128)

        def l2(u):
            s = np.float32(np.sqrt(np.float32(np.sum(u.astype(np.float64) ** 2))))
            return u * (np.float32(1) / max(s, np.float32(1e-6)))

        q = np.stack([l2(h) for h in q])
        k = np.stack([l2(h) for h in k])
        a, dt = lo.vec(p + "ssm_a"), lo.vec(p + "ssm_dt.bias")
        norm = lo.vec(p + "ssm_norm.weight")
        qs = np.float32(1) / np.sqrt(np.float32(128))
        out = np.zeros((48, 128), np.float32)
        for vh in range(48):
            kh = vh % 16
            decay = np.float32(np.exp(np.float32(a[vh] * softplus(alpha_raw[vh] + dt[vh]))))
            st = self.state[vh] * decay  # [column][i]
            pred = st @ k[kh]
            delta = (v[vh] - pred) * beta[vh]
            st = st + delta[:, None] * k[kh][None, :]
            self.state[vh] = st
            res = (st @ q[kh]) * qs
            out[vh] = rmsnorm(res, norm) * silu(z[vh * 128:(vh + 1) * 128])
        return lo.project(p + "ssm_out.weight", out.reshape(-1))

    def _attention(self, x):
        lo, p = self.lo, f"blk.{self.layer}."
        q8 = lo.k.quantize_q8_k(x)
        qg = lo.project(p + "attn_q.weight", x, q8).reshape(24, 512)
        key = lo.project(p + "attn_k.weight", x, q8).reshape(4, 256)
        val = lo.project(p + "attn_v.weight", x, q8).reshape(4, 256)
        qn, kn = lo.vec(p + "attn_q_norm.weight"), lo.vec(p + "attn_k_norm.weight")
        q = np.stack([rmsnorm(h, qn) for h in qg[:, :256]])
        key = np.stack([rmsnorm(h, kn) for h in key])
        q = rope(q, 24, self.position, self.theta_scale)
        key = rope(key, 4, self.position, self.theta_scale)
        self.keys.append(key)
        self.values.append(val)
        K, V = np.stack(self.keys), np.stack(self.values)  # [pos][4][256]
        out = np.zeros((24, 256), np.float32)
        for h in range(24):
            g = h // 6
            scores = (K[:, g, :].astype(np.float64) @ q[h].astype(np.float64)).astype(np.float32) * np.float32(0.0625)
            e = np.exp(scores - scores.max()).astype(np.float32)
            prob = e / np.float32(e.sum(dtype=np.float64))
            out[h] = (prob[:, None] * V[:, g, :]).sum(axis=0) * sigmoid(qg[h, 256:])
        return lo.project(p + "attn_output.weight", out.reshape(-1))

    def step(self, hidden):
        lo, p = self.lo, f"blk.{self.layer}."
        hidden = np.asarray(hidden, np.float32).copy()
        x = rmsnorm(hidden, lo.vec(p + "attn_norm.weight"))
        hidden = hidden + (self._attention(x) if self.full else self._deltanet(x))
        out = hidden + lo.ffn(self.layer, hidden)
        self.position += 1
        return out
