"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Two libraries are wrapped:

* ``_build/libq38oracle.so`` - this project's plain-C restatement of the
  upstream quantized kernels, which also exposes per-superblock integer sums.
* ``_ref/libq38ref.so`` - the upstream engine's own qwen38_quant.c /
  qwen38_gguf.c / qwen38_model.c compiled from its sources (present only where
  the upstream tree was available at build time, and on any machine the
  prebuilt file travelled to).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  The CUDA product never does.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "libq38oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libq38ref.so")
REF_PORTABLE_LIB = os.path.join(HERE, "_ref", "libq38ref_portable.so")
REF_VNNI_LIB = os.path.join(HERE, "_ref", "libq38ref_vnni.so")


def host_has_avx_vnni():
    try:
        with open("/proc/cpuinfo") as handle:
            return any(line.startswith("flags") and " avx_vnni" in line for line in handle)
    except OSError:
        return False


def baseline_reference_lib():
    """The upstream build a CPU baseline should time on this host, and its
    flags: the AVX-VNNI build where the CPU has AVX-VNNI (what the upstream's
    -march=native build compiles there), else the x86-64-v3 build."""
    if host_has_avx_vnni() and os.path.exists(REF_VNNI_LIB):
        return REF_VNNI_LIB, "-O3 -march=x86-64-v3 -mavxvnni -fopenmp (upstream dpbusd branch)"
    return REF_LIB, "-O3 -march=x86-64-v3 -fopenmp (upstream maddubs branch; host has no AVX-VNNI)"

# GGML type ids (GGUF values).
F32, F16, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 0, 1, 8, 10, 11, 12, 13, 14
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS, IQ1_M, BF16 = (
    16, 17, 18, 19, 20, 21, 22, 23, 29, 30)

TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K",
              Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", IQ2_XXS: "IQ2_XXS",
              IQ2_XS: "IQ2_XS", IQ3_XXS: "IQ3_XXS", IQ1_S: "IQ1_S", IQ4_NL: "IQ4_NL",
              IQ3_S: "IQ3_S", IQ2_S: "IQ2_S", IQ4_XS: "IQ4_XS", IQ1_M: "IQ1_M",
              BF16: "BF16"}

BLOCK = {  # type -> (elements, bytes) per GGUF block
    F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), IQ4_NL: (32, 18),
    Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176),
    Q6_K: (256, 210), IQ2_XXS: (256, 66), IQ2_XS: (256, 74), IQ3_XXS: (256, 98),
    IQ1_S: (256, 50), IQ3_S: (256, 110), IQ2_S: (256, 82), IQ4_XS: (256, 136),
    IQ1_M: (256, 56),
}
Q8K_TYPES = (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL,
             IQ3_S, IQ2_S, IQ4_XS, IQ1_S, IQ1_M)

Q8K_DTYPE = np.dtype([("scale", "<f4"), ("quants", "i1", (256,)), ("sums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292


def row_bytes(qtype, width):
    elements, nbytes = BLOCK[qtype]
    assert width % elements == 0
    return width // elements * nbytes


def _ptr(array):
    return ctypes.c_void_p(array.ctypes.data)


class Oracle:
    """The project's C restatement."""

    def __init__(self, path=ORACLE_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(path)
        vp, u64, u32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32
        lib.q38o_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.q38o_f16_to_f32.restype = ctypes.c_float
        lib.q38o_quantize_q8_k.argtypes = [vp, vp, u64]
        lib.q38o_block_sums.argtypes = [u32, vp, vp, vp, vp]
        lib.q38o_block_value.argtypes = [u32, vp, vp]
        lib.q38o_block_value.restype = ctypes.c_float
        lib.q38o_gemm_q8_k.argtypes = [vp, vp, u32, u64, u32, vp, u64]
        lib.q38o_gemm_q8_k_sums.argtypes = [vp, vp, vp, u32, u64, u32, vp, u64]
        lib.q38o_gemm_f32.argtypes = [vp, vp, u32, u64, u32, vp, u64]
        lib.q38o_row_f32.argtypes = [vp, u32, vp, u64, u64, u64]
        self.lib = lib

    def f16_to_f32(self, value):
        return self.lib.q38o_f16_to_f32(value)

    def quantize_q8_k(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size // 256, dtype=Q8K_DTYPE)
        assert self.lib.q38o_quantize_q8_k(_ptr(out), _ptr(x), x.size) == 1
        return out.reshape(x.shape[:-1] + (x.shape[-1] // 256,)) if x.ndim > 1 else out

    def gemm_q8_k(self, qtype, data, rows, width, act):
        act = np.ascontiguousarray(act).reshape(-1, width // 256)
        batch = act.shape[0]
        out = np.zeros((batch, rows), dtype=np.float32)
        data = np.ascontiguousarray(data, dtype=np.uint8)
        assert self.lib.q38o_gemm_q8_k(_ptr(out), _ptr(act), batch, width, qtype, _ptr(data), rows) == 1
        return out

    def gemm_q8_k_sums(self, qtype, data, rows, width, act):
        act = np.ascontiguousarray(act).reshape(-1, width // 256)
        batch = act.shape[0]
        w = np.zeros((batch, rows, width // 256), dtype=np.int32)
        x = np.zeros_like(w)
        data = np.ascontiguousarray(data, dtype=np.uint8)
        assert self.lib.q38o_gemm_q8_k_sums(_ptr(w), _ptr(x), _ptr(act), batch, width, qtype,
                                            _ptr(data), rows) == 1
        return w, x

    def gemm_f32(self, qtype, data, rows, width, x):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, width)
        out = np.zeros((x.shape[0], rows), dtype=np.float32)
        data = np.ascontiguousarray(data, dtype=np.uint8)
        assert self.lib.q38o_gemm_f32(_ptr(out), _ptr(x), x.shape[0], width, qtype, _ptr(data), rows) == 1
        return out

    def row_f32(self, qtype, data, rows, width, row):
        out = np.zeros(width, dtype=np.float32)
        data = np.ascontiguousarray(data, dtype=np.uint8)
        assert self.lib.q38o_row_f32(_ptr(out), qtype, _ptr(data), width, rows, row) == 1
        return out


class _GGUFString(ctypes.Structure):
    _fields_ = [("data", ctypes.c_char_p), ("length", ctypes.c_uint64)]


class GGUFTensor(ctypes.Structure):
    """Mirror of the upstream Q38GGUFTensor (include/qwen38/qwen38_gguf.h:186-195)."""
    _fields_ = [("name", _GGUFString), ("n_dims", ctypes.c_uint32),
                ("shape", ctypes.c_uint64 * 8), ("type", ctypes.c_uint32),
                ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("data", ctypes.c_void_p), ("iq1_s_repack", ctypes.c_void_p)]


def make_tensor(qtype, data, rows, width):
    t = GGUFTensor()
    t.n_dims = 2
    t.shape[0] = width
    t.shape[1] = rows
    t.type = qtype
    t.nbytes = data.nbytes
    t.data = data.ctypes.data
    return t


class Reference:
    """The upstream engine's own kernels (built from its sources)."""

    def __init__(self, path=REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing (built only where the upstream tree exists)")
        lib = ctypes.CDLL(path)
        vp, u64, u32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32
        lib.q38_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.q38_f16_to_f32.restype = ctypes.c_float
        lib.q38_quantize_q8_k.argtypes = [vp, vp, u64]
        lib.q38_tensor_gemv_q8_k.argtypes = [vp, vp, u64, ctypes.POINTER(GGUFTensor)]
        lib.q38_tensor_gemm_q8_k.argtypes = [vp, vp, u32, u64, ctypes.POINTER(GGUFTensor)]
        lib.q38_tensor_gemv_f32.argtypes = [vp, vp, ctypes.POINTER(GGUFTensor)]
        lib.q38_tensor_gemm_f32.argtypes = [vp, vp, u32, u64, ctypes.POINTER(GGUFTensor)]
        lib.q38_tensor_row_f32.argtypes = [vp, ctypes.POINTER(GGUFTensor), u64]
        self.lib = lib

    def f16_to_f32(self, value):
        return self.lib.q38_f16_to_f32(value)

    def quantize_q8_k(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size // 256, dtype=Q8K_DTYPE)
        assert self.lib.q38_quantize_q8_k(_ptr(out), _ptr(x), x.size) == 1
        return out.reshape(x.shape[:-1] + (x.shape[-1] // 256,)) if x.ndim > 1 else out

    def gemm_q8_k(self, qtype, data, rows, width, act):
        act = np.ascontiguousarray(act).reshape(-1, width // 256)
        batch = act.shape[0]
        data = np.ascontiguousarray(data, dtype=np.uint8)
        t = make_tensor(qtype, data, rows, width)
        out = np.zeros((batch, rows), dtype=np.float32)
        if batch == 1:
            ok = self.lib.q38_tensor_gemv_q8_k(_ptr(out), _ptr(act), width, ctypes.byref(t))
        else:
            ok = self.lib.q38_tensor_gemm_q8_k(_ptr(out), _ptr(act), batch, width, ctypes.byref(t))
        assert ok == 1
        return out

    def gemm_f32(self, qtype, data, rows, width, x):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, width)
        data = np.ascontiguousarray(data, dtype=np.uint8)
        t = make_tensor(qtype, data, rows, width)
        out = np.zeros((x.shape[0], rows), dtype=np.float32)
        if x.shape[0] == 1:
            ok = self.lib.q38_tensor_gemv_f32(_ptr(out), _ptr(x), ctypes.byref(t))
        else:
            ok = self.lib.q38_tensor_gemm_f32(_ptr(out), _ptr(x), x.shape[0], width, ctypes.byref(t))
        assert ok == 1
        return out

    def row_f32(self, qtype, data, rows, width, row):
        data = np.ascontiguousarray(data, dtype=np.uint8)
        t = make_tensor(qtype, data, rows, width)
        out = np.zeros(width, dtype=np.float32)
        assert self.lib.q38_tensor_row_f32(_ptr(out), ctypes.byref(t), row) == 1
        return out


def reference_available():
    return os.path.exists(REF_LIB)


class ReferenceModel:
    """The upstream Q38Model (qwen38_model.c compiled from its sources): the
    model-level oracle.  Same method names as q38b200.model.Model."""

    VOCAB = 248320

    def __init__(self, path, context_length=4096, lib_path=REF_LIB):
        if not os.path.exists(lib_path):
            raise FileNotFoundError(f"{lib_path} missing (built only where the upstream tree exists)")
        lib = ctypes.CDLL(lib_path)
        vp, u32 = ctypes.c_void_p, ctypes.c_uint32
        fpp = ctypes.POINTER(ctypes.POINTER(ctypes.c_float))
        u32p = ctypes.POINTER(ctypes.c_uint32)
        sig = {
            "q38_model_open_gguf": ([ctypes.c_char_p, u32], vp),
            "q38_model_close": ([vp], None),
            "q38_model_reset": ([vp], None),
            "q38_model_forward_token": ([vp, u32, fpp], ctypes.c_int),
            "q38_model_prefill": ([vp, u32p, u32, fpp], ctypes.c_int),
            "q38_model_enable_mtp": ([vp], ctypes.c_int),
            "q38_model_mtp_forward": ([vp, u32, fpp], ctypes.c_int),
            "q38_model_speculative_greedy": ([vp, u32, u32, u32, u32p, u32p, fpp], ctypes.c_int),
            "q38_model_forward_token_layers": ([vp, u32, u32, vp], ctypes.c_int),
            "q38_model_position": ([vp], u32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        self.lib = lib
        self.handle = lib.q38_model_open_gguf(str(path).encode(), context_length)
        assert self.handle, "upstream q38_model_open_gguf failed"

    def close(self):
        if self.handle:
            self.lib.q38_model_close(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def _logits(self, p):
        return np.ctypeslib.as_array(p, shape=(self.VOCAB,)).copy()

    def reset(self):
        self.lib.q38_model_reset(self.handle)

    def forward_token(self, token):
        p = ctypes.POINTER(ctypes.c_float)()
        assert self.lib.q38_model_forward_token(self.handle, token, ctypes.byref(p)) == 1
        return self._logits(p)

    def forward_token_layers(self, token, layers):
        out = np.zeros(5120, np.float32)
        assert self.lib.q38_model_forward_token_layers(self.handle, token, layers, _ptr(out)) == 1
        return out

    def prefill(self, tokens):
        ids = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = ctypes.POINTER(ctypes.c_float)()
        assert self.lib.q38_model_prefill(self.handle, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                          ids.size, ctypes.byref(p)) == 1
        return self._logits(p)

    def enable_mtp(self):
        assert self.lib.q38_model_enable_mtp(self.handle) == 1

    def mtp_forward(self, token):
        p = ctypes.POINTER(ctypes.c_float)()
        assert self.lib.q38_model_mtp_forward(self.handle, token, ctypes.byref(p)) == 1
        return self._logits(p)

    def speculative_greedy(self, token, stop_token, draft_count):
        accepted = np.zeros(max(draft_count, 1), np.uint32)
        count = ctypes.c_uint32(0)
        p = ctypes.POINTER(ctypes.c_float)()
        assert self.lib.q38_model_speculative_greedy(
            self.handle, token, stop_token, draft_count,
            accepted.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), ctypes.byref(count), ctypes.byref(p)) == 1
        return accepted[:count.value].tolist(), self._logits(p)

    def generate_greedy(self, token, count):
        """The upstream greedy loop: forward_token, then argmax (q38_argmax:
        the first index of the maximum) as the next input."""
        out = []
        for _ in range(count):
            token = int(np.argmax(self.forward_token(token)))
            out.append(token)
        return out

    @property
    def position(self):
        return self.lib.q38_model_position(self.handle)
