"""ctypes binding of the device model (include/q38cuda_model.h).

`Model` mirrors the upstream model API (include/qwen38/qwen38_model.h):
open, forward_token, prefill, MTP and speculative greedy decoding, the layer
probe, plus the device-side greedy generation loop.  Logits come back as
numpy copies of the model-owned host buffer.
"""
import ctypes

import numpy as np

from . import lib as _lib, last_error

VOCAB = 248320
HIDDEN = 5120

_BOUND = False


def _bind():
    global _BOUND
    lib = _lib()
    if _BOUND:
        return lib
    vp, u32, fpp = ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.POINTER(ctypes.c_float))
    u32p = ctypes.POINTER(ctypes.c_uint32)
    sig = {
        "q38_model_open_gguf": ([ctypes.c_char_p, u32], vp),
        "q38_model_attach_mtp_gguf": ([vp, ctypes.c_char_p], ctypes.c_int),
        "q38_model_close": ([vp], None),
        "q38_model_reset": ([vp], None),
        "q38_model_forward_token": ([vp, u32, fpp], ctypes.c_int),
        "q38_model_prefill": ([vp, u32p, u32, fpp], ctypes.c_int),
        "q38_model_enable_mtp": ([vp], ctypes.c_int),
        "q38_model_mtp_forward": ([vp, u32, fpp], ctypes.c_int),
        "q38_model_speculative_greedy": ([vp, u32, u32, u32, u32p, u32p, fpp], ctypes.c_int),
        "q38_model_forward_token_layers": ([vp, u32, u32, vp], ctypes.c_int),
        "q38_model_vocab_size": ([vp], u32),
        "q38_model_position": ([vp], u32),
        "q38_model_context_length": ([vp], u32),
        "q38cu_model_generate_greedy": ([vp, u32, u32, u32p], ctypes.c_int),
        "q38cu_model_stream": ([vp], vp),
        "q38cu_model_step_kernels": ([vp], ctypes.c_int),
        "q38cu_model_trace": ([vp, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int], ctypes.c_int),
        "q38cu_model_open_tp": ([ctypes.c_char_p, u32, u32, u32, ctypes.c_char_p], vp),
        "q38cu_nccl_unique_id": ([ctypes.c_char_p], ctypes.c_int),
        "q38cu_tp_shard": ([u32, u32, ctypes.POINTER(TPShard)], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _BOUND = True
    return lib


class ModelError(RuntimeError):
    pass


class TPShard(ctypes.Structure):
    """Q38CuTPShard (include/q38cuda_model.h): what one tensor-parallel rank holds."""
    _fields_ = [("rank", ctypes.c_uint32), ("world", ctypes.c_uint32),
                ("key_heads", ctypes.c_uint32 * 16), ("n_key_heads", ctypes.c_uint32),
                ("value_blocks", ctypes.c_uint32 * 24), ("n_value_blocks", ctypes.c_uint32),
                ("attn_head0", ctypes.c_uint32), ("attn_heads", ctypes.c_uint32),
                ("kv_head0", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("ffn0", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("vocab0", ctypes.c_uint32), ("vocab", ctypes.c_uint32)]


def tp_shard(rank, world):
    """The partition of the model that rank `rank` of `world` GPUs holds (host only)."""
    lib = _bind()
    out = TPShard()
    if lib.q38cu_tp_shard(rank, world, ctypes.byref(out)) != 1:
        raise ModelError(f"q38cu_tp_shard failed: {last_error()}")
    return out


def nccl_unique_id():
    """128 bytes of NCCL communicator id (call on one rank, send to the others)."""
    lib = _bind()
    buf = ctypes.create_string_buffer(128)
    if lib.q38cu_nccl_unique_id(buf) != 1:
        raise ModelError(f"q38cu_nccl_unique_id failed: {last_error()}")
    return buf.raw


class Model:
    """The device-resident model (one CUDA device, the current one at open)."""

    def __init__(self, path, context_length=4096, rank=0, world=1, nccl_id=None):
        """One GPU, or (world > 1) this process's tensor-parallel shard: every
        rank passes the same path, context length, world and nccl_id."""
        self.lib = _bind()
        self.world = world
        if world == 1:
            self.handle = self.lib.q38_model_open_gguf(str(path).encode(), context_length)
        else:
            assert nccl_id is not None and len(nccl_id) == 128
            self.handle = self.lib.q38cu_model_open_tp(str(path).encode(), context_length, rank, world, nccl_id)
        if not self.handle:
            raise ModelError(f"model open failed: {last_error()}")

    def close(self):
        if self.handle:
            self.lib.q38_model_close(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def _logits(self, ptr, rows=1):
        return np.ctypeslib.as_array(ptr, shape=(rows * VOCAB,)).reshape(rows, VOCAB)[-1].copy()

    def _check(self, ok, what):
        if ok != 1:
            raise ModelError(f"{what} failed: {last_error()}")

    def reset(self):
        self.lib.q38_model_reset(self.handle)

    def forward_token(self, token):
        p = ctypes.POINTER(ctypes.c_float)()
        self._check(self.lib.q38_model_forward_token(self.handle, token, ctypes.byref(p)), "forward_token")
        return self._logits(p)

    def forward_token_layers(self, token, layers):
        out = np.zeros(HIDDEN, np.float32)
        self._check(self.lib.q38_model_forward_token_layers(self.handle, token, layers,
                                                            out.ctypes.data_as(ctypes.c_void_p)),
                    "forward_token_layers")
        return out

    def prefill(self, tokens):
        ids = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = ctypes.POINTER(ctypes.c_float)()
        self._check(self.lib.q38_model_prefill(self.handle, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                               ids.size, ctypes.byref(p)), "prefill")
        return self._logits(p)

    def enable_mtp(self):
        self._check(self.lib.q38_model_enable_mtp(self.handle), "enable_mtp")

    def mtp_forward(self, token):
        p = ctypes.POINTER(ctypes.c_float)()
        self._check(self.lib.q38_model_mtp_forward(self.handle, token, ctypes.byref(p)), "mtp_forward")
        return self._logits(p)

    def speculative_greedy(self, token, stop_token, draft_count):
        accepted = np.zeros(max(draft_count, 1), np.uint32)
        count = ctypes.c_uint32(0)
        p = ctypes.POINTER(ctypes.c_float)()
        self._check(self.lib.q38_model_speculative_greedy(
            self.handle, token, stop_token, draft_count,
            accepted.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), ctypes.byref(count), ctypes.byref(p)),
            "speculative_greedy")
        return accepted[:count.value].tolist(), self._logits(p)

    def generate_greedy(self, token, count):
        out = np.zeros(count, np.uint32)
        self._check(self.lib.q38cu_model_generate_greedy(self.handle, token, count,
                                                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))),
                    "generate_greedy")
        return out.tolist()

    @property
    def position(self):
        return self.lib.q38_model_position(self.handle)

    @property
    def context_length(self):
        return self.lib.q38_model_context_length(self.handle)

    @property
    def stream(self):
        return self.lib.q38cu_model_stream(self.handle)

    @property
    def step_kernels(self):
        return self.lib.q38cu_model_step_kernels(self.handle)

    def trace(self, max_records=1024):
        """Launch timeline of the decode step since the last call (needs
        Q38CU_TRACE=1 at open): uint64 array [kernels][11] in ns, launch
        order: min start, min ready, max end, max staged, max decoded, max
        start, max ready, min staged, min RMSNorm sum known, min first
        activation floats arrived, min warp 0 quantized (fields 3.. are only
        set by the weight-streaming GEMV; the last three only for a fused
        RMSNorm input)."""
        buf = np.zeros((max_records, 11), np.uint64)
        n = self.lib.q38cu_model_trace(self.handle, buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                       max_records)
        if n < 0:
            raise ModelError(f"trace failed: {last_error()}")
        return buf[:n]
