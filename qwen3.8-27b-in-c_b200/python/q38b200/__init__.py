"""Python binding of libq38cuda.so (the C ABI in include/q38cuda.h).

The binding is a thin ctypes layer with the upstream kernel API's names and
semantics (src/qwen38/qwen38_quant.h): q38cu_quantize_q8_k,
q38cu_tensor_gemv_q8_k, q38cu_tensor_gemm_q8_k, q38cu_tensor_gemv_f32,
q38cu_tensor_gemm_f32, q38cu_tensor_row_f32.  PyTorch only provides device
memory and the current CUDA stream; every computation runs in the library's
own sm_100a kernels.  If the library is missing the import fails loudly -
there is no CPU fallback.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.normpath(os.path.join(_HERE, "..", "..", "lib", "libq38cuda.so"))

Q8K_BYTES = 292


LAYOUT_GGUF = 0
LAYOUT_TILED = 1


class CuTensor(ctypes.Structure):
    """Q38CuTensor (include/q38cuda.h)."""
    _fields_ = [("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
                ("shape", ctypes.c_uint64 * 2), ("nbytes", ctypes.c_uint64),
                ("data", ctypes.c_void_p), ("layout", ctypes.c_uint32), ("tile_rows", ctypes.c_uint32),
                ("scratch", ctypes.c_void_p), ("scratch_bytes", ctypes.c_uint64)]


class Q38CudaError(RuntimeError):
    pass


def _load(path=LIB_PATH):
    if not os.path.exists(path):
        raise Q38CudaError(f"{path} is missing: build it with `make -C qwen3.8-27b-in-c_b200/csrc` "
                           "(or __graft_entry__.build()); there is no CPU fallback")
    lib = ctypes.CDLL(path)
    vp, u64, u32, i32p = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p
    tp = ctypes.POINTER(CuTensor)
    sig = {
        "q38cu_f16_to_f32": ([ctypes.c_uint16], ctypes.c_float),
        "q38cu_quantize_q8_k": ([vp, vp, u64, vp], ctypes.c_int),
        "q38cu_tensor_gemv_q8_k": ([vp, vp, u64, tp, vp], ctypes.c_int),
        "q38cu_tensor_gemm_q8_k": ([vp, vp, u32, u64, tp, vp], ctypes.c_int),
        "q38cu_tensor_gemm_q8_k_sums": ([vp, i32p, i32p, vp, u32, u64, tp, vp], ctypes.c_int),
        "q38cu_tensor_gemv_f32": ([vp, vp, tp, vp], ctypes.c_int),
        "q38cu_tensor_gemm_f32": ([vp, vp, u32, u64, tp, vp], ctypes.c_int),
        "q38cu_tensor_row_f32": ([vp, tp, u64, vp], ctypes.c_int),
        "q38cu_tensor_dot_row_f32": ([vp, vp, tp, u64, vp], ctypes.c_int),
        "q38cu_tensor_upload": ([tp, u32, u64, u64, vp, u32, vp], ctypes.c_int),
        "q38cu_tensor_repack": ([tp, tp, vp], ctypes.c_int),
        "q38cu_tensor_free": ([tp], None),
        "q38cu_block_bytes": ([u32], u32),
        "q38cu_block_elements": ([u32], u32),
        "q38cu_last_error": ([], ctypes.c_char_p),
        "q38cu_device_status": ([vp], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def last_error():
    msg = lib().q38cu_last_error()
    return msg.decode() if msg else ""


def _check(ok, what):
    if ok != 1:
        raise Q38CudaError(f"{what} failed: {last_error()}")


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


class DeviceTensor:
    """A GGUF tensor resident in device memory (16-byte aligned, padded)."""

    def __init__(self, qtype, width, rows, host_bytes=None, layout=LAYOUT_GGUF):
        self.desc = CuTensor()
        buf = None
        if host_bytes is not None:
            buf = np.ascontiguousarray(host_bytes, dtype=np.uint8)
        src = ctypes.c_void_p(buf.ctypes.data) if buf is not None else None
        _check(lib().q38cu_tensor_upload(ctypes.byref(self.desc), qtype, width, rows, src, layout, _stream()),
               "q38cu_tensor_upload")
        self.qtype, self.width, self.rows, self.layout = qtype, width, rows, layout

    @property
    def nbytes(self):
        return self.desc.nbytes

    def free(self):
        if self.desc.data:
            lib().q38cu_tensor_free(ctypes.byref(self.desc))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def quantize_q8_k(x, out=None):
    """fp32 [.., K] cuda tensor -> uint8 [.., K/256*292] Q8_K blocks."""
    import torch
    assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
    k = x.shape[-1]
    if out is None:
        out = torch.empty(x.shape[:-1] + (k // 256 * Q8K_BYTES,), dtype=torch.uint8, device=x.device)
    _check(lib().q38cu_quantize_q8_k(_ptr(out), _ptr(x), x.numel(), _stream()), "q38cu_quantize_q8_k")
    return out


def gemm_q8_k(tensor, act, batch, out=None):
    """Batch-major [batch, N] integer GEMM of Q8_K activations against a tensor."""
    import torch
    if out is None:
        out = torch.empty((batch, tensor.rows), dtype=torch.float32, device=act.device)
    if batch == 1:
        ok = lib().q38cu_tensor_gemv_q8_k(_ptr(out), _ptr(act), tensor.width, ctypes.byref(tensor.desc), _stream())
    else:
        ok = lib().q38cu_tensor_gemm_q8_k(_ptr(out), _ptr(act), batch, tensor.width,
                                          ctypes.byref(tensor.desc), _stream())
    _check(ok, "q38cu_tensor_gemm_q8_k")
    return out


def gemm_q8_k_sums(tensor, act, batch):
    """GEMM plus the per-(token, row, superblock) integer sums (w, x)."""
    import torch
    nb = tensor.width // 256
    out = torch.empty((batch, tensor.rows), dtype=torch.float32, device=act.device)
    w = torch.empty((batch, tensor.rows, nb), dtype=torch.int32, device=act.device)
    x = torch.empty_like(w)
    _check(lib().q38cu_tensor_gemm_q8_k_sums(_ptr(out), _ptr(w), _ptr(x), _ptr(act), batch, tensor.width,
                                             ctypes.byref(tensor.desc), _stream()),
           "q38cu_tensor_gemm_q8_k_sums")
    return out, w, x


def gemm_f32(tensor, x, out=None):
    """Float-activation GEMM, x [batch, K] fp32 -> [batch, N]."""
    import torch
    batch = x.shape[0] if x.dim() == 2 else 1
    if out is None:
        out = torch.empty((batch, tensor.rows), dtype=torch.float32, device=x.device)
    _check(lib().q38cu_tensor_gemm_f32(_ptr(out), _ptr(x), batch, tensor.width, ctypes.byref(tensor.desc),
                                       _stream()), "q38cu_tensor_gemm_f32")
    return out


def dot_row_f32(tensor, x, row):
    """Row `row` . x (x [width] fp32 on the device) -> a 1-element device
    tensor; raises when the result is not finite (the upstream's contract)."""
    import torch
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    _check(lib().q38cu_tensor_dot_row_f32(_ptr(out), _ptr(x), ctypes.byref(tensor.desc), row, _stream()),
           "q38cu_tensor_dot_row_f32")
    return out


def row_f32(tensor, row, out=None):
    import torch
    if out is None:
        out = torch.empty(tensor.width, dtype=torch.float32, device="cuda")
    _check(lib().q38cu_tensor_row_f32(_ptr(out), ctypes.byref(tensor.desc), row, _stream()), "q38cu_tensor_row_f32")
    return out


def device_status():
    return lib().q38cu_device_status(_stream())
