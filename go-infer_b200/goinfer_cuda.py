"""Host-side mirror of go-infer's GPU backend API over libgoinfer_cuda.so.

go-infer's engine reaches its GPU through package ``pkg/metal``
(metal_darwin.go, with stubs in metal_fallback.go): ``Init``,
``IsAvailable``, ``BeginBatch``/``EndBatch``, ``CreateBuffer``/
``ReleaseBuffer``, ``MatMulBuf``, ``MatMulBatchBuf`` and the per-type
``MatMulQ8_0``/``MatMulQ4_K``/``MatMulQ6_K``/``MatMulBatch``.  This module
exposes the same names with the same argument meaning over the C ABI in
include/goinfer_cuda.h; where the Go function returns an ``error`` this
one raises ``GoInferCudaError`` carrying the C status code.  ``Weights``
mirrors the dispatch of pkg/engine/weights.go (``MatMul``/``MatMulBatch``)
with the CUDA backend as its only backend: there is no CPU fallback, and
loading fails loudly when the CUDA library is missing.

The device-pointer helpers (``gemv_dev``, ``gemm_dev``) are the measured
path used by bench.py; they take raw device addresses (e.g. from
``torch.Tensor.data_ptr()``) and a stream handle.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgoinfer_cuda.so")

# GGML type ids, pkg/gguf/types.go:25-52
TYPE_F32 = 0
TYPE_Q8_0 = 8
TYPE_Q4_K = 12
TYPE_Q6_K = 14

OK = 0
ERR_UNAVAILABLE = -1
ERR_UNSUPPORTED_TYPE = -2
ERR_BUFFER = -3
ERR_SHAPE = -4
ERR_CUDA = -5
ERR_TIMEOUT = -6

# Every function include/goinfer_cuda.h declares.
EXPORTS = (
    "gi_cuda_init", "gi_cuda_init_device", "gi_cuda_is_available", "gi_cuda_begin_batch",
    "gi_cuda_end_batch", "gi_cuda_create_buffer", "gi_cuda_release_buffer", "gi_cuda_gemv_buf",
    "gi_cuda_gemm_buf", "gi_cuda_gemv_q8_0", "gi_cuda_gemv_q4_k", "gi_cuda_gemv_q6_k",
    "gi_cuda_gemm_q8_0", "gi_cuda_gemm_q4_k", "gi_cuda_gemm_q6_k", "gi_cuda_gemv_dev",
    "gi_cuda_gemm_dev", "gi_cuda_gemm_dev_noalloc", "gi_cuda_gemv_multi_dev", "gi_cuda_buffer_device_ptr", "gi_cuda_buffer_bytes", "gi_cuda_set_pdl",
    "gi_cuda_last_error", "gi_quant_row_bytes", "gi_quantize",
)


class GoInferCudaError(RuntimeError):
    def __init__(self, what: str, code: int, detail: str = ""):
        super().__init__(f"{what} failed: {code}" + (f" ({detail})" if detail else ""))
        self.code = code


_lib: Optional[ctypes.CDLL] = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libgoinfer_cuda.so (raises if it was never built: no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise GoInferCudaError("load libgoinfer_cuda.so", ERR_UNAVAILABLE,
                               f"{path} is missing; run __graft_entry__.build()")
    L = ctypes.CDLL(path)
    f32p = ctypes.POINTER(ctypes.c_float)
    vp, u32, i32, sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t
    sig = {
        "gi_cuda_init": ([], i32),
        "gi_cuda_init_device": ([i32], i32),
        "gi_cuda_is_available": ([], ctypes.c_bool),
        "gi_cuda_begin_batch": ([], None),
        "gi_cuda_end_batch": ([], None),
        "gi_cuda_create_buffer": ([vp, sz], vp),
        "gi_cuda_release_buffer": ([vp], None),
        "gi_cuda_gemv_buf": ([i32, f32p, f32p, vp, u32, u32], i32),
        "gi_cuda_gemm_buf": ([i32, f32p, f32p, vp, u32, u32, u32], i32),
        "gi_cuda_gemv_q8_0": ([f32p, f32p, vp, u32, u32], i32),
        "gi_cuda_gemv_q4_k": ([f32p, f32p, vp, u32, u32], i32),
        "gi_cuda_gemv_q6_k": ([f32p, f32p, vp, u32, u32], i32),
        "gi_cuda_gemm_q8_0": ([f32p, f32p, vp, u32, u32, u32], i32),
        "gi_cuda_gemm_q4_k": ([f32p, f32p, vp, u32, u32, u32], i32),
        "gi_cuda_gemm_q6_k": ([f32p, f32p, vp, u32, u32, u32], i32),
        "gi_cuda_gemv_dev": ([i32, vp, vp, vp, sz, u32, u32, vp], i32),
        "gi_cuda_gemm_dev": ([i32, vp, vp, vp, sz, u32, u32, u32, vp], i32),
        "gi_cuda_gemm_dev_noalloc": ([i32, vp, vp, vp, sz, u32, u32, u32, vp], i32),
        "gi_cuda_gemv_multi_dev": ([i32, i32, vp, vp, vp, vp, vp, u32, vp], i32),
        "gi_cuda_buffer_device_ptr": ([vp], vp),
        "gi_cuda_buffer_bytes": ([vp], sz),
        "gi_cuda_set_pdl": ([i32], i32),
        "gi_cuda_last_error": ([], ctypes.c_char_p),
        "gi_quant_row_bytes": ([i32, ctypes.c_int64], ctypes.c_int64),
        "gi_quantize": ([i32, f32p, ctypes.c_int64, ctypes.c_int64, vp, i32], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _err(what: str, rc: int) -> None:
    if rc != 0:
        detail = load_library().gi_cuda_last_error().decode(errors="replace")
        raise GoInferCudaError(what, rc, detail)


def _f32(a: np.ndarray):
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _bytes_ptr(raw) -> tuple[ctypes.c_void_p, int, object]:
    arr = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                               else np.asarray(raw).view(np.uint8).reshape(-1))
    return ctypes.c_void_p(arr.ctypes.data), arr.size, arr


# ---- pkg/metal API mirror -------------------------------------------------

def Init(device: Optional[int] = None) -> None:
    """metal.Init (metal_darwin.go:26): bind the library to a CUDA device."""
    L = load_library()
    _err("gi_cuda_init", L.gi_cuda_init() if device is None else L.gi_cuda_init_device(device))


def IsAvailable() -> bool:
    """metal.IsAvailable (metal_darwin.go:37)."""
    try:
        return bool(load_library().gi_cuda_is_available())
    except GoInferCudaError:
        return False


def BeginBatch() -> None:
    """metal.BeginBatch (metal_darwin.go:45)."""
    load_library().gi_cuda_begin_batch()


def EndBatch() -> None:
    """metal.EndBatch (metal_darwin.go:50)."""
    load_library().gi_cuda_end_batch()


class Buffer:
    """A device-resident weight tensor (metal.CreateBuffer's handle)."""

    def __init__(self, handle: int, nbytes: int):
        self.handle = handle
        self.nbytes = nbytes

    @property
    def device_ptr(self) -> int:
        return load_library().gi_cuda_buffer_device_ptr(self.handle) or 0


def CreateBuffer(raw) -> Optional[Buffer]:
    """metal.CreateBuffer (metal_darwin.go:55): None for empty input or on
    failure, as the Go function returns a nil pointer (the reason is in
    gi_cuda_last_error)."""
    ptr, n, _keep = _bytes_ptr(raw)
    if n == 0:
        return None
    h = load_library().gi_cuda_create_buffer(ptr, n)
    return Buffer(h, n) if h else None


def ReleaseBuffer(buf: Optional[Buffer]) -> None:
    """metal.ReleaseBuffer (metal_darwin.go:63)."""
    if buf is not None and buf.handle:
        load_library().gi_cuda_release_buffer(buf.handle)
        buf.handle = 0


def MatMulBuf(quant_type: int, y: np.ndarray, x: np.ndarray, buf: Buffer, rows: int, cols: int) -> None:
    """metal.MatMulBuf (metal_darwin.go:525): y[:rows] = W x."""
    if buf is None or y.size < rows or x.size < cols:
        raise GoInferCudaError("gi_cuda_gemv_buf", ERR_UNAVAILABLE, "bad arguments")
    _err("gi_cuda_gemv_buf", load_library().gi_cuda_gemv_buf(quant_type, _f32(y), _f32(x), buf.handle, rows, cols))


def MatMulBatchBuf(quant_type: int, y: np.ndarray, x: np.ndarray, buf: Buffer, batch: int, rows: int,
                   cols: int) -> None:
    """metal.MatMulBatchBuf (metal_darwin.go:544): y[b*rows + r], x[b*cols + k]."""
    if buf is None or y.size < batch * rows or x.size < batch * cols:
        raise GoInferCudaError("gi_cuda_gemm_buf", ERR_UNAVAILABLE, "bad arguments")
    _err("gi_cuda_gemm_buf", load_library().gi_cuda_gemm_buf(quant_type, _f32(y), _f32(x), buf.handle,
                                                              batch, rows, cols))


def _host_gemv(name: str, y, x, raw, rows, cols):
    ptr, _n, _keep = _bytes_ptr(raw)
    _err(name, getattr(load_library(), name)(_f32(y), _f32(x), ptr, rows, cols))


def MatMulQ8_0(y, x, raw, rows, cols):
    """metal.MatMulQ8_0 (metal_darwin.go:804)."""
    _host_gemv("gi_cuda_gemv_q8_0", y, x, raw, rows, cols)


def MatMulQ4_K(y, x, raw, rows, cols):
    """metal.MatMulQ4_K (metal_darwin.go:819)."""
    _host_gemv("gi_cuda_gemv_q4_k", y, x, raw, rows, cols)


def MatMulQ6_K(y, x, raw, rows, cols):
    """metal.MatMulQ6_K (metal_darwin.go:834)."""
    _host_gemv("gi_cuda_gemv_q6_k", y, x, raw, rows, cols)


def MatMulBatch(y, x, raw, qtype: int, batch: int, rows: int, cols: int) -> None:
    """metal.MatMulBatch (metal_darwin.go:849)."""
    name = {TYPE_Q8_0: "gi_cuda_gemm_q8_0", TYPE_Q4_K: "gi_cuda_gemm_q4_k",
            TYPE_Q6_K: "gi_cuda_gemm_q6_k"}.get(qtype)
    if name is None:
        raise GoInferCudaError("MatMulBatch", ERR_UNSUPPORTED_TYPE)
    ptr, _n, _keep = _bytes_ptr(raw)
    _err(name, getattr(load_library(), name)(_f32(y), _f32(x), ptr, batch, rows, cols))


# ---- device-pointer path (bench, graphs) --------------------------------

def gemv_dev(quant_type: int, y_ptr: int, x_ptr: int, w_ptr: int, w_bytes: int, rows: int, cols: int,
             stream: int = 0) -> None:
    _err("gi_cuda_gemv_dev", load_library().gi_cuda_gemv_dev(quant_type, y_ptr, x_ptr, w_ptr, w_bytes,
                                                              rows, cols, stream or None))


def gemm_dev(quant_type: int, y_ptr: int, x_ptr: int, w_ptr: int, w_bytes: int, batch: int, rows: int,
             cols: int, stream: int = 0) -> None:
    _err("gi_cuda_gemm_dev", load_library().gi_cuda_gemm_dev(quant_type, y_ptr, x_ptr, w_ptr, w_bytes,
                                                              batch, rows, cols, stream or None))


def gemm_dev_noalloc(quant_type: int, y_ptr: int, x_ptr: int, w_ptr: int, w_bytes: int, batch: int, rows: int,
                     cols: int, stream: int = 0) -> None:
    """gemm_dev with the library's fixed 16 MiB scratch: allocates nothing."""
    _err("gi_cuda_gemm_dev_noalloc", load_library().gi_cuda_gemm_dev_noalloc(
        quant_type, y_ptr, x_ptr, w_ptr, w_bytes, batch, rows, cols, stream or None))


def gemv_multi_dev(quant_type: int, ys: list[int], x_ptr: int, ws: list[int], w_bytes: list[int],
                   rows: list[int], cols: int, stream: int = 0) -> None:
    """Up to 3 matrices against one activation vector in one launch (device pointers)."""
    n = len(ys)
    arr_p = ctypes.c_void_p * n
    _err("gi_cuda_gemv_multi_dev", load_library().gi_cuda_gemv_multi_dev(
        quant_type, n, arr_p(*ys), x_ptr, arr_p(*ws), (ctypes.c_size_t * n)(*w_bytes),
        (ctypes.c_uint32 * n)(*rows), cols, stream or None))


def set_pdl(enable: bool) -> None:
    load_library().gi_cuda_set_pdl(1 if enable else 0)


def row_bytes(quant_type: int, cols: int) -> int:
    return int(load_library().gi_quant_row_bytes(quant_type, cols))


def quantize(quant_type: int, src: np.ndarray, threads: int = 0) -> np.ndarray:
    """Quantise a rows x cols float32 matrix into GGUF blocks (host)."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    if src.ndim == 1:
        src = src.reshape(1, -1)
    rows, cols = src.shape
    rb = row_bytes(quant_type, cols)
    if rb < 0:
        raise GoInferCudaError("gi_quantize", ERR_UNSUPPORTED_TYPE)
    out = np.empty(max(rows * rb, 1), dtype=np.uint8)
    _err("gi_quantize", load_library().gi_quantize(quant_type, _f32(src), rows, cols,
                                                    ctypes.c_void_p(out.ctypes.data), threads))
    return out


# ---- pkg/engine/weights.go dispatch mirror --------------------------------

class Weights:
    """Named raw GGUF tensors kept on the device, as NewWeights pre-wraps
    them (pkg/engine/weights.go:21-77), with MatMul/MatMulBatch dispatch
    (weights.go:237-350) going to the CUDA backend only."""

    def __init__(self):
        self.meta: dict[str, tuple[int, int, int]] = {}  # name -> (type, rows, cols)
        self.bufs: dict[str, Buffer] = {}

    def add(self, name: str, qtype: int, rows: int, cols: int, raw) -> None:
        self.meta[name] = (qtype, rows, cols)
        self.bufs[name] = CreateBuffer(raw)

    def MatMul(self, y: np.ndarray, x: np.ndarray, name: str, rows: int, cols: int) -> None:
        qtype, _r, _c = self.meta[name]
        MatMulBuf(qtype, y, x, self.bufs[name], rows, cols)

    def MatMulBatch(self, y: np.ndarray, x: np.ndarray, name: str, batch: int, rows: int, cols: int) -> bool:
        qtype, _r, _c = self.meta[name]
        MatMulBatchBuf(qtype, y, x, self.bufs[name], batch, rows, cols)
        return True

    def Close(self) -> None:
        for b in self.bufs.values():
            ReleaseBuffer(b)
        self.bufs.clear()
