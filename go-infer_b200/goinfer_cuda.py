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
    "gi_cuda_gemm_buf", "gi_cuda_gemm_fused_gate_up_buf", "gi_cuda_add_residual", "gi_cuda_swiglu",
    "gi_cuda_gemv_q8_0", "gi_cuda_gemv_q4_k", "gi_cuda_gemv_q6_k",
    "gi_cuda_gemm_q8_0", "gi_cuda_gemm_q4_k", "gi_cuda_gemm_q6_k", "gi_cuda_gemv_dev",
    "gi_cuda_gemm_dev", "gi_cuda_gemm_dev_noalloc", "gi_cuda_gemv_multi_dev", "gi_cuda_ffn_dev", "gi_cuda_ffn_buf", "gi_cuda_buffer_device_ptr", "gi_cuda_buffer_bytes", "gi_cuda_set_pdl", "gi_cuda_set_q6k_mma", "gi_cuda_set_prefill_pair",
    "gi_cuda_last_error", "gi_quant_row_bytes", "gi_quantize", "gi_quantize_seeded",
    "gi_cuda_alloc_buffers", "gi_cuda_forward_transformer", "gi_cuda_model_create", "gi_cuda_model_destroy",
    "gi_cuda_model_reset", "gi_cuda_model_set_persistent", "gi_cuda_model_generate", "gi_cuda_tp_prepare", "gi_cuda_tp_connect", "gi_cuda_tp_close",
    "gi_cuda_alloc_buffer", "gi_synth_weights", "gi_cuda_buffer_read",
)


class LayerWeights(ctypes.Structure):
    """gi_cuda_layer_weights_t (metal_layer_weights_t, metal_bridge.h:54-67)."""
    _fields_ = [("wq", ctypes.c_void_p), ("wq_type", ctypes.c_int),
                ("wk", ctypes.c_void_p), ("wk_type", ctypes.c_int),
                ("wv", ctypes.c_void_p), ("wv_type", ctypes.c_int),
                ("wo", ctypes.c_void_p), ("wo_type", ctypes.c_int),
                ("ffn_gate", ctypes.c_void_p), ("ffn_gate_type", ctypes.c_int),
                ("ffn_up", ctypes.c_void_p), ("ffn_up_type", ctypes.c_int),
                ("ffn_down", ctypes.c_void_p), ("ffn_down_type", ctypes.c_int),
                ("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p),
                ("bq", ctypes.c_void_p), ("bk", ctypes.c_void_p), ("bv", ctypes.c_void_p)]


class ModelDesc(ctypes.Structure):
    """gi_cuda_model_desc_t."""
    _fields_ = [("num_layers", ctypes.c_uint32), ("dim", ctypes.c_uint32), ("hidden_dim", ctypes.c_uint32),
                ("num_heads", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("vocab_size", ctypes.c_uint32), ("max_seq", ctypes.c_uint32), ("max_pos", ctypes.c_uint32),
                ("norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("layers", ctypes.POINTER(LayerWeights)),
                ("token_embd", ctypes.c_void_p), ("token_embd_type", ctypes.c_int),
                ("output_norm", ctypes.c_void_p),
                ("output_weight", ctypes.c_void_p), ("output_weight_type", ctypes.c_int),
                ("tp_world", ctypes.c_uint32), ("tp_rank", ctypes.c_uint32), ("vocab_offset", ctypes.c_uint32)]


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
        "gi_cuda_gemv_buf": ([i32, vp, vp, vp, u32, u32], i32),
        "gi_cuda_gemm_buf": ([i32, vp, vp, vp, u32, u32, u32], i32),
        "gi_cuda_gemm_fused_gate_up_buf": ([i32, vp, vp, vp, vp, u32, u32, u32], i32),
        "gi_cuda_add_residual": ([vp, vp, u32], i32),
        "gi_cuda_swiglu": ([vp, vp, u32], i32),
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
        "gi_cuda_ffn_dev": ([vp, vp, vp, vp, vp, sz, sz, sz, vp, u32, u32, ctypes.c_float, vp], i32),
        "gi_cuda_ffn_buf": ([f32p, vp, vp, vp, vp, u32, u32, ctypes.c_float], i32),
        "gi_cuda_set_pdl": ([i32], i32),
        "gi_cuda_set_q6k_mma": ([i32], i32),
        "gi_cuda_set_prefill_pair": ([i32], i32),
        "gi_cuda_last_error": ([], ctypes.c_char_p),
        "gi_quant_row_bytes": ([i32, ctypes.c_int64], ctypes.c_int64),
        "gi_quantize": ([i32, f32p, ctypes.c_int64, ctypes.c_int64, vp, i32], i32),
        "gi_quantize_seeded": ([i32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int64, vp, i32], i32),
        "gi_cuda_alloc_buffers": ([u32, u32, u32, u32, u32, u32], i32),
        "gi_cuda_forward_transformer": ([f32p, f32p, ctypes.POINTER(u32), ctypes.POINTER(LayerWeights), vp, vp, i32,
                                         u32, u32, u32, u32, u32, u32, u32, u32, u32, u32, u32, u32,
                                         ctypes.c_float, ctypes.c_float, ctypes.c_float], i32),
        "gi_cuda_model_create": ([ctypes.POINTER(ModelDesc)], vp),
        "gi_cuda_tp_prepare": ([i32, u32, vp], i32),
        "gi_cuda_tp_connect": ([i32, i32, vp], i32),
        "gi_cuda_tp_close": ([], i32),
        "gi_cuda_alloc_buffer": ([sz], vp),
        "gi_cuda_buffer_read": ([vp, vp, sz], i32),
        "gi_synth_weights": ([vp, i32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_int64], i32),
        "gi_cuda_model_destroy": ([vp], None),
        "gi_cuda_model_reset": ([vp], i32),
        "gi_cuda_model_set_persistent": ([vp, i32], i32),
        "gi_cuda_model_generate": ([vp, ctypes.POINTER(ctypes.c_int32), u32, u32, u32, ctypes.POINTER(u32), f32p,
                                    f32p], i32),
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


def _f32_addr(a: np.ndarray) -> int:
    """Address of a C-contiguous float32 array (the per-call hot path: no
    ctypes pointer object is built)."""
    if a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float32 array")
    return a.__array_interface__["data"][0]


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
    rc = (_lib or load_library()).gi_cuda_gemv_buf(quant_type, _f32_addr(y), _f32_addr(x), buf.handle, rows, cols)
    if rc:
        _err("gi_cuda_gemv_buf", rc)


def MatMulBatchBuf(quant_type: int, y: np.ndarray, x: np.ndarray, buf: Buffer, batch: int, rows: int,
                   cols: int) -> None:
    """metal.MatMulBatchBuf (metal_darwin.go:544): y[b*rows + r], x[b*cols + k]."""
    if buf is None or y.size < batch * rows or x.size < batch * cols:
        raise GoInferCudaError("gi_cuda_gemm_buf", ERR_UNAVAILABLE, "bad arguments")
    _err("gi_cuda_gemm_buf", load_library().gi_cuda_gemm_buf(quant_type, _f32_addr(y), _f32_addr(x), buf.handle,
                                                              batch, rows, cols))


def MatMulFusedGateUpBatchBuf(quant_type: int, y: np.ndarray, x: np.ndarray, gate: Buffer, up: Buffer,
                              batch: int, rows: int, cols: int) -> None:
    """metal.MatMulFusedGateUpBatchBuf (metal_darwin.go:564):
    y[b*rows + r] = silu(gate x_b)[r] * (up x_b)[r]; Q4_K only."""
    if gate is None or up is None or y.size < batch * rows or x.size < batch * cols:
        raise GoInferCudaError("gi_cuda_gemm_fused_gate_up_buf", ERR_UNAVAILABLE, "bad arguments")
    _err("gi_cuda_gemm_fused_gate_up_buf", load_library().gi_cuda_gemm_fused_gate_up_buf(
        quant_type, _f32_addr(y), _f32_addr(x), gate.handle, up.handle, batch, rows, cols))


def AddResidual(x: np.ndarray, proj: np.ndarray, dim: int) -> None:
    """metal.AddResidual (metal_darwin.go:743): x[:dim] += proj[:dim], in
    the open batch's order."""
    if x.size < dim or proj.size < dim:
        raise GoInferCudaError("gi_cuda_add_residual", ERR_SHAPE, "bad arguments")
    _err("gi_cuda_add_residual", load_library().gi_cuda_add_residual(_f32_addr(x), _f32_addr(proj), dim))


def SwiGLU(gate: np.ndarray, up: np.ndarray, hidden_dim: int) -> None:
    """metal.SwiGLU (metal_darwin.go:730): gate = silu(gate) * up over the
    first hidden_dim values, in the open batch's order."""
    if gate.size < hidden_dim or up.size < hidden_dim:
        raise GoInferCudaError("gi_cuda_swiglu", ERR_SHAPE, "bad arguments")
    _err("gi_cuda_swiglu", load_library().gi_cuda_swiglu(_f32_addr(gate), _f32_addr(up), hidden_dim))


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


def ffn_dev(x_ptr: int, norm_ptr: int, gate_ptr: int, up_ptr: int, down_ptr: int, gate_bytes: int, up_bytes: int,
            down_bytes: int, h_ptr: int, dim: int, hidden: int, eps: float, stream: int = 0) -> None:
    """x += down(SwiGLU(gate(n), up(n))), n = RMSNorm(x) * norm, on this rank's
    shard (forward.go:275-287; the down partials summed across the ranks after
    tp_connect).  Device pointers; h: `hidden` floats of scratch."""
    _err("gi_cuda_ffn_dev", load_library().gi_cuda_ffn_dev(x_ptr, norm_ptr, gate_ptr, up_ptr, down_ptr, gate_bytes,
                                                            up_bytes, down_bytes, h_ptr, dim, hidden, eps,
                                                            stream or None))


def FFNBuf(x: np.ndarray, norm: Buffer, gate: Buffer, up: Buffer, down: Buffer, dim: int, hidden: int,
           eps: float) -> None:
    """ffn_dev with x in host memory (updated in place) and buffer weights."""
    _err("gi_cuda_ffn_buf", load_library().gi_cuda_ffn_buf(_f32(x), _h(norm), _h(gate), _h(up), _h(down), dim,
                                                            hidden, eps))


def set_pdl(enable: bool) -> None:
    load_library().gi_cuda_set_pdl(1 if enable else 0)


def set_prefill_pair(enable: bool) -> None:
    """Batched GEMMs on CTA pairs (256-row cta_group::2 tcgen05 MMAs) or on single CTAs (the default)."""
    load_library().gi_cuda_set_prefill_pair(1 if enable else 0)


def set_q6k_mma(enable: bool) -> None:
    """Q6_K GEMVs (rows of whole 2048-column groups) on the int8 tensor cores."""
    load_library().gi_cuda_set_q6k_mma(1 if enable else 0)


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
        """weights.go:328-350: False (the caller then loops MatMul per
        token) when the tensor is unknown or the batched call fails."""
        if name not in self.meta or self.bufs.get(name) is None:
            return False
        qtype, _r, _c = self.meta[name]
        try:
            MatMulBatchBuf(qtype, y, x, self.bufs[name], batch, rows, cols)
        except GoInferCudaError:
            return False
        return True

    def MatMulFusedGateUpBatch(self, y: np.ndarray, x: np.ndarray, gate: str, up: str, batch: int, rows: int,
                               cols: int) -> bool:
        """weights.go:352-385: y = silu(gate x) * (up x) per token when both
        tensors are on the device with the same type, else False (the
        caller then runs gate, up and SwiGLU separately)."""
        if gate not in self.meta or up not in self.meta:
            return False
        if self.meta[gate][0] != self.meta[up][0] or self.bufs.get(gate) is None or self.bufs.get(up) is None:
            return False
        try:
            MatMulFusedGateUpBatchBuf(self.meta[gate][0], y, x, self.bufs[gate], self.bufs[up], batch, rows, cols)
        except GoInferCudaError:
            return False
        return True

    def Close(self) -> None:
        for b in self.bufs.values():
            ReleaseBuffer(b)
        self.bufs.clear()


# ---- whole-model decode ----------------------------------------------------

def quantize_seeded(quant_type: int, seed: int, std: float, rows: int, cols: int, threads: int = 0,
                    row0: int = 0, col0: int = 0) -> np.ndarray:
    """Rows [row0, row0+rows) x cols [col0, col0+cols) of a seeded N(0, std)
    matrix, quantised (F32: the float32 values)."""
    rb = cols * 4 if quant_type == TYPE_F32 else row_bytes(quant_type, cols)
    if rb < 0:
        raise GoInferCudaError("gi_quantize_seeded", ERR_UNSUPPORTED_TYPE)
    out = np.empty(max(rows * rb, 1), np.uint8)
    _err("gi_quantize_seeded", load_library().gi_quantize_seeded(quant_type, seed, std, row0, rows, col0, cols,
                                                                   out.ctypes.data, threads))
    return out


def _h(buf) -> Optional[int]:
    return None if buf is None else buf.handle


def layer_table(layers: list[dict]) -> ctypes.Array:
    """LayerWeights[] from dicts of Buffers (keys wq, wk, wv, wo, ffn_gate, ffn_up, ffn_down, attn_norm,
    ffn_norm, optional bq/bk/bv) and their types (wq_type ...)."""
    arr = (LayerWeights * len(layers))()
    for i, L in enumerate(layers):
        e = arr[i]
        for k in ("wq", "wk", "wv", "wo", "ffn_gate", "ffn_up", "ffn_down"):
            setattr(e, k, _h(L[k]))
            setattr(e, k + "_type", L[k + "_type"])
        for k in ("attn_norm", "ffn_norm", "bq", "bk", "bv"):
            setattr(e, k, _h(L.get(k)))
    return arr


def AllocBuffers(dim: int, hidden_dim: int, kv_dim: int, vocab_size: int, num_layers: int, max_seq: int) -> None:
    """metal.AllocBuffers (metal_bridge.h:23)."""
    _err("gi_cuda_alloc_buffers", load_library().gi_cuda_alloc_buffers(dim, hidden_dim, kv_dim, vocab_size,
                                                                         num_layers, max_seq))


def ForwardTransformer(x: np.ndarray, layers: ctypes.Array, out_norm, out_weight, out_type: int, *, num_layers: int,
                       dim: int, hidden_dim: int, kv_dim: int, vocab_size: int, num_heads: int, num_kv_heads: int,
                       head_dim: int, pos: int, slot: int, max_seq: int, active_context: int, norm_eps: float,
                       rope_theta: float, attn_scale: float, want_logits: bool = True):
    """metal.ForwardTransformer (metal_bridge.h:134-157): (logits or None, token)."""
    logits = np.empty(vocab_size, np.float32) if want_logits else None
    tok = ctypes.c_uint32(0)
    _err("gi_cuda_forward_transformer", load_library().gi_cuda_forward_transformer(
        _f32(np.ascontiguousarray(x, np.float32)), _f32(logits) if logits is not None else None,
        ctypes.byref(tok), layers, _h(out_norm), _h(out_weight), out_type, num_layers, dim, hidden_dim, kv_dim,
        vocab_size, num_heads, num_kv_heads, head_dim, pos, slot, max_seq, active_context, norm_eps, rope_theta,
        attn_scale))
    return logits, tok.value


class Model:
    """A device-resident model (gi_cuda_model_*): greedy generation on the GPU."""

    def __init__(self, desc: ModelDesc, keep: object = None):
        self._keep = keep  # buffers and tables that must outlive the handle
        self.vocab = desc.vocab_size
        h = load_library().gi_cuda_model_create(ctypes.byref(desc))
        if not h:
            raise GoInferCudaError("gi_cuda_model_create", ERR_UNAVAILABLE,
                                   load_library().gi_cuda_last_error().decode(errors="replace"))
        self.handle = h

    def generate(self, tokens, n_gen: int, start_pos: int = 0, want_logits: bool = False):
        """(generated ids, last logits or None, device ms of the n_gen - 1 decode steps)."""
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(n_gen, np.uint32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        ms = ctypes.c_float(0.0)
        _err("gi_cuda_model_generate", load_library().gi_cuda_model_generate(
            self.handle, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), toks.size, start_pos, n_gen,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), _f32(logits) if logits is not None else None,
            ctypes.byref(ms)))
        return out, logits, ms.value

    def reset(self) -> None:
        _err("gi_cuda_model_reset", load_library().gi_cuda_model_reset(self.handle))

    def set_persistent(self, enable: bool = True) -> None:
        """Run each step's layers as one persistent kernel (Q4_K layers, no biases)."""
        _err("gi_cuda_model_set_persistent", load_library().gi_cuda_model_set_persistent(self.handle, int(enable)))

    def close(self) -> None:
        if self.handle:
            load_library().gi_cuda_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- tensor parallelism (TPCoordinator's device counterpart) -----------------

def tp_prepare(world: int, max_dim: int) -> bytes:
    """Allocate this rank's exchange region; returns its 64-byte IPC handle."""
    out = ctypes.create_string_buffer(64)
    _err("gi_cuda_tp_prepare", load_library().gi_cuda_tp_prepare(world, max_dim, out))
    return out.raw


def tp_connect(rank: int, world: int, handles: bytes) -> None:
    """Map every rank's region (handles = the ranks' 64-byte handles, in rank order)."""
    if len(handles) != 64 * world:
        raise GoInferCudaError("gi_cuda_tp_connect", ERR_SHAPE, "need 64 bytes per rank")
    buf = ctypes.create_string_buffer(handles, len(handles))
    _err("gi_cuda_tp_connect", load_library().gi_cuda_tp_connect(rank, world, buf))


def tp_close() -> None:
    _err("gi_cuda_tp_close", load_library().gi_cuda_tp_close())


def synth_buffer(quant_type: int, seed: int, std: float, rows: int, cols: int, row0: int = 0,
                 col0: int = 0) -> Buffer:
    """A device buffer holding the synthetic matrix slice drawn on the GPU."""
    rb = cols * 4 if quant_type == TYPE_F32 else row_bytes(quant_type, cols)
    n = rows * rb
    h = load_library().gi_cuda_alloc_buffer(n)
    if not h:
        raise GoInferCudaError("gi_cuda_alloc_buffer", ERR_BUFFER,
                               load_library().gi_cuda_last_error().decode(errors="replace"))
    buf = Buffer(h, n)
    try:
        _err("gi_synth_weights", load_library().gi_synth_weights(h, quant_type, seed, std, row0, rows, col0, cols))
    except Exception:
        ReleaseBuffer(buf)
        raise
    return buf


def read_buffer(buf: Buffer) -> np.ndarray:
    """A buffer's bytes, copied to the host."""
    out = np.empty(buf.nbytes, np.uint8)
    _err("gi_cuda_buffer_read", load_library().gi_cuda_buffer_read(buf.handle, out.ctypes.data, buf.nbytes))
    return out
