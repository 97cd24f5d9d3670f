"""ctypes view of the CPU restatement of go-infer's quantised GEMV path.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py may import this module; the product library never
calls it and never falls back to it.

Each wrapper names the Go function it restates (file:line within
abmarcum/go-infer); goinfer_ref.c holds the restatement itself.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgoinfer_ref.so")

# GGML type ids, pkg/gguf/types.go:25-52
GGML_F32 = 0
GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q6_K = 14

BLOCK = {GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}

_lib = None


def build() -> None:
    """Compile libgoinfer_ref.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        f64p = ctypes.POINTER(ctypes.c_double)
        i64 = ctypes.c_int64
        L.ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.ref_fp16_to_fp32.restype = ctypes.c_float
        L.ref_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.ref_fp32_to_fp16.restype = ctypes.c_uint16
        for name in ("ref_dequantize_q8_0", "ref_dequantize_q4_k", "ref_dequantize_q6_k"):
            getattr(L, name).argtypes = [u8p, ctypes.c_size_t, f32p, i64]
            getattr(L, name).restype = None
        L.ref_dot_vec_f32.argtypes = [f32p, f32p, i64]
        L.ref_dot_vec_f32.restype = ctypes.c_float
        for name in ("ref_dot_vec_q8_0", "ref_dot_vec_q4_k", "ref_dot_vec_q6_k"):
            getattr(L, name).argtypes = [f32p, u8p, i64]
            getattr(L, name).restype = ctypes.c_float
        L.ref_quantize_q8_0.argtypes = [f32p, i64, u8p]
        L.ref_quantize_q8_0.restype = None
        L.ref_bytes_per_row.argtypes = [ctypes.c_int, i64]
        L.ref_bytes_per_row.restype = i64
        L.ref_matmul.argtypes = [ctypes.c_int, f32p, f32p, u8p, i64, i64, ctypes.c_int]
        L.ref_matmul.restype = ctypes.c_int
        L.ref_matmul_f64.argtypes = [ctypes.c_int, f64p, f32p, u8p, i64, i64, ctypes.c_int]
        L.ref_matmul_f64.restype = ctypes.c_int
        L.ref_matmul_absdot.argtypes = [ctypes.c_int, f64p, f32p, u8p, i64, i64, ctypes.c_int]
        L.ref_matmul_absdot.restype = ctypes.c_int
        L.ref_matmul_batch.argtypes = [ctypes.c_int, f32p, f32p, u8p, i64, i64, i64, ctypes.c_int]
        L.ref_matmul_batch.restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _u8(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def fp16_to_fp32(h: int) -> float:
    """FP16ToFP32, pkg/quant/fp16.go:8-35."""
    return lib().ref_fp16_to_fp32(h)


def fp32_to_fp16(v: float) -> int:
    """FP32ToFP16 (truncating), pkg/quant/fp16.go:38-69."""
    return lib().ref_fp32_to_fp16(v)


def bytes_per_row(qtype: int, cols: int) -> int:
    """pkg/math/gemv.go:99,135,171."""
    return int(lib().ref_bytes_per_row(qtype, cols))


def dequantize(qtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    """Dequantize{Q8_0,Q4_K,Q6_K}, pkg/quant/quant.go:196-291."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    out = np.empty(n, dtype=np.float32)
    fn = {GGML_Q8_0: lib().ref_dequantize_q8_0, GGML_Q4_K: lib().ref_dequantize_q4_k,
          GGML_Q6_K: lib().ref_dequantize_q6_k}[qtype]
    fn(_u8(raw), raw.size, _f32(out), n)
    return out


def dot_vec(qtype: int, x: np.ndarray, raw: np.ndarray, n: int) -> float:
    """DotVec{Q8_0,Q4_K,Q6_K,F32}, pkg/quant/quant.go:320-339, 536-566."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if qtype == GGML_F32:
        w = np.ascontiguousarray(raw, dtype=np.float32)
        return float(lib().ref_dot_vec_f32(_f32(x), _f32(w), n))
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    fn = {GGML_Q8_0: lib().ref_dot_vec_q8_0, GGML_Q4_K: lib().ref_dot_vec_q4_k,
          GGML_Q6_K: lib().ref_dot_vec_q6_k}[qtype]
    return float(fn(_f32(x), _u8(raw), n))


def quantize_q8_0(src: np.ndarray) -> np.ndarray:
    """QuantizeQ8_0, pkg/quant/quant.go:407-455."""
    src = np.ascontiguousarray(src, dtype=np.float32).reshape(-1)
    out = np.empty(((src.size + 31) // 32) * 34, dtype=np.uint8)
    lib().ref_quantize_q8_0(_f32(src), src.size, _u8(out))
    return out


def matmul(qtype: int, x: np.ndarray, raw: np.ndarray, rows: int, cols: int,
           nthreads: int | None = None) -> np.ndarray:
    """GEMVEngine.MatMul{Q8_0,Q4_K,Q6_K}, pkg/math/gemv.go:98-203."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    assert x.size >= cols and raw.size >= rows * bytes_per_row(qtype, cols)
    y = np.empty(rows, dtype=np.float32)
    rc = lib().ref_matmul(qtype, _f32(y), _f32(x), _u8(raw), rows, cols,
                          nthreads or os.cpu_count() or 1)
    if rc:
        raise ValueError(f"ref_matmul: unsupported type {qtype}")
    return y


def matmul_f64(qtype: int, x: np.ndarray, raw: np.ndarray, rows: int, cols: int,
               nthreads: int | None = None) -> np.ndarray:
    """Double-accumulated dot over the reference's float32 dequantised rows."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    y = np.empty(rows, dtype=np.float64)
    rc = lib().ref_matmul_f64(qtype, y.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                              _f32(x), _u8(raw), rows, cols, nthreads or os.cpu_count() or 1)
    if rc:
        raise ValueError(f"ref_matmul_f64: unsupported type {qtype}")
    return y


def matmul_absdot(qtype: int, x: np.ndarray, raw: np.ndarray, rows: int, cols: int,
                  nthreads: int | None = None) -> np.ndarray:
    """Per row, sum over k of |w[r,k] * x[k]| (double) over the reference's
    float32 dequantised weights: the conditioning of each output."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    y = np.empty(rows, dtype=np.float64)
    rc = lib().ref_matmul_absdot(qtype, y.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                                 _f32(x), _u8(raw), rows, cols, nthreads or os.cpu_count() or 1)
    if rc:
        raise ValueError(f"ref_matmul_absdot: unsupported type {qtype}")
    return y


def matmul_batch(qtype: int, x: np.ndarray, raw: np.ndarray, batch: int, rows: int,
                 cols: int, nthreads: int | None = None) -> np.ndarray:
    """Per-token Weights.MatMul loop of pkg/engine/forward.go:482-495; y is [batch, rows]."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    assert x.size >= batch * cols
    y = np.empty(batch * rows, dtype=np.float32)
    rc = lib().ref_matmul_batch(qtype, _f32(y), _f32(x), _u8(raw), batch, rows, cols,
                                nthreads or os.cpu_count() or 1)
    if rc:
        raise ValueError(f"ref_matmul_batch: unsupported type {qtype}")
    return y.reshape(batch, rows)


# ---- whole-model decode (ref_forward, the CPU branch of Engine.Forward) ------

class RefMat(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("raw", ctypes.c_void_p)]


class RefLayer(ctypes.Structure):
    _fields_ = [("wq", RefMat), ("wk", RefMat), ("wv", RefMat), ("wo", RefMat), ("gate", RefMat),
                ("up", RefMat), ("down", RefMat), ("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p),
                ("bq", ctypes.c_void_p), ("bk", ctypes.c_void_p), ("bv", ctypes.c_void_p)]


class RefModelC(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("dim", ctypes.c_int), ("hidden", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("vocab", ctypes.c_int),
                ("max_seq", ctypes.c_int), ("eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("tok_embd", RefMat), ("out_norm", ctypes.c_void_p), ("out", RefMat),
                ("layers", ctypes.POINTER(RefLayer)), ("nthreads", ctypes.c_int)]


def _forward_sigs(L):
    L.ref_forward.argtypes = [ctypes.POINTER(RefModelC), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                              ctypes.c_int, ctypes.c_void_p]
    L.ref_forward.restype = ctypes.c_int
    L.ref_rmsnorm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_float]
    L.ref_apply_rope.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    L.ref_swiglu.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    L.ref_softmax.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    L.ref_math_sqrt.argtypes = [ctypes.c_double]
    L.ref_math_sqrt.restype = ctypes.c_double
    L.ref_argmax.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    L.ref_argmax.restype = ctypes.c_int


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    L = lib(); _forward_sigs(L)
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    L.ref_rmsnorm(out.ctypes.data, x.ctypes.data, w.ctypes.data, x.size, eps)
    return out


def apply_rope(vec: np.ndarray, pos: int, theta: float) -> np.ndarray:
    L = lib(); _forward_sigs(L)
    v = np.array(vec, np.float32)
    L.ref_apply_rope(v.ctypes.data, pos, v.size, theta)
    return v


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    L = lib(); _forward_sigs(L)
    g = np.array(gate, np.float32); u = np.ascontiguousarray(up, np.float32)
    L.ref_swiglu(g.ctypes.data, u.ctypes.data, g.size)
    return g


def softmax(x: np.ndarray) -> np.ndarray:
    L = lib(); _forward_sigs(L)
    v = np.array(x, np.float32)
    L.ref_softmax(v.ctypes.data, v.size)
    return v


def math_sqrt(x: float) -> float:
    L = lib(); _forward_sigs(L)
    return L.ref_math_sqrt(x)


class RefModel:
    """The oracle's view of a model: raw tensors {name: (type, array)} with
    go-infer's GGUF names, its own float32 KV cache, Engine.Forward per step."""

    def __init__(self, cfg, tensors: dict, nthreads: int = 0):
        self.cfg = cfg
        self._keep = []

        def mat(name):
            qt, arr = tensors[name]
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            return RefMat(qt, arr.ctypes.data)

        def vec(name):
            _qt, arr = tensors[name]
            arr = np.ascontiguousarray(arr, np.float32)
            self._keep.append(arr)
            return arr.ctypes.data

        def bias(name, n):  # optional (forward.go:211-225): NULL when the model has none
            if name not in tensors:
                return None
            if np.asarray(tensors[name][1]).size != n:
                raise ValueError(f"{name}: {np.asarray(tensors[name][1]).size} values, expected {n}")
            return vec(name)

        layers = (RefLayer * cfg.n_layers)()
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            layers[l] = RefLayer(mat(p + "attn_q.weight"), mat(p + "attn_k.weight"), mat(p + "attn_v.weight"),
                                 mat(p + "attn_output.weight"), mat(p + "ffn_gate.weight"), mat(p + "ffn_up.weight"),
                                 mat(p + "ffn_down.weight"), vec(p + "attn_norm.weight"),
                                 vec(p + "ffn_norm.weight"), bias(p + "attn_q.bias", cfg.q_dim),
                                 bias(p + "attn_k.bias", cfg.kv_dim), bias(p + "attn_v.bias", cfg.kv_dim))
        self._layers = layers
        self.c = RefModelC(cfg.n_layers, cfg.dim, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.vocab, cfg.max_seq,
                           cfg.eps, cfg.rope_theta, mat("token_embd.weight"), vec("output_norm.weight"),
                           mat("output.weight"), layers, nthreads or os.cpu_count() or 1)
        kv = cfg.n_layers * cfg.max_seq * cfg.kv_dim
        self.key = np.zeros(kv, np.float32)
        self.value = np.zeros(kv, np.float32)

    def forward(self, token: int, pos: int) -> np.ndarray:
        L = lib(); _forward_sigs(L)
        logits = np.empty(self.cfg.vocab, np.float32)
        rc = L.ref_forward(ctypes.byref(self.c), self.key.ctypes.data, self.value.ctypes.data, token, pos,
                           logits.ctypes.data)
        if rc:
            raise RuntimeError(f"ref_forward failed: {rc}")
        return logits

    def greedy(self, prompt, n_gen: int, start_pos: int = 0, progress=None):
        """Engine.Generate at temperature 0 with sequential prefill: the ids
        and, per generated id, the top-2 logit margin.  progress(i, n), if
        given, is called before forward step i of n."""
        L = lib(); _forward_sigs(L)
        pos = start_pos
        logits = None
        total = len(prompt) + n_gen - 1
        for t in prompt:
            if progress:
                progress(pos - start_pos, total)
            logits = self.forward(int(t), pos)
            pos += 1
        ids, margins = [], []
        for i in range(n_gen):
            nxt = int(L.ref_argmax(logits.ctypes.data, logits.size))
            top = np.sort(logits)[-2:]
            ids.append(nxt)
            margins.append(float(top[1] - top[0]))
            if i + 1 < n_gen:
                if progress:
                    progress(pos - start_pos, total)
                logits = self.forward(nxt, pos)
                pos += 1
        return np.array(ids, np.uint32), np.array(margins), logits
