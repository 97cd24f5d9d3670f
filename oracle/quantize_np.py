"""numpy restatement of the library's Q4_K block quantiser.

TEST INFRASTRUCTURE ONLY.  bench.py's reference arm uses it to prepare the
Q4_K weights it times go-infer's CPU GEMV on, so that arm loads nothing of
the product library; tests/test_quantize.py checks it byte for byte
against the library's own quantiser (go-infer_b200/csrc/quantize.cu,
q4_k_block).

go-infer has no Q4_K quantiser; the block format is the one
DequantizeQ4_K decodes (pkg/quant/quant.go:215-253): fp16 d and dmin, 12
bytes of packed 6-bit sub-block scales and mins (getScaleMin,
quant.go:228-235), 128 bytes of nibbles (quant.go:237-249).  The fit: per
32-weight sub-block j, step_j = (max - min(0, min)) / 15 and off_j =
-min(0, min); d = max_j step_j / 63 and dmin = max_j off_j / 63, each
through the truncating FP32ToFP16 (pkg/quant/fp16.go:38-69); sc_j =
round(step_j / d), m_j = round(off_j / dmin), q = round((w + dmin*m_j) /
(d*sc_j)) clamped to [0, 15].  Every step is one float32 operation and
round() is round-half-away-from-zero (C roundf), computed in float64 where
the float32 input makes it exact.
"""
from __future__ import annotations

import numpy as np


def _f32_to_f16_trunc(v: np.ndarray) -> np.ndarray:
    """FP32ToFP16 by mantissa truncation (pkg/quant/fp16.go:38-69), elementwise."""
    bits = np.ascontiguousarray(v, np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    mant = bits & 0x7FFFFF
    out = sign | (np.clip(exp, 0, 31) << 10) | (mant >> 13)
    inf_nan = ((bits >> 23) & 0xFF) == 255
    out = np.where(inf_nan, sign | np.where(mant != 0, 0x7E00, 0x7C00), out)
    out = np.where(~inf_nan & (exp >= 31), sign | 0x7C00, out)
    sub_shift = np.clip(1 - exp, 0, 31)
    sub = sign | (((mant | 0x800000) >> sub_shift) >> 13)
    out = np.where(~inf_nan & (exp <= 0), np.where(exp < -10, sign, sub), out)
    return out.astype(np.uint16)


def _f16_to_f32(h: np.ndarray) -> np.ndarray:
    return h.astype(np.uint16).view(np.float16).astype(np.float32)


def _roundf(v: np.ndarray) -> np.ndarray:
    """C roundf (half away from zero) of float32 values, exact in float64."""
    a = v.astype(np.float64)
    return (np.sign(a) * np.floor(np.abs(a) + 0.5)).astype(np.float32)


def quantize_q4_k(w: np.ndarray, chunk_rows: int = 256) -> np.ndarray:
    """rows x cols float32 (cols a multiple of 256) -> the rows' Q4_K blocks,
    row after row, as one flat uint8 array (rows * cols/256 * 144 bytes).
    Row chunks run on a thread pool (numpy releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    import os
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    assert cols % 256 == 0
    out = np.empty(rows * (cols // 256) * 144, np.uint8).reshape(rows, -1)

    def work(r0):
        out[r0:r0 + chunk_rows] = _q4_k_rows(w[r0:r0 + chunk_rows]).reshape(-1, out.shape[1])

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        list(ex.map(work, range(0, rows, chunk_rows)))
    return out.reshape(-1)


def _q4_k_rows(w: np.ndarray) -> np.ndarray:
    f = np.float32
    b = w.reshape(-1, 8, 32)
    lo = np.minimum(b.min(axis=2), f(0))
    hi = b.max(axis=2)
    step = (hi - lo) / f(15)
    off = -lo
    # the largest step / offset, starting from +0 as the C loop does (an
    # all-zero sub-block's offset is -0 and must not reach the fp16 sign)
    max_step = np.where(step.max(axis=1) > 0, step.max(axis=1), f(0))
    max_off = np.where(off.max(axis=1) > 0, off.max(axis=1), f(0))
    dh = _f32_to_f16_trunc(max_step / f(63))
    mh = _f32_to_f16_trunc(max_off / f(63))
    d, dmin = _f16_to_f32(dh)[:, None], _f16_to_f32(mh)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d > 0, np.clip(_roundf(step / d), f(0), f(63)), f(0)).astype(np.uint8)
        mn = np.where(dmin > 0, np.clip(_roundf(off / dmin), f(0), f(63)), f(0)).astype(np.uint8)
        ds = (d * sc.astype(f))[:, :, None]
        dm = (dmin * mn.astype(f))[:, :, None]
        # q is clamped to [0, 15], so roundf's negative half never matters:
        # floor(t + 0.5) of the float32 quotient, exact in float64
        t = ((b + dm) / ds).astype(np.float64)
        t += 0.5
        np.floor(t, out=t)
        np.clip(t, 0, 15, out=t)
        t[np.broadcast_to(~(ds > 0), t.shape)] = 0
        q = t.astype(np.uint8)
    out = np.empty((b.shape[0], 144), np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = mh.view(np.uint8).reshape(-1, 2)
    out[:, 4:8] = (sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)
    out[:, 8:12] = (mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)
    out[:, 12:16] = (sc[:, 4:] & 0xF) | ((mn[:, 4:] & 0xF) << 4)
    q = q.reshape(-1, 4, 2, 32)  # (block, chunk c, low/high half, l)
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(-1, 128)
    return out.reshape(-1)
