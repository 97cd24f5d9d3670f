"""Pins the CPU oracle (oracle/goinfer_ref.c) before anything is compared to it.

Three independent checks:
  1. the reference's own known-answer tests for this path, re-run against the
     oracle (pkg/quant/quant_test.go, pkg/metal/metal_test.go of go-infer);
  2. a second, pure-Python restatement of the same Go functions, written
     separately and compared bit for bit on random blocks;
  3. format properties (fp16 decode of all 65536 codes, truncation of
     FP32ToFP16, the committed golden vectors).
"""
import os
import struct

import numpy as np
import pytest

import oracle as O
from _util import GOLDEN, seeded_weights, seeded_x

F32 = np.float32


def f16(v):
    return O.fp32_to_fp16(float(v))


# ---------------------------------------------------------------- 1. KATs

def test_fp16_roundtrip_kat():
    # pkg/quant/quant_test.go:10-19
    for v in [0.0, 1.0, -1.0, 0.5, -0.5, 3.14159, 128.0, -0.001953125]:
        got = O.fp16_to_fp32(O.fp32_to_fp16(v))
        assert abs(got - np.float32(v)) <= 0.01 * abs(v) + 1e-4


def test_q8_0_dot_equals_dequant_dot_kat():
    # pkg/quant/quant_test.go:55-83: 2 blocks, scale 0.5, q = j-16, x = i+1
    x = np.arange(1, 65, dtype=np.float32)
    raw = bytearray()
    for _ in range(2):
        raw += struct.pack("<H", f16(0.5))
        raw += bytes((j - 16) & 0xFF for j in range(32))
    raw = np.frombuffer(bytes(raw), dtype=np.uint8)
    deq = O.dequantize(O.GGML_Q8_0, raw, 64)
    expected = F32(0)
    for i in range(64):
        expected = F32(expected + F32(x[i] * deq[i]))
    got = O.dot_vec(O.GGML_Q8_0, x, raw, 64)
    assert abs(got - float(expected)) <= 1e-4


def test_q8_0_quantize_roundtrip_kat():
    # pkg/quant/quant_test.go:129-143
    src = (np.arange(64) - 32).astype(np.float32)
    q = O.quantize_q8_0(src)
    deq = O.dequantize(O.GGML_Q8_0, q, 64)
    assert np.all(np.abs(src - deq) <= 0.5)


def _q4k_kat_bytes(rows):
    # pkg/metal/metal_test.go:127-164: d=1, dmin=0, every scale byte 1, qs=0x22
    raw = bytearray()
    for _ in range(rows):
        raw += struct.pack("<HH", f16(1.0), f16(0.0)) + bytes([1] * 12) + bytes([0x22] * 128)
    return np.frombuffer(bytes(raw), dtype=np.uint8)


def test_q4_k_gemv_kat():
    raw = _q4k_kat_bytes(2)
    y = O.matmul(O.GGML_Q4_K, np.ones(256, np.float32), raw, 2, 256)
    assert np.all(np.abs(y - 512.0) <= 1e-2)
    assert np.all(y == 512.0)  # exact: every weight dequantises to 2


def test_q8_0_gemv_kat():
    # pkg/metal/metal_test.go:91-125: 4x32, d=0.25, q=4, x=1 -> 32
    raw = bytearray()
    for _ in range(4):
        raw += struct.pack("<H", f16(0.25)) + bytes([4] * 32)
    y = O.matmul(O.GGML_Q8_0, np.ones(32, np.float32), np.frombuffer(bytes(raw), np.uint8), 4, 32)
    assert np.all(np.abs(y - 32.0) <= 1e-3)


# ------------------------------------- 2. independent Python restatement

def py_fp16(h):
    return np.array([h], dtype=np.uint16).view(np.float16).astype(np.float32)[0]


def py_dequant_q4_k(raw, n):
    # restated from pkg/quant/quant.go:215-253
    out = np.zeros(n, dtype=np.float32)
    for i in range(n // 256):
        blk = raw[144 * i:144 * (i + 1)]
        d = py_fp16(int(blk[0]) | int(blk[1]) << 8)
        dmin = py_fp16(int(blk[2]) | int(blk[3]) << 8)
        sc = [int(b) for b in blk[4:16]]
        qs = blk[16:144]

        def scale_min(j):
            if j < 4:
                return F32(F32(sc[j] & 63) * d), F32(F32(sc[j + 4] & 63) * dmin)
            s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4)
            m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)
            return F32(F32(s) * d), F32(F32(m) * dmin)

        for c in range(4):
            d1, m1 = scale_min(2 * c)
            d2, m2 = scale_min(2 * c + 1)
            for l in range(32):
                b = int(qs[32 * c + l])
                out[256 * i + 64 * c + l] = F32(F32(F32(b & 0xF) * d1) - m1)
                out[256 * i + 64 * c + 32 + l] = F32(F32(F32(b >> 4) * d2) - m2)
    return out


def py_dequant_q6_k(raw, n):
    # restated from pkg/quant/quant.go:256-291
    out = np.zeros(n, dtype=np.float32)
    for i in range(n // 256):
        blk = raw[210 * i:210 * (i + 1)]
        ql, qh, sc = blk[0:128], blk[128:192], blk[192:208]
        d = py_fp16(int(blk[208]) | int(blk[209]) << 8)
        for h in range(2):
            for l in range(32):
                a, b, c = int(ql[64 * h + l]), int(ql[64 * h + l + 32]), int(qh[32 * h + l])
                qv = [((a & 0xF) | ((c >> 0) & 3) << 4) - 32, ((b & 0xF) | ((c >> 2) & 3) << 4) - 32,
                      ((a >> 4) | ((c >> 4) & 3) << 4) - 32, ((b >> 4) | ((c >> 6) & 3) << 4) - 32]
                for k in range(4):
                    s = np.int8(np.uint8(sc[8 * h + l // 16 + 2 * k]))
                    out[256 * i + 128 * h + l + 32 * k] = F32(F32(d * F32(s)) * F32(qv[k]))
    return out


def py_dot_f32(x, w):
    # restated from pkg/quant/quant.go:548-566
    s = F32(0)
    n = len(x)
    i = 0
    while i <= n - 8:
        g = F32(x[i] * w[i])
        for k in range(1, 8):
            g = F32(g + F32(x[i + k] * w[i + k]))
        s = F32(s + g)
        i += 8
    while i < n:
        s = F32(s + F32(x[i] * w[i]))
        i += 1
    return s


def py_dot_q8_0(x, raw, n):
    # restated from pkg/quant/quant.go:320-339
    total = F32(0)
    for b in range(n // 32):
        d = py_fp16(int(raw[34 * b]) | int(raw[34 * b + 1]) << 8)
        bs = F32(0)
        for j in range(32):
            bs = F32(bs + F32(F32(np.int8(np.uint8(raw[34 * b + 2 + j]))) * x[32 * b + j]))
        total = F32(total + F32(bs * d))
    return total


def _random_blocks(rng, nblocks, size, fp16_offsets):
    raw = rng.integers(0, 256, size=nblocks * size, dtype=np.uint8)
    for b in range(nblocks):
        for off in fp16_offsets:  # keep the fp16 scales finite and moderate
            h = int(rng.integers(0x0400, 0x3C00))
            raw[b * size + off] = h & 0xFF
            raw[b * size + off + 1] = h >> 8
    return raw


def test_python_and_c_restatements_agree_bitwise():
    rng = np.random.default_rng(7)
    n = 512
    x = rng.normal(size=n).astype(np.float32)
    raw4 = _random_blocks(rng, n // 256, 144, (0, 2))
    raw6 = _random_blocks(rng, n // 256, 210, (208,))
    raw8 = _random_blocks(rng, n // 32, 34, (0,))
    d4 = O.dequantize(O.GGML_Q4_K, raw4, n)
    d6 = O.dequantize(O.GGML_Q6_K, raw6, n)
    assert np.array_equal(d4.view(np.uint32), py_dequant_q4_k(raw4, n).view(np.uint32))
    assert np.array_equal(d6.view(np.uint32), py_dequant_q6_k(raw6, n).view(np.uint32))
    assert np.float32(O.dot_vec(O.GGML_Q4_K, x, raw4, n)) == py_dot_f32(x, d4)
    assert np.float32(O.dot_vec(O.GGML_Q6_K, x, raw6, n)) == py_dot_f32(x, d6)
    assert np.float32(O.dot_vec(O.GGML_Q8_0, x, raw8, n)) == py_dot_q8_0(x, raw8, n)
    assert np.float32(O.dot_vec(O.GGML_F32, x, d4, n)) == py_dot_f32(x, d4)


def test_matmul_rows_equal_dot_vec_and_threads_do_not_matter():
    rng = np.random.default_rng(11)
    rows, cols = 37, 512
    raw = _random_blocks(rng, rows * cols // 256, 144, (0, 2))
    x = rng.normal(size=cols).astype(np.float32)
    y1 = O.matmul(O.GGML_Q4_K, x, raw, rows, cols, nthreads=1)
    y8 = O.matmul(O.GGML_Q4_K, x, raw, rows, cols, nthreads=8)
    assert np.array_equal(y1, y8)
    for r in (0, 5, 36):
        assert y1[r] == np.float32(O.dot_vec(O.GGML_Q4_K, x, raw[r * 288:(r + 1) * 288], cols))


# -------------------------------------------------- 3. format properties

def test_fp16_decode_all_codes_exact():
    codes = np.arange(65536, dtype=np.uint32)
    got = np.array([O.fp16_to_fp32(int(h)) for h in codes], dtype=np.float32)
    want = codes.astype(np.uint16).view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_fp32_to_fp16_truncates():
    rng = np.random.default_rng(3)
    vals = (rng.uniform(-1, 1, 2000) * 2.0 ** rng.integers(-13, 15, 2000)).astype(np.float32)
    for v in vals:
        h = O.fp32_to_fp16(float(v))
        back = abs(float(py_fp16(h)))
        nxt = float(np.nextafter(np.float16(back), np.float16(np.inf)))
        assert back <= abs(float(v)) < nxt  # largest magnitude not above |v|
        assert (h >> 15) == (1 if v < 0 else 0)


def test_golden_vectors_reproduce():
    path = os.path.join(GOLDEN, "gemv_golden.npz")
    g = np.load(path)
    for name in sorted({k.split("__")[0] for k in g.files}):
        qtype, rows, cols = (int(v) for v in g[name + "__shape"])
        y = O.matmul(qtype, g[name + "__x"], g[name + "__w"], rows, cols)
        assert np.array_equal(y.view(np.uint32), g[name + "__y"].view(np.uint32)), name


def test_seeded_inputs_are_stable():
    # the generator every test and bench.py use: PCG64 via default_rng
    w = seeded_weights(1, 2, 4)
    x = seeded_x(2, 4)
    assert w.dtype == np.float32 and x.dtype == np.float32
    assert np.array_equal(w, seeded_weights(1, 2, 4))
