"""The library's host quantisers (gi_quantize), checked through the oracle.

Q8_0 must reproduce go-infer's QuantizeQ8_0 byte for byte; the Q4_K/Q6_K
fits (go-infer has none) must decode, through the reference dequantisers,
to within their format's step size of the input.
"""
import numpy as np
import pytest

import goinfer_cuda as G
import oracle as O
from _util import seeded_weights


def test_q8_0_matches_reference_quantiser_bytewise():
    w = seeded_weights(1, 64, 4096)
    ours = G.quantize(G.TYPE_Q8_0, w)
    ref = np.concatenate([O.quantize_q8_0(row) for row in w])
    assert np.array_equal(ours, ref)


def test_q8_0_edge_values():
    w = np.zeros((3, 64), np.float32)
    w[1, :] = 1e-30          # scale underflows the truncating fp16 -> all-zero block
    w[2, ::2] = 7.0
    w[2, 1::2] = -7.0
    ours = G.quantize(G.TYPE_Q8_0, w)
    ref = np.concatenate([O.quantize_q8_0(row) for row in w])
    assert np.array_equal(ours, ref)


@pytest.mark.parametrize("qt,bpb", [(G.TYPE_Q4_K, 144), (G.TYPE_Q6_K, 210)])
def test_k_quant_roundtrip(qt, bpb):
    rows, cols = 16, 1024
    w = seeded_weights(5, rows, cols)
    raw = G.quantize(qt, w)
    assert raw.size == rows * cols // 256 * bpb == rows * G.row_bytes(qt, cols)
    deq = O.dequantize(qt, raw, rows * cols).reshape(rows, cols)
    err = np.abs(deq - w)
    # Q4_K: 16 levels per 32-weight sub-block; Q6_K: 63 levels per 16
    step = (w.max() - w.min()) / (15 if qt == G.TYPE_Q4_K else 31)
    assert err.max() <= step
    rel = np.linalg.norm(deq - w) / np.linalg.norm(w)
    assert rel < (0.12 if qt == G.TYPE_Q4_K else 0.03)


def test_k_quant_constant_and_zero_blocks():
    w = np.zeros((2, 256), np.float32)
    w[1, :] = -0.5
    for qt in (G.TYPE_Q4_K, G.TYPE_Q6_K):
        deq = O.dequantize(qt, G.quantize(qt, w), 512).reshape(2, 256)
        assert np.all(deq[0] == 0)
        assert np.allclose(deq[1], -0.5, atol=0.02)


def test_quantize_rejects_bad_shapes():
    with pytest.raises(G.GoInferCudaError) as e:
        G.quantize(G.TYPE_Q4_K, np.zeros((2, 100), np.float32))
    assert e.value.code == G.ERR_SHAPE
    with pytest.raises(G.GoInferCudaError) as e:
        G.quantize(3, np.zeros((2, 256), np.float32))
    assert e.value.code == G.ERR_UNSUPPORTED_TYPE


def test_numpy_q4_k_restatement_matches_library_bytewise():
    """oracle/quantize_np.py (the reference arm's input preparation, which
    must not load the product library) gives the library's Q4_K bytes."""
    import quantize_np
    rng = np.random.default_rng(17)
    for rows, cols, std in ((64, 4096, 0.02), (300, 512, 3e4), (8, 256, 1e-6), (16, 1024, 1.0)):
        w = rng.normal(0, std, (rows, cols)).astype(np.float32)
        w[0, :32] = 0           # one all-zero sub-block
        w[1, :256] = 5.0        # constant positive block (offset -0)
        w[2, :256] = -1e-30     # scales underflow the truncating fp16
        w[3, :256] = 0          # all-zero block
        w[4, :256] = -2.0       # constant negative block
        assert np.array_equal(quantize_np.quantize_q4_k(w), G.quantize(G.TYPE_Q4_K, w))
