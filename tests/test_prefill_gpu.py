"""GPU parity of the tensor-core prefill dequant-GEMM (Q4_K, Q6_K, Q8_0;
batches of at least 16 tokens) against the CPU oracle, through the C ABI.

The oracle is the restatement of go-infer's per-token prefill semantics
(MatMulBatch declining, pkg/engine/forward.go:482-495: one GEMVEngine.MatMul
per token, pkg/math/gemv.go:134-167).  Small and ragged shapes are checked on
every element; the config-3 shapes (512 tokens x 4096 columns, N = 4096 /
11008 Q4_K and 32000 Q6_K) on a sample of tokens against the oracle and on
every element against the decode GEMV, which the decode tests pin to the
oracle.  Raw-block tests feed random bytes (every 6-bit scale/min pattern,
int8 scales down to -128) to cover blocks no quantiser would emit.
"""
import numpy as np
import pytest

import goinfer_cuda as G
import oracle as O
from _util import assert_parity, rel_err, seeded_weights

pytestmark = pytest.mark.gpu

TC_MIN_BATCH = 16  # kGemmTcMinBatch in go-infer_b200/csrc/gemm.cuh


@pytest.fixture(scope="module", autouse=True)
def cuda():
    G.Init(0)
    assert G.IsAvailable()
    yield


@pytest.fixture(params=[True, False], ids=["pair", "single"], autouse=True)
def launch_shape(request):
    """Every test on both launch shapes of the tensor-core GEMM: single CTAs
    (the default) and CTA pairs (clusters of two, 256-row cta_group::2 MMAs)."""
    G.set_prefill_pair(request.param)
    yield request.param
    G.set_prefill_pair(False)


def gpu_gemm(qt, raw, x, batch, rows, cols):
    buf = G.CreateBuffer(raw)
    try:
        y = np.full(batch * rows, np.nan, np.float32)
        G.MatMulBatchBuf(qt, y, np.ascontiguousarray(x, np.float32).reshape(-1), buf, batch, rows, cols)
        return y.reshape(batch, rows)
    finally:
        G.ReleaseBuffer(buf)


def gpu_gemv_rows(qt, raw, x, rows, cols):
    """Every token through the decode GEMV (one call per token)."""
    buf = G.CreateBuffer(raw)
    try:
        out = np.empty((x.shape[0], rows), np.float32)
        for b in range(x.shape[0]):
            G.MatMulBuf(qt, out[b], np.ascontiguousarray(x[b]), buf, rows, cols)
        return out
    finally:
        G.ReleaseBuffer(buf)


def exact_rows(qt, raw, x, rows, cols):
    """float64 product of the dequantised weights (the conditioning yardstick)."""
    w = O.dequantize(qt, raw, rows * cols).reshape(rows, cols).astype(np.float64)
    return x.astype(np.float64) @ w.T


def check_against_oracle(qt, raw, x, y, rows, cols, what):
    ref = O.matmul_batch(qt, x, raw, x.shape[0], rows, cols).reshape(x.shape[0], rows)
    assert_parity(y.reshape(-1), ref.reshape(-1), what=what)
    # At least as close to the float64 product as the reference itself.
    exact = exact_rows(qt, raw, x, rows, cols)
    scale = np.abs(exact).max() + 1e-30
    gpu_dev = np.abs(y - exact).max()
    ref_dev = np.abs(ref - exact).max()
    assert gpu_dev <= 4 * ref_dev + 1e-6 * scale, f"{what}: |gpu-exact| {gpu_dev:.3e} vs |ref-exact| {ref_dev:.3e}"


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
@pytest.mark.parametrize("batch,rows,cols", [
    (16, 128, 256),     # one tile, one super-block
    (17, 130, 512),     # ragged tokens and rows
    (130, 200, 1024),   # two token tiles, two row tiles
    (256, 384, 4096),   # full tiles, config-3 width
    (300, 77, 2304),    # nine super-blocks: Q6_K rows alternate 2-byte alignment
])
def test_tc_shapes_match_oracle(qt, batch, rows, cols):
    raw = G.quantize(qt, seeded_weights(1000 + rows, rows, cols))
    x = np.random.default_rng(2000 + batch).normal(size=(batch, cols)).astype(np.float32)
    y = gpu_gemm(qt, raw, x, batch, rows, cols)
    check_against_oracle(qt, raw, x, y, rows, cols, f"tc {qt} {batch}x{rows}x{cols}")


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_tc_pair_agrees_with_single(qt, launch_shape):
    """The two launch shapes sum the same products in the same K order: the
    results agree to float32 rounding (an odd row-tile count included)."""
    if not launch_shape:
        pytest.skip("compares the two shapes once")
    batch, rows, cols = 200, 3 * 128 + 5, 1536
    raw = G.quantize(qt, seeded_weights(41, rows, cols))
    x = np.random.default_rng(42).normal(size=(batch, cols)).astype(np.float32)
    y_pair = gpu_gemm(qt, raw, x, batch, rows, cols)
    G.set_prefill_pair(False)
    y_single = gpu_gemm(qt, raw, x, batch, rows, cols)
    diff = np.abs(y_pair - y_single).max() / (np.abs(y_single).max() + 1e-30)
    print(f"pair vs single: max |diff| / max |y| = {diff:.3e}, identical: {np.array_equal(y_pair, y_single)}")
    assert diff <= 1e-6


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_tc_threshold_agrees_with_per_token_path(qt):
    """batch 15 runs per token, batch 16 on the tensor cores: same answers."""
    rows, cols = 96, 768
    raw = G.quantize(qt, seeded_weights(31, rows, cols))
    x = np.random.default_rng(32).normal(size=(TC_MIN_BATCH, cols)).astype(np.float32)
    y16 = gpu_gemm(qt, raw, x, TC_MIN_BATCH, rows, cols)
    y15 = gpu_gemm(qt, raw, x[:15], 15, rows, cols)
    assert_parity(y16[:15].reshape(-1), y15.reshape(-1), what="tc vs per-token")
    check_against_oracle(qt, raw, x, y16, rows, cols, "tc at threshold")


def random_q4k_blocks(rng, rows, nsb):
    raw = rng.integers(0, 256, size=(rows, nsb, 144), dtype=np.uint8)
    d = rng.uniform(1e-4, 2e-2, size=(rows, nsb)).astype(np.float16)
    dmin = rng.uniform(0.0, 2e-2, size=(rows, nsb)).astype(np.float16)
    raw[:, :, 0:2] = d.view(np.uint8).reshape(rows, nsb, 2)
    raw[:, :, 2:4] = dmin.view(np.uint8).reshape(rows, nsb, 2)
    return raw.reshape(-1)


def random_q6k_blocks(rng, rows, nsb):
    raw = rng.integers(0, 256, size=(rows, nsb, 210), dtype=np.uint8)
    raw[:, :, 192] = 0x80  # one int8 scale of -128 per block
    d = rng.uniform(1e-5, 1e-3, size=(rows, nsb)).astype(np.float16)
    raw[:, :, 208:210] = d.view(np.uint8).reshape(rows, nsb, 2)
    return raw.reshape(-1)


def random_q80_blocks(rng, rows, nsb):
    """Random int8 quants; fp16 scales spread over six decades, so blocks of
    one 256-column group carry very different d (the kernel folds d into the
    weight operand under one power of two per group)."""
    raw = rng.integers(0, 256, size=(rows, nsb * 8, 34), dtype=np.uint8)
    d = (10.0 ** rng.uniform(-7, -1, size=(rows, nsb * 8))).astype(np.float16)
    d[:, ::5] = 0  # some all-zero blocks
    raw[:, :, 0:2] = d.view(np.uint8).reshape(rows, nsb * 8, 2)
    return raw.reshape(-1)


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_tc_random_raw_blocks(qt):
    rng = np.random.default_rng(44)
    batch, rows, cols = 48, 160, 1536
    make = {G.TYPE_Q4_K: random_q4k_blocks, G.TYPE_Q6_K: random_q6k_blocks, G.TYPE_Q8_0: random_q80_blocks}[qt]
    raw = make(rng, rows, cols // 256)
    x = rng.normal(size=(batch, cols)).astype(np.float32)
    y = gpu_gemm(qt, raw, x, batch, rows, cols)
    check_against_oracle(qt, raw, x, y, rows, cols, f"raw blocks {qt}")


def test_tc_q6k_extreme_products():
    """sc = -128 with q = -32 gives 4096; sc = 127 with q = 31 gives 3937,
    which fp16 cannot hold: the hi/lo weight split must carry it exactly."""
    rows, cols, batch = 128, 512, 32
    raw = np.zeros((rows, 2, 210), np.uint8)
    rng = np.random.default_rng(5)
    for r in range(rows):
        for sb in range(2):
            q6 = rng.choice([0, 63, 1, 62], size=256)  # q = -32, 31, -31, 30
            blk = raw[r, sb]
            for h in range(2):
                for l in range(32):
                    v = [q6[128 * h + l + 32 * k] for k in range(4)]
                    blk[64 * h + l] = (v[0] & 15) | ((v[2] & 15) << 4)
                    blk[64 * h + 32 + l] = (v[1] & 15) | ((v[3] & 15) << 4)
                    blk[128 + 32 * h + l] = (v[0] >> 4) | ((v[1] >> 4) << 2) | ((v[2] >> 4) << 4) | ((v[3] >> 4) << 6)
            blk[192:208] = rng.choice([0x80, 0x7F, 0x81, 0x7E], size=16).astype(np.uint8)
            blk[208:210] = np.frombuffer(np.float16(1e-4).tobytes(), np.uint8)
    raw = raw.reshape(-1)
    x = rng.normal(size=(batch, cols)).astype(np.float32)
    y = gpu_gemm(G.TYPE_Q6_K, raw, x, batch, rows, cols)
    check_against_oracle(G.TYPE_Q6_K, raw, x, y, rows, cols, "q6k extreme products")


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_tc_activation_scaling_extremes(qt):
    """Per-token power-of-two scaling: tiny, huge and mixed-magnitude rows."""
    rows, cols, batch = 128, 1024, 24
    raw = G.quantize(qt, seeded_weights(61, rows, cols))
    rng = np.random.default_rng(62)
    x = rng.normal(size=(batch, cols)).astype(np.float32)
    x[0] *= np.float32(1e-30)
    x[1] *= np.float32(1e25)
    x[2, ::7] *= np.float32(1e-6)     # small elements beside normal ones
    x[3, 5] = np.float32(3e4)         # one dominant element
    x[4] = 0.0                        # all-zero token
    x[5] *= np.float32(1e-38)         # subnormal-adjacent
    y = gpu_gemm(qt, raw, x, batch, rows, cols)
    ref = O.matmul_batch(qt, x, raw, batch, rows, cols).reshape(batch, rows)
    for b in range(batch):
        assert_parity(y[b], ref[b], what=f"token {b}")


@pytest.mark.parametrize("qt,rows,seed", [
    (G.TYPE_Q4_K, 4096, 8), (G.TYPE_Q4_K, 11008, 9), (G.TYPE_Q6_K, 32000, 10),
    (G.TYPE_Q8_0, 4096, 1)])  # config 1's Q8_0 matrix as a 512-token prefill
def test_tc_config3_shapes(qt, rows, seed):
    """Config 3: X 512 x 4096 ~ N(0,1) (seed 7), W ~ N(0, 0.02) quantised."""
    batch, cols = 512, 4096
    raw = G.quantize(qt, seeded_weights(seed, rows, cols))
    x = np.random.default_rng(7).normal(size=(batch, cols)).astype(np.float32)
    y = gpu_gemm(qt, raw, x, batch, rows, cols)
    assert np.isfinite(y).all()
    # Every element against the decode GEMV (itself pinned to the oracle).
    yv = gpu_gemv_rows(qt, raw, x, rows, cols)
    e = rel_err(y.reshape(-1), yv.reshape(-1))
    assert e.max() <= 1e-3, f"tc vs gemv max rel {e.max():.3e}"
    # A sample of tokens from every token tile against the oracle itself.
    toks = np.array([0, 1, 127, 128, 255, 300, 384, 511])
    ref = O.matmul_batch(qt, x[toks], raw, len(toks), rows, cols).reshape(len(toks), rows)
    assert_parity(y[toks].reshape(-1), ref.reshape(-1), what="config-3 token sample")
    # Deterministic: a second run is bitwise identical.
    y2 = gpu_gemm(qt, raw, x, batch, rows, cols)
    assert np.array_equal(y, y2)
