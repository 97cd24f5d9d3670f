"""GPU parity of the decode GEMV against the CPU oracle, through the C ABI.

Every case feeds the same raw GGUF bytes and fp32 activations to the CUDA
library and to the restatement of go-infer's GEMVEngine.MatMul*
(oracle/goinfer_ref.c) and requires per-element relative error <= 1e-3
(denominator floored at 1e-2 * rms(ref), see tests/_util.py).  The tests
mirror the reference's own GPU tests (pkg/metal/metal_test.go) where those
exist.
"""
import struct

import numpy as np
import pytest

import goinfer_cuda as G
import oracle as O
from _util import GOLDEN, assert_parity, rel_err, seeded_weights, seeded_x

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def cuda():
    G.Init(0)
    assert G.IsAvailable()
    yield


def gpu_gemv(qt, raw, x, rows, cols):
    buf = G.CreateBuffer(raw)
    try:
        y = np.full(rows, np.nan, np.float32)
        G.MatMulBuf(qt, y, np.ascontiguousarray(x, np.float32), buf, rows, cols)
        return y
    finally:
        G.ReleaseBuffer(buf)


def f16(v):
    return O.fp32_to_fp16(float(v))


# ---------------------------------------------- reference GPU tests, mirrored

def test_metal_gemv_q4_k_kat():
    # pkg/metal/metal_test.go:127-164
    raw = bytearray()
    for _ in range(2):
        raw += struct.pack("<HH", f16(1.0), f16(0.0)) + bytes([1] * 12) + bytes([0x22] * 128)
    y = np.zeros(2, np.float32)
    G.MatMulQ4_K(y, np.ones(256, np.float32), bytes(raw), 2, 256)
    assert np.all(np.abs(y - 512.0) <= 1e-2)


def test_metal_gemv_q8_0_kat():
    # pkg/metal/metal_test.go:91-125
    raw = bytearray()
    for _ in range(4):
        raw += struct.pack("<H", f16(0.25)) + bytes([4] * 32)
    y = np.zeros(4, np.float32)
    G.MatMulQ8_0(y, np.ones(32, np.float32), bytes(raw), 4, 32)
    assert np.all(np.abs(y - 32.0) <= 1e-3)


def test_q8_0_fused_dot_kat_through_gpu():
    # pkg/quant/quant_test.go:55-83 on the GPU: 1 row, 2 blocks
    raw = bytearray()
    for _ in range(2):
        raw += struct.pack("<H", f16(0.5)) + bytes((j - 16) & 0xFF for j in range(32))
    x = np.arange(1, 65, dtype=np.float32)
    y = np.zeros(1, np.float32)
    G.MatMulQ8_0(y, x, bytes(raw), 1, 64)
    ref = O.dot_vec(O.GGML_Q8_0, x, np.frombuffer(bytes(raw), np.uint8), 64)
    assert abs(y[0] - ref) <= 1e-4 * max(1.0, abs(ref))


# ------------------------------------------------------------ golden vectors

def test_golden_vectors():
    g = np.load(f"{GOLDEN}/gemv_golden.npz")
    for name in sorted({k.split("__")[0] for k in g.files}):
        qt, rows, cols = (int(v) for v in g[name + "__shape"])
        y = gpu_gemv(qt, g[name + "__w"], g[name + "__x"], rows, cols)
        assert_parity(y, g[name + "__y"], what=name)


# ------------------------------------------------ seeded parity, config shapes

CONFIG_SHAPES = [
    ("config1 Q8_0 4096x4096", G.TYPE_Q8_0, 4096, 4096, 1, 2),
    ("config2 Q4_K gate 11008x4096", G.TYPE_Q4_K, 11008, 4096, 3, 4),
    ("config2 Q4_K down 4096x11008", G.TYPE_Q4_K, 4096, 11008, 5, 6),
    ("lm_head Q6_K 32000x4096", G.TYPE_Q6_K, 32000, 4096, 10, 11),
]


@pytest.mark.parametrize("what,qt,rows,cols,ws,xs", CONFIG_SHAPES, ids=[c[0] for c in CONFIG_SHAPES])
def test_config_shapes_match_oracle(what, qt, rows, cols, ws, xs):
    w = seeded_weights(ws, rows, cols)
    raw = G.quantize(qt, w)
    x = seeded_x(xs, cols)
    y = gpu_gemv(qt, raw, x, rows, cols)
    ref = O.matmul(qt, x, raw, rows, cols)
    assert_parity(y, ref, what=what, absdot=O.matmul_absdot(qt, x, raw, rows, cols))
    # the GPU sits as close to the exact product as the reference itself does
    exact = O.matmul_f64(qt, x, raw, rows, cols)
    scale = np.sqrt(np.mean(exact ** 2))
    assert np.max(np.abs(y - exact)) <= 4 * np.max(np.abs(ref - exact)) + 1e-6 * scale


@pytest.mark.parametrize("rows,cols", [(32000, 4096), (1000, 2048), (17, 8192), (3, 2048), (4100, 2048),
                                       (160, 45056)])
def test_q6k_tensor_core_kernel_matches_oracle(rows, cols):
    """The Q6_K GEMV on the int8 tensor cores (the default for rows of whole
    2048-column groups; gi_cuda_set_q6k_mma) against DotVecQ6_K (quant.go:256-291, 542-545):
    the lm_head shape, ragged row counts and a row too long to stage."""
    raw = G.quantize_seeded(G.TYPE_Q6_K, 600 + rows, 0.02, rows, cols)
    x = seeded_x(rows + 3, cols)
    x[::131] *= 40  # activation outliers
    G.set_q6k_mma(True)  # the default
    y = gpu_gemv(G.TYPE_Q6_K, raw, x, rows, cols)
    again = gpu_gemv(G.TYPE_Q6_K, raw, x, rows, cols)
    ref = O.matmul(G.TYPE_Q6_K, x, raw, rows, cols)
    assert_parity(y, ref, what=f"q6k mma {rows}x{cols}", absdot=O.matmul_absdot(G.TYPE_Q6_K, x, raw, rows, cols))
    assert np.array_equal(y.view(np.uint32), again.view(np.uint32))
    exact = O.matmul_f64(G.TYPE_Q6_K, x, raw, rows, cols)
    scale = np.sqrt(np.mean(exact ** 2))
    assert np.max(np.abs(y - exact)) <= 4 * np.max(np.abs(ref - exact)) + 1e-6 * scale


def test_q6k_tensor_core_kernel_70b_head_rows():
    """The 128256 x 8192 head shape on the Q6_K tensor-core kernel: every row
    against the CPU-core kernel's, a row sample against the oracle."""
    rows, cols = 128256, 8192
    raw = G.quantize_seeded(G.TYPE_Q6_K, 77, 0.02, rows, cols)
    x = seeded_x(78, cols)
    buf = G.CreateBuffer(raw)
    try:
        y_mma, y_core = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
        G.MatMulBuf(G.TYPE_Q6_K, y_mma, x, buf, rows, cols)
        G.set_q6k_mma(False)  # the CUDA-core kernel
        try:
            G.MatMulBuf(G.TYPE_Q6_K, y_core, x, buf, rows, cols)
        finally:
            G.set_q6k_mma(True)
    finally:
        G.ReleaseBuffer(buf)
    assert_parity(y_mma, y_core.astype(np.float64), what="q6k mma vs cuda-core kernel")
    pick = np.sort(np.random.default_rng(79).choice(rows, 512, replace=False))
    rb = G.row_bytes(G.TYPE_Q6_K, cols)
    sub = np.concatenate([raw[r * rb:(r + 1) * rb] for r in pick])
    assert_parity(y_mma[pick], O.matmul(G.TYPE_Q6_K, x, sub, len(pick), cols), what="q6k mma head rows")


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 256), (17, 256), (33, 512), (16, 4096), (100, 1280), (3, 11008),
                                       (4100, 256)])  # many short rows: 8 warps, 3 ring stages
def test_small_and_ragged_shapes(qt, rows, cols):
    w = seeded_weights(rows * 7 + cols, rows, cols)
    raw = G.quantize(qt, w)
    x = seeded_x(cols + 1, cols)
    y = gpu_gemv(qt, raw, x, rows, cols)
    assert_parity(y, O.matmul(qt, x, raw, rows, cols), what=f"{qt} {rows}x{cols}")


@pytest.mark.parametrize("rows,cols", [(32, 96), (7, 160), (50, 32)])
def test_q8_0_rows_not_16_byte_aligned(rows, cols):
    w = seeded_weights(rows + cols, rows, cols)
    raw = G.quantize(G.TYPE_Q8_0, w)
    x = seeded_x(3, cols)
    y = gpu_gemv(G.TYPE_Q8_0, raw, x, rows, cols)
    assert_parity(y, O.matmul(G.TYPE_Q8_0, x, raw, rows, cols))


def test_70b_shapes_on_row_samples():
    # 70B-shaped projections (d=8192, FFN 28672): check a random row subset
    # against the oracle, and linearity of the whole output.
    rng = np.random.default_rng(12)
    for rows, cols in [(28672, 8192), (8192, 28672)]:
        w = seeded_weights(rows + 1, rows, cols)
        raw = G.quantize(G.TYPE_Q4_K, w)
        rb = G.row_bytes(G.TYPE_Q4_K, cols)
        x1, x2 = seeded_x(20, cols), seeded_x(21, cols)
        buf = G.CreateBuffer(raw)
        y1, y2, y12 = (np.zeros(rows, np.float32) for _ in range(3))
        G.MatMulBuf(G.TYPE_Q4_K, y1, x1, buf, rows, cols)
        G.MatMulBuf(G.TYPE_Q4_K, y2, x2, buf, rows, cols)
        G.MatMulBuf(G.TYPE_Q4_K, y12, x1 + x2, buf, rows, cols)
        G.ReleaseBuffer(buf)
        pick = np.sort(rng.choice(rows, 256, replace=False))
        sub = np.concatenate([raw[r * rb:(r + 1) * rb] for r in pick])
        assert_parity(y1[pick], O.matmul(G.TYPE_Q4_K, x1, sub, len(pick), cols))
        assert np.max(rel_err(y12, (y1.astype(np.float64) + y2))) < 1e-3


def test_activation_scaling_extremes():
    rows, cols = 64, 4096
    raw = G.quantize(G.TYPE_Q4_K, seeded_weights(30, rows, cols))
    for mag in (1e-30, 1e-6, 1.0, 3e3, 1e7):
        x = seeded_x(31, cols) * np.float32(mag)
        x[::97] *= 50  # outliers, as LLM activations have
        y = gpu_gemv(G.TYPE_Q4_K, raw, x, rows, cols)
        assert_parity(y, O.matmul(G.TYPE_Q4_K, x, raw, rows, cols), what=f"|x|~{mag}")
    y = gpu_gemv(G.TYPE_Q4_K, raw, np.zeros(cols, np.float32), rows, cols)
    assert np.all(y == 0)


def test_deterministic_and_device_path_identical():
    import torch
    rows, cols = 4096, 11008
    raw = G.quantize(G.TYPE_Q4_K, seeded_weights(5, rows, cols))
    x = seeded_x(6, cols)
    a = gpu_gemv(G.TYPE_Q4_K, raw, x, rows, cols)
    b = gpu_gemv(G.TYPE_Q4_K, raw, x, rows, cols)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    wd = torch.from_numpy(raw).cuda()
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for pdl in (False, True):
        G.set_pdl(pdl)
        G.gemv_dev(G.TYPE_Q4_K, yd.data_ptr(), xd.data_ptr(), wd.data_ptr(), raw.size, rows, cols, s)
        torch.cuda.synchronize()
        assert np.array_equal(yd.cpu().numpy().view(np.uint32), a.view(np.uint32))
    G.set_pdl(False)


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_multi_matrix_gemv_matches_single(qt):
    import torch
    cols = 4096
    shapes = [4096, 1024, 1040]  # Q, K, V of a GQA layer; the last one ragged
    raws = [G.quantize(qt, seeded_weights(80 + i, r, cols)) for i, r in enumerate(shapes)]
    x = seeded_x(83, cols)
    ws = [torch.from_numpy(r).cuda() for r in raws]
    xd = torch.from_numpy(x).cuda()
    ys = [torch.full((r,), float("nan"), device="cuda") for r in shapes]
    s = torch.cuda.current_stream().cuda_stream
    G.gemv_multi_dev(qt, [y.data_ptr() for y in ys], xd.data_ptr(), [w.data_ptr() for w in ws],
                     [r.size for r in raws], shapes, cols, s)
    torch.cuda.synchronize()
    for raw, y, r in zip(raws, ys, shapes):
        assert_parity(y.cpu().numpy(), O.matmul(qt, x, raw, r, cols), what=f"multi {qt} {r}")
        # A launch's CTA and warp split depends on the rows it holds, so the
        # float32 order of a row's partial sums (not the result's accuracy)
        # can differ between the 3-matrix launch and a single one.
        single = gpu_gemv(qt, raw, x, r, cols)
        assert_parity(y.cpu().numpy(), single.astype(np.float64), what=f"multi vs single {qt} {r}")
    # the same launch twice: bit-identical
    ys2 = [torch.empty(r, device="cuda") for r in shapes]
    G.gemv_multi_dev(qt, [y.data_ptr() for y in ys2], xd.data_ptr(), [w.data_ptr() for w in ws],
                     [r.size for r in raws], shapes, cols, s)
    torch.cuda.synchronize()
    for y, y2 in zip(ys, ys2):
        assert np.array_equal(y.cpu().numpy().view(np.uint32), y2.cpu().numpy().view(np.uint32))


def test_batch_mode_defers_outputs():
    rows, cols = 256, 1024
    raws = [G.quantize(qt, seeded_weights(40 + i, rows, cols)) for i, qt in
            enumerate((G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0))]
    bufs = [G.CreateBuffer(r) for r in raws]
    xs = [seeded_x(50 + i, cols) for i in range(3)]
    ys = [np.zeros(rows, np.float32) for _ in range(3)]
    G.BeginBatch()
    for qt, buf, x, y in zip((G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0), bufs, xs, ys):
        G.MatMulBuf(qt, y, x, buf, rows, cols)
    G.EndBatch()
    for qt, raw, x, y in zip((G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0), raws, xs, ys):
        assert_parity(y, O.matmul(qt, x, raw, rows, cols))
    for b in bufs:
        G.ReleaseBuffer(b)


def test_weights_dispatch_mirror():
    ws = G.Weights()
    raw = G.quantize(G.TYPE_Q4_K, seeded_weights(60, 512, 4096))
    ws.add("blk.0.ffn_gate.weight", G.TYPE_Q4_K, 512, 4096, raw)
    x = seeded_x(61, 4096)
    y = np.zeros(512, np.float32)
    ws.MatMul(y, x, "blk.0.ffn_gate.weight", 512, 4096)
    assert_parity(y, O.matmul(G.TYPE_Q4_K, x, raw, 512, 4096))
    ws.Close()


def test_error_codes():
    raw = np.zeros(16 * 144, np.uint8)
    buf = G.CreateBuffer(raw)
    y = np.zeros(16, np.float32)
    with pytest.raises(G.GoInferCudaError) as e:
        G.MatMulBuf(G.TYPE_Q4_K, y, np.zeros(200, np.float32), buf, 16, 200)  # cols % 256 != 0
    assert e.value.code == G.ERR_SHAPE
    with pytest.raises(G.GoInferCudaError) as e:
        G.MatMulBuf(3, y, np.zeros(256, np.float32), buf, 16, 256)  # not a supported type
    assert e.value.code == G.ERR_UNSUPPORTED_TYPE
    with pytest.raises(G.GoInferCudaError) as e:
        G.MatMulBuf(G.TYPE_Q4_K, np.zeros(32, np.float32), np.zeros(256, np.float32), buf, 32, 256)
    assert e.value.code == G.ERR_SHAPE  # buffer too small for 32 rows
    G.ReleaseBuffer(buf)


def test_prefill_batch_matches_per_token_oracle():
    batch, rows, cols = 5, 96, 512
    for qt in (G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0):
        raw = G.quantize(qt, seeded_weights(70, rows, cols))
        x = np.random.default_rng(71).normal(size=(batch, cols)).astype(np.float32)
        buf = G.CreateBuffer(raw)
        y = np.zeros(batch * rows, np.float32)
        G.MatMulBatchBuf(qt, y, x.reshape(-1), buf, batch, rows, cols)
        G.ReleaseBuffer(buf)
        ref = O.matmul_batch(qt, x, raw, batch, rows, cols)
        assert_parity(y, ref.reshape(-1), what=f"batch {qt}")


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0])
def test_pinned_host_output_written_directly(qt):
    """A page-locked, device-mapped y is written by the kernel itself (no
    device-to-host copy); the results are bit-identical to the copied ones
    (batch 1, per-token batch 3, tensor-core batch 16)."""
    import torch
    rows, cols = 1000, 2048
    raw = G.quantize(qt, seeded_weights(90, rows, cols))
    x = seeded_x(91, cols)
    buf = G.CreateBuffer(raw)
    try:
        y_page = np.full(rows, np.nan, np.float32)
        G.MatMulBuf(qt, y_page, x, buf, rows, cols)
        y_pin = torch.full((rows,), float("nan")).pin_memory().numpy()
        x_pin = torch.from_numpy(x).pin_memory().numpy()
        G.MatMulBuf(qt, y_pin, x_pin, buf, rows, cols)
        assert np.array_equal(y_pin.view(np.uint32), y_page.view(np.uint32))
        assert_parity(y_pin, O.matmul(qt, x, raw, rows, cols), what=f"pinned {qt}")
        for nb in (3, 16):  # per-token GEMVs, then the tensor-core prefill
            xb = np.stack([seeded_x(92 + b, cols) for b in range(nb)])
            yb_page = np.zeros(nb * rows, np.float32)
            G.MatMulBatchBuf(qt, yb_page, xb.reshape(-1), buf, nb, rows, cols)
            yb_pin = torch.zeros(nb * rows).pin_memory().numpy()
            G.MatMulBatchBuf(qt, yb_pin, torch.from_numpy(xb.reshape(-1)).pin_memory().numpy(), buf, nb, rows, cols)
            assert np.array_equal(yb_pin.view(np.uint32), yb_page.view(np.uint32)), f"batch {nb}"
    finally:
        G.ReleaseBuffer(buf)


@pytest.mark.parametrize("batch", [1, 3, 16])
def test_fused_gate_up_swiglu_matches_oracle(batch):
    """gi_cuda_gemm_fused_gate_up_buf (metal_gemm_fused_gate_up_buf,
    metal_bridge.h:51): y[b*rows + r] = silu(G x_b)[r] * (U x_b)[r], the
    SwiGLU of kernels.go:39-46; one fused GEMV for a single token, the
    prefill GEMMs for a batch; Q4_K only (-2 otherwise, as the reference)."""
    rows, cols = 100, 512
    graw = G.quantize(G.TYPE_Q4_K, seeded_weights(51, rows, cols))
    uraw = G.quantize(G.TYPE_Q4_K, seeded_weights(52, rows, cols))
    x = np.stack([seeded_x(60 + b, cols) for b in range(batch)])
    gb, ub = G.CreateBuffer(graw), G.CreateBuffer(uraw)
    try:
        y = np.full(batch * rows, np.nan, np.float32)
        G.MatMulFusedGateUpBatchBuf(G.TYPE_Q4_K, y, x.reshape(-1), gb, ub, batch, rows, cols)
        for b in range(batch):
            want = O.swiglu(O.matmul(G.TYPE_Q4_K, x[b], graw, rows, cols),
                            O.matmul(G.TYPE_Q4_K, x[b], uraw, rows, cols))
            assert_parity(y[b * rows:(b + 1) * rows], want, what=f"token {b}")
        with pytest.raises(G.GoInferCudaError) as e:
            G.MatMulFusedGateUpBatchBuf(G.TYPE_Q8_0, y, x.reshape(-1), gb, ub, batch, rows, cols)
        assert e.value.code == G.ERR_UNSUPPORTED_TYPE
    finally:
        G.ReleaseBuffer(gb)
        G.ReleaseBuffer(ub)


def ffn_oracle(x, norm, graw, uraw, draw, dim, hidden, eps):
    """Engine.Forward's FFN half (forward.go:275-287) through the oracle."""
    n = O.rmsnorm(x, norm, eps)
    hb = O.swiglu(O.matmul(G.TYPE_Q4_K, n, graw, hidden, dim), O.matmul(G.TYPE_Q4_K, n, uraw, hidden, dim))
    return (x + O.matmul(G.TYPE_Q4_K, hb, draw, dim, hidden)).astype(np.float32)


@pytest.mark.parametrize("dim,hidden", [(4096, 11008), (512, 1280)])
def test_ffn_block_matches_oracle(dim, hidden):
    """gi_cuda_ffn_buf / gi_cuda_ffn_dev on one GPU: RMSNorm, gate/up, SwiGLU,
    down and the residual add in two launches, against the oracle's steps."""
    import torch
    graw = G.quantize(G.TYPE_Q4_K, seeded_weights(110, hidden, dim))
    uraw = G.quantize(G.TYPE_Q4_K, seeded_weights(111, hidden, dim))
    draw = G.quantize(G.TYPE_Q4_K, seeded_weights(112, dim, hidden))
    norm = (1.0 + 0.1 * seeded_x(113, dim)).astype(np.float32)
    x0 = seeded_x(114, dim)
    want = ffn_oracle(x0, norm, graw, uraw, draw, dim, hidden, 1e-5)
    bufs = [G.CreateBuffer(a) for a in (norm, graw, uraw, draw)]
    try:
        x = x0.copy()
        G.FFNBuf(x, *bufs, dim, hidden, 1e-5)
        assert_parity(x, want, what=f"ffn {dim}x{hidden}")
        dev = [torch.from_numpy(a).cuda() for a in (norm, graw, uraw, draw)]
        xd = torch.from_numpy(x0).cuda()
        hd = torch.empty(hidden, device="cuda")
        G.ffn_dev(xd.data_ptr(), dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), dev[3].data_ptr(),
                  graw.size, uraw.size, draw.size, hd.data_ptr(), dim, hidden, 1e-5,
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert np.array_equal(xd.cpu().numpy().view(np.uint32), x.view(np.uint32))
        with pytest.raises(G.GoInferCudaError) as e:
            G.FFNBuf(x, bufs[0], bufs[1], bufs[2], bufs[3], dim, hidden + 100, 1e-5)
        assert e.value.code == G.ERR_SHAPE
    finally:
        for b in bufs:
            G.ReleaseBuffer(b)


@pytest.mark.parametrize("batch", [3, 16])
def test_batch_mode_chained_prefill_ffn(batch):
    """go-infer's prefill FFN inside one BeginBatch/EndBatch (forward.go:
    607-640): gate and up into host slices, SwiGLU on them, down reading
    the SwiGLU slice, the residual add reading the down slice -- every
    later call reads an earlier call's output through the host slice,
    which inside a batch still lives on the device (Metal's shared-memory
    contract).  The outputs equal the same calls made one by one, bit for
    bit, and the oracle's chain within the bar."""
    dim, hidden = 512, 1280
    graw = G.quantize(G.TYPE_Q4_K, seeded_weights(120, hidden, dim))
    uraw = G.quantize(G.TYPE_Q4_K, seeded_weights(121, hidden, dim))
    draw = G.quantize(G.TYPE_Q4_K, seeded_weights(122, dim, hidden))
    bufs = [G.CreateBuffer(r) for r in (graw, uraw, draw)]
    xs = np.random.default_rng(123).normal(size=(batch, dim)).astype(np.float32).reshape(-1)
    xn = np.random.default_rng(124).normal(size=(batch, dim)).astype(np.float32).reshape(-1)

    def chain(batched):
        x, g, u, d = xs.copy(), np.full(batch * hidden, np.nan, np.float32), \
            np.full(batch * hidden, np.nan, np.float32), np.full(batch * dim, np.nan, np.float32)
        if batched:
            G.BeginBatch()
        G.MatMulBatchBuf(G.TYPE_Q4_K, g, xn, bufs[0], batch, hidden, dim)
        G.MatMulBatchBuf(G.TYPE_Q4_K, u, xn, bufs[1], batch, hidden, dim)
        G.SwiGLU(g, u, batch * hidden)
        G.MatMulBatchBuf(G.TYPE_Q4_K, d, g, bufs[2], batch, dim, hidden)
        G.AddResidual(x, d, batch * dim)
        if batched:
            G.EndBatch()
        return x, g, d

    try:
        plain = chain(False)
        batched = chain(True)
    finally:
        for b in bufs:
            G.ReleaseBuffer(b)
    for a, b in zip(plain, batched):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for t in range(batch):
        n = xn[t * dim:(t + 1) * dim]
        h = O.swiglu(O.matmul(G.TYPE_Q4_K, n, graw, hidden, dim), O.matmul(G.TYPE_Q4_K, n, uraw, hidden, dim))
        want = (xs[t * dim:(t + 1) * dim] + O.matmul(G.TYPE_Q4_K, h, draw, dim, hidden)).astype(np.float32)
        assert_parity(batched[0][t * dim:(t + 1) * dim], want, what=f"batched chain token {t}")
