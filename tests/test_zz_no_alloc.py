"""gi_cuda_gemm_dev_noalloc against gi_cuda_gemm_dev, through the C ABI.

The no-alloc entry point runs the same kernels with its workspace in the
library's fixed device array, so on identical inputs two consecutive calls
must reproduce gi_cuda_gemm_dev bit for bit.  Kept in its own file, named to
be collected last, so it runs both alone and after every other test.
"""
import numpy as np
import pytest

import goinfer_cuda as G
from _util import seeded_weights

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def cuda():
    G.Init(0)
    assert G.IsAvailable()
    yield


def run(fn, qt, raw_dev, nbytes, x, batch, rows, cols, stream):
    y = torch.full((batch, rows), float("nan"), device="cuda:0")
    fn(qt, y.data_ptr(), x.data_ptr(), raw_dev.data_ptr(), nbytes, batch, rows, cols, stream.cuda_stream)
    stream.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("qt,batch,rows,cols", [
    (G.TYPE_Q4_K, 512, 4096, 4096),   # tensor-core path, config-3 width
    (G.TYPE_Q6_K, 200, 300, 2304),    # tensor-core path, ragged
    (G.TYPE_Q4_K, 8, 256, 1024),      # below the tensor-core batch: per-token GEMV
    (G.TYPE_Q8_0, 20, 96, 512),       # Q8_0 batches run per token
])
def test_noalloc_matches_gemm_dev(qt, batch, rows, cols):
    raw = G.quantize(qt, seeded_weights(900 + rows, rows, cols))
    raw_dev = torch.from_numpy(raw).to("cuda:0")
    x = torch.from_numpy(np.random.default_rng(901).normal(size=(batch, cols)).astype(np.float32)).to("cuda:0")
    stream = torch.cuda.Stream()
    ref = run(G.gemm_dev, qt, raw_dev, raw.nbytes, x, batch, rows, cols, stream)
    assert np.isfinite(ref).all()
    for _ in range(2):  # two consecutive calls on the same static scratch
        y = run(G.gemm_dev_noalloc, qt, raw_dev, raw.nbytes, x, batch, rows, cols, stream)
        assert np.array_equal(y, ref)


def test_noalloc_rejects_oversize_request():
    qt, batch, rows, cols = G.TYPE_Q4_K, 4096, 128, 4096  # ~67 MB of staged activations
    raw = G.quantize(qt, seeded_weights(902, rows, cols))
    raw_dev = torch.from_numpy(raw).to("cuda:0")
    x = torch.zeros((batch, cols), device="cuda:0")
    y = torch.zeros((batch, rows), device="cuda:0")
    with pytest.raises(G.GoInferCudaError) as e:
        G.gemm_dev_noalloc(qt, y.data_ptr(), x.data_ptr(), raw_dev.data_ptr(), raw.nbytes, batch, rows, cols)
    assert e.value.code == G.ERR_SHAPE
    assert "static buffer" in str(e.value)
