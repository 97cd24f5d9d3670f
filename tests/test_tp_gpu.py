"""Tensor-parallel decode on 2+ GPUs: greedy ids of a 2-way (and, with more
GPUs, 4- and 8-way) split equal the single-GPU decode of the same model,
and are identical on every rank.  Each split runs tests/tp_worker.py under
torchrun (one process per GPU, 127.0.0.1 rendezvous)."""
import os
import subprocess
import sys

import numpy as np
import pytest

import goinfer_cuda as G
import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from tp_worker import CONFIGS  # noqa: E402


def run_split(world: int, tmp_path, port: int):
    out = str(tmp_path / f"tp{world}.npz")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "tp_worker.py"), "--out", out]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return np.load(out)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_greedy_matches_single_gpu(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = run_split(world, tmp_path, 29500 + world)
    assert bool(res["same_on_all_ranks"])
    G.Init(0)
    cfg = CONFIGS["small"]
    dev = synth.DeviceModel(synth.synth_model(cfg, 21))
    model = dev.model()
    try:
        ids, _l, _ms = model.generate(res["prompt"], len(res["ids"]))
    finally:
        model.close()
        dev.close()
    assert np.array_equal(ids, res["ids"]), f"tp{world} {res['ids']} vs 1-GPU {ids}"
