"""Tensor-parallel decode on 2+ GPUs: the greedy ids of a 2-way (and, with
more GPUs, 4- and 8-way) split equal the CPU oracle's Engine.Forward on the
whole model and are identical on every rank, with the per-layer launches
and with the persistent decode-layer kernel; config 5 (the 70B shape) is
held to its oracle golden.  Each split runs tests/tp_worker.py under
torchrun (one process per GPU, 127.0.0.1 rendezvous)."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))
from tp_worker import CONFIGS  # noqa: E402


def run_split(world: int, tmp_path, port: int, extra=()):
    out = str(tmp_path / f"tp{world}.npz")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "tp_worker.py"), "--out", out, *extra]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return np.load(out)


@pytest.mark.parametrize("persistent", [False, True], ids=["per_layer", "persistent"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_greedy_matches_oracle(world, persistent, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = run_split(world, tmp_path, 29500 + 2 * world + persistent, ["--persistent"] if persistent else [])
    assert bool(res["same_on_all_ranks"])
    cfg = CONFIGS["small"]
    host = synth.synth_model(cfg, 21)
    want, margins, _l = O.RefModel(cfg, host.tensors).greedy(res["prompt"], len(res["ids"]))
    assert np.array_equal(res["ids"], want), \
        f"tp{world} {res['ids']} vs oracle {want} (smallest oracle top-2 margin {margins.min():.3e})"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_config5_matches_oracle_golden(world, tmp_path):
    """Config 5 (Llama-3-70B shape) split over `world` GPUs, weights drawn on
    the devices: 512-token prompt and 64 greedy steps, ids identical to the
    CPU oracle's golden."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import make_decode_golden as MG
    _cfg, seed, pseed, plen, steps, fname = MG.GOLDENS["70b"]
    path = os.path.join(HERE, "golden", fname)
    if not os.path.exists(path):
        pytest.skip(f"{fname} not generated (python tests/golden/make_decode_golden.py 70b)")
    gold = np.load(path)
    res = run_split(world, tmp_path, 29600 + world,
                    ["--config", "llama70b", "--device-synth", "--seed", str(seed), "--prompt", str(plen),
                     "--prompt-seed", str(pseed), "--gen", str(steps)])
    assert bool(res["same_on_all_ranks"])
    assert np.array_equal(res["prompt"], gold["prompt"])
    if not np.array_equal(res["ids"], gold["ids"]):
        i = int(np.argmax(res["ids"] != gold["ids"]))
        pytest.fail(f"tp{world} config-5 ids differ first at step {i}: {res['ids'][i]} vs oracle {gold['ids'][i]} "
                    f"(oracle top-2 margin {gold['margins'][i]:.3e})")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_ffn_block_matches_oracle(world, tmp_path):
    """gi_cuda_ffn_buf split over `world` GPUs (unequal hidden slices), three
    blocks in a row: every rank ends with the same x, which matches the
    oracle's FFN half of Engine.Forward on the whole matrices."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import goinfer_cuda as G
    from _util import assert_parity
    from tp_worker import FFN_SHAPE, ffn_weights
    res = run_split(world, tmp_path, 29700 + world, ["--ffn", "--seed", "31"])
    assert bool(res["same_on_all_ranks"])
    dim, hidden = FFN_SHAPE
    gate, up, down, norm, x = ffn_weights(31)
    raws = [G.quantize(G.TYPE_Q4_K, m) for m in (gate, up, down)]
    for k in range(3):
        n = O.rmsnorm(x, norm, 1e-5)
        hb = O.swiglu(O.matmul(G.TYPE_Q4_K, n, raws[0], hidden, dim), O.matmul(G.TYPE_Q4_K, n, raws[1], hidden, dim))
        x = (x + O.matmul(G.TYPE_Q4_K, hb, raws[2], dim, hidden)).astype(np.float32)
        assert_parity(res["xs"][k], x, what=f"tp{world} ffn block {k}")
