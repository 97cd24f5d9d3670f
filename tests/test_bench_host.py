"""Host logic of bench.py without a GPU: the Megatron split of config 2's
FFN over N ranks and the line's config, which both arms must print alike."""
import importlib.util
import os

import numpy as np
import pytest

from _util import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ffn_shards_tile_the_hidden_dimension(bench, world):
    """Every 256-column Q4_K block of the 11008-wide hidden dimension lands
    on exactly one rank, in rank order, and slices differ by at most one
    block (the down rows split on block boundaries)."""
    shards = [bench.ffn_shard(world, r) for r in range(world)]
    assert shards[0][0] == 0
    for (h0, hn), (h1, _) in zip(shards, shards[1:]):
        assert h0 + hn == h1
    assert sum(hn for _, hn in shards) == bench.GATE[0]
    assert all(h0 % 256 == 0 and hn % 256 == 0 and hn > 0 for h0, hn in shards)
    assert max(hn for _, hn in shards) - min(hn for _, hn in shards) <= 256


@pytest.mark.parametrize("world", [1, 2, 8])
def test_config_is_shared_by_both_arms(bench, world):
    cfg = bench.step_config(world)
    assert set(cfg) == {"workload", "parallelism", "l2", "graph"}
    assert cfg == bench.step_config(world)
    assert ("tensor parallel" in cfg["parallelism"]) == (world > 1)


def test_step_bytes(bench):
    # two 11008 x 4096 GEMVs and one 4096 x 11008, raw Q4_K plus fp32 x and y
    assert bench.STEP_BYTES == 76_268_544
    assert bench.gemv_bytes(*bench.GATE) == bench.gemv_bytes(*bench.DOWN) == 25_422_848
    assert np.isclose(bench.STEP_BYTES / 22.44e-6 / 1e9, 3398.8, rtol=1e-3)
