"""Host side of the tensor-parallel split, on CPU with world_size-2 gloo
ranks: each rank's shard (synth.synth_model(rank, world)) is a slice of the
same model; the row-split projections' partial products, summed across ranks
(an all-reduce, as TPCoordinator.AllReduce does), give the full projection;
and the vocabulary-sliced argmax rule (largest value, lowest index on ties)
picks the full argmax (forward.go:397-404)."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
import synth

CFG = synth.LlamaConfig(n_layers=1, dim=512, hidden=1024, n_heads=8, n_kv_heads=4, vocab=1000, max_seq=16)


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        full = synth.synth_model(CFG, 5)
        shard = synth.synth_model(CFG, 5, rank=rank, world=world)
        rng = np.random.default_rng(9)
        att = rng.normal(size=CFG.q_dim).astype(np.float32)
        h = rng.normal(size=CFG.hidden).astype(np.float32)
        sl = synth.shard_slices(CFG, rank, world)
        res = {}
        for name, vec in (("wo", att), ("ffn_down", h)):
            qt, w = shard.tensors[synth.layer_tensor(0, name)]
            _r0, nr, c0, nc = sl[name]
            part = O.matmul(qt, vec[c0:c0 + nc], w, nr, nc, nthreads=1)
            t = torch.from_numpy(part.copy())
            dist.all_reduce(t)
            qf, wf = full.tensors[synth.layer_tensor(0, name)]
            want = O.matmul_f64(qf, vec, wf, nr, len(vec), nthreads=1)
            res[name] = float(np.abs(t.numpy() - want).max() / (np.abs(want).max() + 1e-30))
        logits = rng.normal(size=CFG.vocab).astype(np.float32)
        logits[[17, 603]] = 9.0  # a tie across the two vocabulary slices
        v0 = CFG.vocab // world * rank
        loc = logits[v0:v0 + CFG.vocab // world]
        mine = torch.tensor([float(loc.max()), float(v0 + int(np.argmax(loc)))])
        got = [torch.zeros(2) for _ in range(world)]
        dist.all_gather(got, mine)
        best = min(((-float(g[0]), int(g[1])) for g in got))
        res["argmax"] = (best[1], int(np.argmax(logits)))
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:  # surface the failure to the parent
        q.put((rank, repr(e)))


def test_row_split_all_reduce_and_vocab_argmax():
    world, port = 2, 29651
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r, res in results.items():
        assert isinstance(res, dict), f"rank {r}: {res}"
        assert res["wo"] < 1e-5 and res["ffn_down"] < 1e-5, res
        assert res["argmax"][0] == res["argmax"][1] == 17
