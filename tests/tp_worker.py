"""One rank of a tensor-parallel greedy decode (run under torchrun by
tests/test_tp_gpu.py and bench.py): builds this rank's shard of a seeded
synthetic model, connects the exchange regions, decodes, and (rank 0) writes
the ids and device time to --out as .npz."""
import argparse
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "go-infer_b200"))

import goinfer_cuda as G  # noqa: E402
import synth  # noqa: E402
import tp  # noqa: E402

CONFIGS = {
    # small enough for a test; every split is whole 256-column blocks for 2 / 4 / 8 ranks
    "small": synth.LlamaConfig(n_layers=2, dim=2048, hidden=4096, n_heads=16, n_kv_heads=8, vocab=4096, max_seq=64),
    "llama70b": synth.LLAMA3_70B,
}


# dim, hidden of the tensor-parallel FFN test: 11 blocks of 256 hidden
# columns, so 2, 4 and 8 ranks get unequal slices.
FFN_SHAPE = (2048, 2816)


def ffn_shard(world: int, rank: int, hidden: int):
    """(h0, hn): rank's hidden slice in whole 256-column blocks."""
    nsb = hidden // 256
    b0, b1 = nsb * rank // world, nsb * (rank + 1) // world
    return 256 * b0, 256 * (b1 - b0)


def ffn_weights(seed: int):
    """The FFN test's full matrices (gate, up: hidden x dim; down: dim x
    hidden) as float32, and its norm weight and input."""
    dim, hidden = FFN_SHAPE
    rng = np.random.default_rng(seed)
    gate = rng.normal(0, 0.02, (hidden, dim)).astype(np.float32)
    up = rng.normal(0, 0.02, (hidden, dim)).astype(np.float32)
    down = rng.normal(0, 0.02, (dim, hidden)).astype(np.float32)
    norm = (1.0 + 0.1 * rng.normal(0, 1, dim)).astype(np.float32)
    x = rng.normal(0, 1, dim).astype(np.float32)
    return gate, up, down, norm, x


def ffn_blocks(a, rank: int, world: int):
    dim, hidden = FFN_SHAPE
    tp.connect(rank, world, dim)
    gate, up, down, norm, x = ffn_weights(a.seed)
    h0, hn = ffn_shard(world, rank, hidden)
    bufs = [G.CreateBuffer(norm), G.CreateBuffer(G.quantize(G.TYPE_Q4_K, gate[h0:h0 + hn])),
            G.CreateBuffer(G.quantize(G.TYPE_Q4_K, up[h0:h0 + hn])),
            G.CreateBuffer(G.quantize(G.TYPE_Q4_K, np.ascontiguousarray(down[:, h0:h0 + hn])))]
    xs = []
    for _ in range(3):
        G.FFNBuf(x, *bufs, dim, hn, 1e-5)
        xs.append(x.copy())
    all_x = [None] * world
    dist.all_gather_object(all_x, x.tobytes())
    if rank == 0:
        np.savez(a.out, xs=np.stack(xs), same_on_all_ranks=np.array(all(v == all_x[0] for v in all_x)))
    for b in bufs:
        G.ReleaseBuffer(b)
    dist.barrier()
    G.tp_close()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="small")
    ap.add_argument("--seed", type=int, default=21)
    ap.add_argument("--prompt", type=int, default=12)
    ap.add_argument("--prompt-seed", type=int, default=None, help="numpy seed of the prompt (default seed + 1)")
    ap.add_argument("--gen", type=int, default=16)
    ap.add_argument("--out", required=True)
    ap.add_argument("--device-synth", action="store_true", help="draw the weights on the GPU")
    ap.add_argument("--persistent", action="store_true", help="every layer of a step in one persistent launch")
    ap.add_argument("--ffn", action="store_true",
                    help="instead of decoding: three tensor-parallel FFN blocks (gi_cuda_ffn_buf) on FFN_SHAPE")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", init_method="env://")
    G.Init(local)
    if a.ffn:
        return ffn_blocks(a, rank, world)
    cfg = CONFIGS[a.config]
    tp.connect(rank, world, cfg.dim)
    dev, model = tp.build(cfg, a.seed, rank, world, device_synth=a.device_synth)
    if a.persistent:
        model.set_persistent(True)
    pseed = a.seed + 1 if a.prompt_seed is None else a.prompt_seed
    prompt = np.random.default_rng(pseed).integers(0, cfg.vocab, a.prompt)
    ids, ms = tp.greedy(model, prompt, a.gen)
    all_ids = [None] * world
    dist.all_gather_object(all_ids, ids.tolist())
    if rank == 0:
        np.savez(a.out, ids=ids, ms=np.array(ms), prompt=prompt,
                 same_on_all_ranks=np.array(all(x == all_ids[0] for x in all_ids)))
    model.close()
    dev.close()
    dist.barrier()
    G.tp_close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
