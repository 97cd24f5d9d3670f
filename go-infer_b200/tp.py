"""Tensor-parallel decode on the GPUs of one node (one process per GPU).

The counterpart of go-infer's TPCoordinator (pkg/distributed/
tensor_parallel.go): NewTPCoordinator(rank, peers) becomes connect(), which
exchanges the ranks' CUDA IPC handles of their exchange regions over an
initialised torch.distributed process group; AllReduce itself runs on the
GPUs inside every decode step (the row-split projections push their
partials over NVLink, see gi_cuda_tp_prepare).
"""
from __future__ import annotations

import numpy as np
import torch.distributed as dist

import goinfer_cuda as G
import synth


def connect(rank: int, world: int, max_dim: int) -> None:
    """Allocate this rank's exchange region and map every peer's."""
    handle = G.tp_prepare(world, max_dim)
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    G.tp_connect(rank, world, b"".join(handles))
    dist.barrier()


def build(cfg: synth.LlamaConfig, seed: int, rank: int, world: int, max_pos: int = 0, device_synth: bool = False):
    """This rank's shard of the seeded synthetic model, on the device (drawn
    on the host, or with device_synth on the GPU)."""
    if device_synth:
        dev = synth.DeviceModel.synth_on_device(cfg, seed, rank=rank, world=world)
    else:
        dev = synth.DeviceModel(synth.synth_model(cfg, seed, rank=rank, world=world))
    return dev, dev.model(max_pos, tp_rank=rank, tp_world=world)


def build_gguf(path: str, rank: int, world: int, max_pos: int = 0, max_seq: int = 8192):
    """This rank's shard of the model in a GGUF file, sliced at load
    (gguf.host_model with rank/world), on the device."""
    import gguf

    with gguf.GGUFReader(path) as r:  # world 1: views of the mapped file, copied to the device here
        dev = synth.DeviceModel(gguf.host_model(r, max_seq=max_seq, rank=rank, world=world))
    return dev, dev.model(max_pos, tp_rank=rank, tp_world=world)


def greedy(model: G.Model, prompt, n_gen: int):
    """Greedy decode on every rank (identical ids on all ranks)."""
    ids, _logits, ms = model.generate(np.asarray(prompt, np.int32), n_gen)
    return ids, ms
