"""Synthetic Llama-shaped GGUF models for the decode workloads.

The benchmark configurations name random-init models (weights N(0, 0.02),
quantised Q4_K, lm_head Q6_K, norms fp32).  This module draws them with the
library's seeded generator (gi_quantize_seeded: one stream per (seed, row,
256-column block), so the bytes are the same on every machine and thread
count, and a tensor-parallel shard is drawn on its own), uploads them
as weight buffers and describes them to the device-resident model
(gi_cuda_model_create) or to gi_cuda_forward_transformer.  Tensor names and
roles follow go-infer's GGUF loader (blk.N.attn_q.weight ...,
pkg/engine/weights.go); norm weights are ones, the usual RMSNorm init.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

import goinfer_cuda as G


@dataclass
class LlamaConfig:
    n_layers: int
    dim: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    vocab: int
    max_seq: int
    eps: float = 1e-5
    rope_theta: float = 10000.0
    wtype: int = G.TYPE_Q4_K
    out_type: int = G.TYPE_Q6_K
    embd_type: int = G.TYPE_Q4_K
    std: float = 0.02
    hd: int = 0  # head dim when it is not dim / n_heads (a tensor-parallel shard)

    @property
    def head_dim(self) -> int:  # config.go:29-37
        return self.hd or self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:  # config.go:48-56
        return self.head_dim * self.n_kv_heads

    @property
    def q_dim(self) -> int:
        return self.head_dim * self.n_heads


# Config 4: Llama-2-7B shape (32 layers, d=4096, 32 heads, FFN 11008, vocab
# 32000, RoPE base 10000), 128-token prompt + 64 greedy steps.
LLAMA2_7B = LlamaConfig(n_layers=32, dim=4096, hidden=11008, n_heads=32, n_kv_heads=32, vocab=32000, max_seq=192)

# Config 5: Llama-3-70B shape (80 layers, d=8192, 64 query / 8 KV heads, FFN
# 28672, vocab 128256, RoPE base 500000), every matrix Q4_K (the output head
# too), 512-token prompt + 64 greedy steps.
LLAMA3_70B = LlamaConfig(n_layers=80, dim=8192, hidden=28672, n_heads=64, n_kv_heads=8, vocab=128256, max_seq=576,
                         rope_theta=500000.0, out_type=G.TYPE_Q4_K)

LAYER_MATS = ("wq", "wk", "wv", "wo", "ffn_gate", "ffn_up", "ffn_down")

# GGUF tensor name of each layer matrix role (pkg/engine/forward.go:146-152,
# engine_test.go:43-56); the roles are the field names of the layer table.
TENSOR_NAMES = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "ffn_gate": "ffn_gate",
                "ffn_up": "ffn_up", "ffn_down": "ffn_down"}


def layer_tensor(l: int, role: str) -> str:
    """GGUF name of layer l's matrix `role` (e.g. blk.3.attn_q.weight)."""
    return f"blk.{l}.{TENSOR_NAMES[role]}.weight"


def layer_shapes(cfg: LlamaConfig) -> dict:
    """rows x cols of each layer matrix (rows = output features)."""
    return {"wq": (cfg.q_dim, cfg.dim), "wk": (cfg.kv_dim, cfg.dim), "wv": (cfg.kv_dim, cfg.dim),
            "wo": (cfg.dim, cfg.q_dim), "ffn_gate": (cfg.hidden, cfg.dim), "ffn_up": (cfg.hidden, cfg.dim),
            "ffn_down": (cfg.dim, cfg.hidden)}


@dataclass
class HostModel:
    """Raw tensors of a model: {name: (ggml type, uint8/float32 array)}."""
    cfg: LlamaConfig
    tensors: dict = field(default_factory=dict)


def shard_config(cfg: LlamaConfig, world: int) -> LlamaConfig:
    """This rank's shapes under Megatron tensor parallelism over `world` GPUs."""
    if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.hidden % (256 * world) or cfg.vocab % world \
            or (cfg.q_dim // world) % 256:
        raise ValueError(f"{cfg} does not split {world} ways on 256-column blocks")
    return LlamaConfig(cfg.n_layers, cfg.dim, cfg.hidden // world, cfg.n_heads // world, cfg.n_kv_heads // world,
                       cfg.vocab // world, cfg.max_seq, cfg.eps, cfg.rope_theta, cfg.wtype, cfg.out_type,
                       cfg.embd_type, cfg.std, hd=cfg.head_dim)


def shard_slices(cfg: LlamaConfig, rank: int, world: int) -> dict:
    """(row0, rows, col0, cols) of rank's shard of each matrix: column split
    (rows) for Q, K, V, gate, up and the output head, row split (columns)
    for the output and down projections; the token table is replicated."""
    q, kv, h, v = cfg.q_dim // world, cfg.kv_dim // world, cfg.hidden // world, cfg.vocab // world
    return {"wq": (rank * q, q, 0, cfg.dim), "wk": (rank * kv, kv, 0, cfg.dim), "wv": (rank * kv, kv, 0, cfg.dim),
            "wo": (0, cfg.dim, rank * q, q), "ffn_gate": (rank * h, h, 0, cfg.dim),
            "ffn_up": (rank * h, h, 0, cfg.dim), "ffn_down": (0, cfg.dim, rank * h, h),
            "output": (rank * v, v, 0, cfg.dim), "token_embd": (0, cfg.vocab, 0, cfg.dim)}


def synth_model(cfg: LlamaConfig, seed: int, threads: int = 0, rank: int = 0, world: int = 1) -> HostModel:
    """Every tensor drawn with seed * 1_000_003 + its index; with world > 1
    only rank's shard of each (a slice of the same tensors), under the
    shard's config."""
    shapes = layer_shapes(cfg)
    sl = shard_slices(cfg, rank, world) if world > 1 else None
    m = HostModel(shard_config(cfg, world) if world > 1 else cfg)
    k = 0

    def draw(qt, name, rows, cols):
        nonlocal k
        k += 1
        r0, nr, c0, nc = sl[name] if sl else (0, rows, 0, cols)
        return (qt, G.quantize_seeded(qt, seed * 1_000_003 + k, cfg.std, nr, nc, threads, row0=r0, col0=c0))

    m.tensors["token_embd.weight"] = draw(cfg.embd_type, "token_embd", cfg.vocab, cfg.dim)
    for l in range(cfg.n_layers):
        for name in LAYER_MATS:
            r, c = shapes[name]
            m.tensors[layer_tensor(l, name)] = draw(cfg.wtype, name, r, c)
        for name in ("attn_norm", "ffn_norm"):
            m.tensors[f"blk.{l}.{name}.weight"] = (G.TYPE_F32, np.ones(cfg.dim, np.float32))
    m.tensors["output_norm.weight"] = (G.TYPE_F32, np.ones(cfg.dim, np.float32))
    m.tensors["output.weight"] = draw(cfg.out_type, "output", cfg.vocab, cfg.dim)
    return m


class DeviceModel:
    """The tensors of a HostModel as weight buffers, with the layer table."""

    def __init__(self, host: HostModel = None, *, cfg: LlamaConfig = None, bufs: dict = None, types: dict = None):
        if host is not None:
            cfg, bufs, types = host.cfg, {}, {}
            for name, (qt, arr) in host.tensors.items():
                b = G.CreateBuffer(arr)
                if b is None:
                    raise G.GoInferCudaError("CreateBuffer " + name, G.ERR_BUFFER)
                bufs[name] = b
                types[name] = qt
        self.cfg, self.bufs, self.types = cfg, bufs, types
        self._layer_table()

    @classmethod
    def synth_on_device(cls, cfg: LlamaConfig, seed: int, rank: int = 0, world: int = 1) -> "DeviceModel":
        """synth_model's tensors (or rank's shard of them) drawn on the GPU
        (gi_synth_weights: same streams, float32 transform), so a 70B-shaped
        model takes seconds rather than host minutes."""
        shapes = layer_shapes(cfg)
        sl = shard_slices(cfg, rank, world) if world > 1 else None
        bufs, types = {}, {}
        k = 0

        def draw(key, qt, name, rows, cols):
            nonlocal k
            k += 1
            r0, nr, c0, nc = sl[name] if sl else (0, rows, 0, cols)
            bufs[key] = G.synth_buffer(qt, seed * 1_000_003 + k, cfg.std, nr, nc, row0=r0, col0=c0)
            types[key] = qt

        ones = np.ones(cfg.dim, np.float32)
        try:
            draw("token_embd.weight", cfg.embd_type, "token_embd", cfg.vocab, cfg.dim)
            for l in range(cfg.n_layers):
                for name in LAYER_MATS:
                    r, c = shapes[name]
                    draw(layer_tensor(l, name), cfg.wtype, name, r, c)
                for name in ("attn_norm", "ffn_norm"):
                    bufs[f"blk.{l}.{name}.weight"] = G.CreateBuffer(ones)
                    types[f"blk.{l}.{name}.weight"] = G.TYPE_F32
            bufs["output_norm.weight"] = G.CreateBuffer(ones)
            types["output_norm.weight"] = G.TYPE_F32
            draw("output.weight", cfg.out_type, "output", cfg.vocab, cfg.dim)
        except Exception:
            for b in bufs.values():
                G.ReleaseBuffer(b)
            raise
        return cls(cfg=shard_config(cfg, world) if world > 1 else cfg, bufs=bufs, types=types)

    def raw(self, name: str) -> np.ndarray:
        """A tensor's bytes copied back to the host (for the oracle)."""
        out = G.read_buffer(self.bufs[name])
        return out.view(np.float32) if self.types[name] == G.TYPE_F32 else out

    def _layer_table(self) -> None:
        layers = []
        for l in range(self.cfg.n_layers):
            d = {}
            for name in LAYER_MATS:
                key = layer_tensor(l, name)
                d[name] = self.bufs[key]
                d[name + "_type"] = self.types[key]
            d["attn_norm"] = self.bufs[f"blk.{l}.attn_norm.weight"]
            d["ffn_norm"] = self.bufs[f"blk.{l}.ffn_norm.weight"]
            # optional Q, K, V biases (Qwen 2; forward.go:211-225)
            for key, bias in (("bq", "attn_q"), ("bk", "attn_k"), ("bv", "attn_v")):
                if f"blk.{l}.{bias}.bias" in self.bufs:
                    d[key] = self.bufs[f"blk.{l}.{bias}.bias"]
            layers.append(d)
        self.table = G.layer_table(layers)

    def desc(self, max_pos: int = 0, tp_rank: int = 0, tp_world: int = 1) -> G.ModelDesc:
        c = self.cfg
        d = G.ModelDesc()
        d.num_layers, d.dim, d.hidden_dim = c.n_layers, c.dim, c.hidden
        d.num_heads, d.num_kv_heads, d.head_dim = c.n_heads, c.n_kv_heads, c.head_dim
        d.vocab_size, d.max_seq, d.max_pos = c.vocab, c.max_seq, max_pos
        d.norm_eps, d.rope_theta = c.eps, c.rope_theta
        d.layers = ctypes.cast(self.table, ctypes.POINTER(G.LayerWeights))
        d.token_embd = self.bufs["token_embd.weight"].handle
        d.token_embd_type = self.types["token_embd.weight"]
        d.output_norm = self.bufs["output_norm.weight"].handle
        d.output_weight = self.bufs["output.weight"].handle
        d.output_weight_type = self.types["output.weight"]
        d.tp_world, d.tp_rank, d.vocab_offset = tp_world, tp_rank, tp_rank * c.vocab if tp_world > 1 else 0
        return d

    def model(self, max_pos: int = 0, tp_rank: int = 0, tp_world: int = 1) -> G.Model:
        return G.Model(self.desc(max_pos, tp_rank, tp_world), keep=self)

    def close(self) -> None:
        for b in self.bufs.values():
            G.ReleaseBuffer(b)
        self.bufs.clear()
