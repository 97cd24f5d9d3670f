"""GGUF reader and writer (go-infer_b200/gguf.py) on CPU: the format as
go-infer's pkg/gguf parses it, mirrored from pkg/gguf/gguf_test.go (corrupted
headers, metadata helpers), plus round trips of the seeded synthetic models,
the alignment rule, Engine's configuration keys and defaults
(pkg/engine/engine.go:71-127), and the oracle's decode over tensors read
from a file matching the decode over the in-memory model."""
import dataclasses
import os
import struct

import numpy as np
import pytest

import gguf
import oracle as O
import synth

SMALL = synth.LlamaConfig(n_layers=2, dim=256, hidden=512, n_heads=4, n_kv_heads=2, vocab=300, max_seq=32,
                          rope_theta=10000.0)


def test_corrupted_headers_are_rejected(tmp_path):  # gguf_test.go:10-34
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(bytes([0x47, 0x47, 0x55, 0x46]))
    with pytest.raises(ValueError):
        gguf.GGUFReader(str(trunc))
    bad = tmp_path / "badmagic.gguf"
    bad.write_bytes(struct.pack("<IIQQ", 0x12345678, 3, 0, 0))
    with pytest.raises(ValueError, match="magic"):
        gguf.GGUFReader(str(bad))
    ver = tmp_path / "version.gguf"
    ver.write_bytes(struct.pack("<IIQQ", gguf.MAGIC, 7, 0, 0))
    with pytest.raises(ValueError, match="version"):
        gguf.GGUFReader(str(ver))
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    with pytest.raises(ValueError):
        gguf.GGUFReader(str(empty))


def test_metadata_helpers(tmp_path):  # gguf_test.go:36-60
    p = str(tmp_path / "meta.gguf")
    gguf.write_gguf(p, {"uint_val": gguf.Typed(gguf.T_U64, 42), "float_val": gguf.Typed(gguf.T_F64, 3.1415),
                        "string_val": "test_string", "flag": True,
                        "names": ["a", "b", "c"]}, [])
    with gguf.GGUFReader(p) as r:
        assert r.get_uint("uint_val", 0) == 42
        assert r.get_uint("missing_val", 99) == 99
        assert r.get_float("float_val", 0.0) == 3.1415
        assert r.get_float("missing_val", 1.0) == 1.0
        assert r.get_string("string_val", "") == "test_string"
        assert r.get_string("missing_val", "x") == "x"
        assert r.get_bool("flag") is True
        assert r.metadata["names"] == ["a", "b", "c"]
        assert r.version == 3 and r.tensors == {}


def test_synthetic_model_round_trip(tmp_path):
    host = synth.synth_model(SMALL, seed=7)
    p = str(tmp_path / "m.gguf")
    gguf.save_model(host, p)
    with gguf.GGUFReader(p) as r:
        assert r.data_offset % 32 == 0
        cfg = gguf.model_config(r)
        for f in ("n_layers", "dim", "hidden", "n_heads", "n_kv_heads", "vocab", "max_seq"):
            assert getattr(cfg, f) == getattr(SMALL, f), f
        assert np.float32(cfg.eps) == np.float32(SMALL.eps) and cfg.rope_theta == SMALL.rope_theta
        assert set(r.tensors) == set(host.tensors)
        for name, (qt, arr) in host.tensors.items():
            info = r.tensors[name]
            assert info.type == qt
            assert np.array_equal(r.tensor_data(name).view(np.uint8), np.asarray(arr).view(np.uint8).reshape(-1))
        # GGML dimension order: dims[0] is the row length
        assert r.tensors["blk.0.attn_q.weight"].dims == [SMALL.dim, SMALL.q_dim]
        assert r.tensors["blk.0.attn_output.weight"].dims == [SMALL.q_dim, SMALL.dim]
        assert r.tensors["blk.0.ffn_down.weight"].dims == [SMALL.hidden, SMALL.dim]
        assert r.tensors["token_embd.weight"].dims == [SMALL.dim, SMALL.vocab]


def test_alignment_and_bounds(tmp_path):
    p = str(tmp_path / "a.gguf")
    data = np.arange(64, dtype=np.float32)
    gguf.write_gguf(p, {"general.architecture": "llama"},
                    [("a", gguf.GGML_F32, [64], data), ("b", gguf.GGML_F32, [8, 8], data * 2)], alignment=64)
    with gguf.GGUFReader(p) as r:
        assert r.get_uint("general.alignment") == 64 and r.data_offset % 64 == 0
        assert np.array_equal(r.tensor_data("a"), data)
        assert np.array_equal(r.tensor_data("b"), data * 2)
        with pytest.raises(KeyError):
            r.tensor_data("missing")
    # a tensor whose bytes run past the end of the file is refused
    raw = bytearray(open(p, "rb").read())
    with open(p, "wb") as f:
        f.write(raw[:-100])
    with gguf.GGUFReader(p) as r:
        with pytest.raises(ValueError, match="exceeds"):
            r.tensor_data("b")


def test_engine_defaults_and_fallbacks(tmp_path):
    p = str(tmp_path / "d.gguf")
    emb = np.zeros((10, 4), np.float32)
    gguf.write_gguf(p, {"general.architecture": "qwen2", "llama.embedding_length": 4,
                        "qwen2.attention.head_count": 2},
                    [("token_embd.weight", gguf.GGML_F32, [4, 10], emb)])
    with gguf.GGUFReader(p) as r:
        c = gguf.model_config(r)
        assert c.dim == 4                          # llama.* fallback
        assert c.n_heads == 2 and c.n_kv_heads == 2  # <arch>.* first; kv defaults to heads
        assert (c.hidden, c.n_layers) == (5632, 16)
        assert c.rope_theta == 500000.0 and np.float32(c.eps) == np.float32(1e-5)
        assert c.vocab == 10                       # token_embd dim 1
        assert c.max_seq == 2048


def test_oracle_decode_from_file_matches_memory(tmp_path):
    host = synth.synth_model(SMALL, seed=9)
    p = str(tmp_path / "o.gguf")
    gguf.save_model(host, p)
    prompt = [3, 141, 59, 26]
    want, _m, want_logits = O.RefModel(SMALL, host.tensors).greedy(prompt, 4)
    with gguf.GGUFReader(p) as r:
        loaded = gguf.host_model(r)
        ids, _m2, logits = O.RefModel(loaded.cfg, loaded.tensors).greedy(prompt, 4)
    assert list(ids) == list(want)
    assert np.array_equal(logits, want_logits)


TP = synth.LlamaConfig(n_layers=2, dim=512, hidden=1024, n_heads=4, n_kv_heads=2, vocab=300, max_seq=32,
                       rope_theta=10000.0)


@pytest.mark.parametrize("world", [2])
def test_sharded_load_equals_the_seeded_shards(tmp_path, world):
    """Rank r's shard sliced out of the whole model's file equals the shard
    synth_model draws for rank r directly (the same seeded streams), byte
    for byte, under the same shard configuration."""
    p = str(tmp_path / "tp.gguf")
    gguf.save_model(synth.synth_model(TP, seed=21), p)
    with gguf.GGUFReader(p) as r:
        for rank in range(world):
            got = gguf.host_model(r, rank=rank, world=world)
            want = synth.synth_model(TP, seed=21, rank=rank, world=world)
            # eps is stored as float32 in the file
            assert got.cfg == dataclasses.replace(want.cfg, eps=float(np.float32(want.cfg.eps)))
            assert set(got.tensors) == set(want.tensors)
            for name, (qt, arr) in want.tensors.items():
                gq, ga = got.tensors[name]
                assert gq == qt, name
                assert np.array_equal(np.asarray(ga).view(np.uint8).reshape(-1),
                                      np.asarray(arr).view(np.uint8).reshape(-1)), (rank, name)


def test_shard_roles_and_block_boundaries():
    assert gguf.matrix_role("blk.3.attn_q.weight") == "wq"
    assert gguf.matrix_role("blk.3.attn_output.weight") == "wo"
    assert gguf.matrix_role("blk.0.ffn_down.weight") == "ffn_down"
    assert gguf.matrix_role("blk.0.attn_k.bias") == "wk"
    assert gguf.matrix_role("blk.0.attn_norm.weight") is None
    assert gguf.matrix_role("output_norm.weight") is None
    assert gguf.matrix_role("output.weight") == "output"
    w = np.arange(4 * 2 * 144, dtype=np.uint8)  # 4 rows x 2 Q4_K super-blocks
    s = gguf.shard_matrix(gguf.GGML_Q4_K, w, 4, 512, 1, 2, 256, 256)
    assert np.array_equal(s, w.reshape(4, 288)[1:3, 144:].reshape(-1))
    with pytest.raises(ValueError):
        gguf.shard_matrix(gguf.GGML_Q4_K, w, 4, 512, 0, 4, 128, 256)  # not on a super-block
    with pytest.raises(ValueError):
        gguf.shard_matrix(gguf.GGML_Q4_K, w, 4, 512, 3, 2, 0, 256)    # past the last row


def test_device_model_wiring_uses_gguf_names(monkeypatch):
    """DeviceModel's layer table takes every layer matrix and norm by its
    GGUF name (the library's buffer calls stubbed: no device needed)."""
    import goinfer_cuda as G

    class Buf:
        def __init__(self, arr):
            self.arr, self.handle = arr, id(arr)

    tables = []
    monkeypatch.setattr(G, "CreateBuffer", lambda arr: Buf(arr))
    monkeypatch.setattr(G, "layer_table", lambda layers: tables.append(layers) or layers)
    host = synth.synth_model(SMALL, seed=5)
    bq = np.ones(SMALL.q_dim, np.float32)
    host.tensors["blk.0.attn_q.bias"] = (gguf.GGML_F32, bq)  # layer 0 only, as a Qwen 2 model has
    dev = synth.DeviceModel(host)
    (layers,) = tables
    assert len(layers) == SMALL.n_layers
    for l, d in enumerate(layers):
        for role in synth.LAYER_MATS:
            qt, arr = host.tensors[synth.layer_tensor(l, role)]
            assert d[role].arr is arr and d[role + "_type"] == qt
        assert d["attn_norm"].arr is host.tensors[f"blk.{l}.attn_norm.weight"][1]
        assert "bk" not in d and "bv" not in d
    assert layers[0]["bq"].arr is bq and "bq" not in layers[1]


def test_device_drawn_model_wiring(monkeypatch):
    """synth_on_device names its buffers as synth_model names its tensors,
    and the layer table finds them (library calls stubbed)."""
    import goinfer_cuda as G

    class Buf:
        def __init__(self, key):
            self.key, self.handle = key, hash(key)

    drawn, tables = [], []
    monkeypatch.setattr(G, "CreateBuffer", lambda arr: Buf(("ones", arr.size)))
    monkeypatch.setattr(G, "synth_buffer",
                        lambda qt, seed, std, rows, cols, row0=0, col0=0: drawn.append((seed, rows, cols)) or
                        Buf((seed, rows, cols)))
    monkeypatch.setattr(G, "layer_table", lambda layers: tables.append(layers) or layers)
    dev = synth.DeviceModel.synth_on_device(TP, seed=3, rank=1, world=2)
    assert set(dev.bufs) == set(synth.synth_model(TP, seed=3, rank=1, world=2).tensors)
    (layers,) = tables
    shard = synth.shard_config(TP, 2)
    for l, d in enumerate(layers):
        for role in synth.LAYER_MATS:
            assert d[role] is dev.bufs[synth.layer_tensor(l, role)]
    assert dev.bufs["blk.0.attn_q.weight"].key[1:] == (shard.q_dim, TP.dim)
    assert dev.bufs["blk.0.attn_output.weight"].key[1:] == (TP.dim, shard.q_dim)


def test_damaged_files_raise_value_error(tmp_path):
    """Truncations, flipped bytes and huge counts in a valid file either
    still parse or raise ValueError -- never another exception, a deep
    recursion or a header parsed out of the tensor data."""
    import random
    good = tmp_path / "good.gguf"
    gguf.write_gguf(str(good), {"general.architecture": "llama", "llama.block_count": 2,
                                "names": ["a", "bb", "ccc"], "nested": [[1, 2], [3]],
                                "f": 0.5},
                    [("t", gguf.GGML_F32, [8, 2], np.arange(16, dtype=np.float32))])
    with gguf.GGUFReader(str(good)) as r:
        assert r.metadata["nested"] == [[1, 2], [3]] and r.metadata["names"] == ["a", "bb", "ccc"]
    raw = good.read_bytes()
    rng = random.Random(5)
    bad = tmp_path / "bad.gguf"
    outcomes = {"ok": 0, "value_error": 0}
    for i in range(1500):
        b = bytearray(raw)
        kind = i % 3
        if kind == 0:
            b = b[:rng.randrange(len(b))]
        elif kind == 1:
            for _ in range(rng.randrange(1, 4)):
                b[rng.randrange(len(b))] = rng.randrange(256)
        else:  # a huge little-endian count somewhere in the header
            pos = rng.randrange(0, min(len(b), 200) - 8)
            b[pos:pos + 8] = rng.choice([2 ** 63 - 1, 2 ** 40, 2 ** 32 + 1, 10 ** 6]).to_bytes(8, "little")
        bad.write_bytes(bytes(b))
        try:
            with gguf.GGUFReader(str(bad)) as r:
                for name in r.tensors:
                    try:
                        r.tensor_data(name)
                    except (ValueError, KeyError):
                        pass
            outcomes["ok"] += 1
        except ValueError:
            outcomes["value_error"] += 1
    assert outcomes["value_error"] > 500 and outcomes["ok"] > 0, outcomes


def test_nested_arrays_are_bounded(tmp_path):
    p = tmp_path / "deep.gguf"
    body = struct.pack("<IIQQ", gguf.MAGIC, 3, 0, 1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", gguf.T_ARR)
    for _ in range(50):  # arrays of one array each, 50 deep
        body += struct.pack("<IQ", gguf.T_ARR, 1)
    body += struct.pack("<IQ", gguf.T_U8, 0)
    p.write_bytes(body)
    with pytest.raises(ValueError, match="nested"):
        gguf.GGUFReader(str(p))


def test_impossible_counts_are_refused_up_front(tmp_path):
    p = tmp_path / "count.gguf"
    p.write_bytes(struct.pack("<IIQQ", gguf.MAGIC, 3, 10 ** 12, 0) + b"\0" * 64)  # 10^12 tensors in 64 bytes
    with pytest.raises(ValueError, match="exceeds the file"):
        gguf.GGUFReader(str(p))
    p.write_bytes(struct.pack("<IIQQ", gguf.MAGIC, 3, 0, 1) + struct.pack("<Q", 1) + b"k"
                  + struct.pack("<IIQ", gguf.T_ARR, gguf.T_U64, 2 ** 40))  # 2^40 u64 values in 0 bytes
    with pytest.raises(ValueError, match="exceeds the file"):
        gguf.GGUFReader(str(p))


def test_tp_build_from_gguf_wires_the_rank_shard(tmp_path, monkeypatch):
    """tp.build_gguf loads rank r's shard of a GGUF file into the device
    model under the shard configuration (library calls stubbed)."""
    import goinfer_cuda as G
    import tp

    p = str(tmp_path / "tp.gguf")
    gguf.save_model(synth.synth_model(TP, seed=23), p)

    class Buf:
        def __init__(self, arr):
            self.arr, self.handle = arr, id(arr)

    made = []
    monkeypatch.setattr(G, "CreateBuffer", lambda arr: Buf(arr))
    monkeypatch.setattr(G, "layer_table", lambda layers: layers)
    monkeypatch.setattr(synth.DeviceModel, "model",
                        lambda self, max_pos=0, tp_rank=0, tp_world=1: made.append((max_pos, tp_rank, tp_world)) or
                        "model")
    dev, model = tp.build_gguf(p, rank=1, world=2, max_pos=64, max_seq=32)
    assert model == "model" and made == [(64, 1, 2)]
    want = synth.synth_model(TP, seed=23, rank=1, world=2)
    assert dev.cfg.q_dim == want.cfg.q_dim and dev.cfg.hidden == want.cfg.hidden
    for name, (qt, arr) in want.tensors.items():
        got = dev.bufs[name].arr
        assert np.array_equal(np.asarray(got).view(np.uint8).reshape(-1), np.asarray(arr).view(np.uint8).reshape(-1))
