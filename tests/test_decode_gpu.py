"""GPU whole-model decode against the oracle's Engine.Forward, through the C ABI.

gi_cuda_forward_transformer (the metal_forward_transformer mirror) is
compared step by step on logits (per-element parity bar); the
device-resident greedy loop (gi_cuda_model_generate) on token ids, which
must be identical to the oracle's greedy decode (forward.go:394-405,
first maximum), with the smallest top-2 margin reported on failure.
"""
import numpy as np
import pytest

import goinfer_cuda as G
import oracle as O
import synth
from _util import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def cuda():
    G.Init(0)
    assert G.IsAvailable()
    yield


SMALL = synth.LlamaConfig(n_layers=2, dim=512, hidden=1024, n_heads=8, n_kv_heads=2, vocab=1000, max_seq=64)


@pytest.fixture(scope="module")
def small():
    host = synth.synth_model(SMALL, seed=11)
    dev = synth.DeviceModel(host)
    yield host, dev
    dev.close()


def embedding(host, token):
    qt, raw = host.tensors["token_embd.weight"]
    rb = O.bytes_per_row(qt, host.cfg.dim)
    return O.dequantize(qt, raw[token * rb:(token + 1) * rb], host.cfg.dim)


def test_forward_transformer_matches_oracle(small):
    host, dev = small
    c = host.cfg
    ref = O.RefModel(c, host.tensors)
    G.AllocBuffers(c.dim, c.hidden, c.kv_dim, c.vocab, c.n_layers, c.max_seq)
    scale = float(np.float32(1.0 / O.math_sqrt(float(c.head_dim))))
    for pos, tok in enumerate([3, 141, 59, 26, 535, 897, 932, 384]):
        logits, nxt = G.ForwardTransformer(
            embedding(host, tok), dev.table, dev.bufs["output_norm.weight"], dev.bufs["output.weight"],
            dev.types["output.weight"], num_layers=c.n_layers, dim=c.dim, hidden_dim=c.hidden, kv_dim=c.kv_dim,
            vocab_size=c.vocab, num_heads=c.n_heads, num_kv_heads=c.n_kv_heads, head_dim=c.head_dim, pos=pos,
            slot=pos % c.max_seq, max_seq=c.max_seq, active_context=min(pos + 1, c.max_seq), norm_eps=c.eps,
            rope_theta=c.rope_theta, attn_scale=scale)
        want = ref.forward(tok, pos)
        assert_parity(logits, want, what=f"logits at pos {pos}")
        assert nxt == int(np.argmax(logits))


def check_greedy(dev_model, ref, prompt, n_gen):
    ids, logits, _ms = dev_model.generate(prompt, n_gen, want_logits=True)
    want, margins, want_logits = ref.greedy(prompt, n_gen)
    if not np.array_equal(ids, want):
        i = int(np.argmax(ids != want))
        pytest.fail(f"greedy ids differ first at step {i}: gpu {ids[i]} vs oracle {want[i]} "
                    f"(oracle top-2 margin there {margins[i]:.3e}, smallest {margins.min():.3e})")
    # Whole-model logits carry the float32 summation-order noise of every
    # layer: held to a normwise bar, max |gpu - oracle| <= 1e-3 * rms(oracle).
    ref = want_logits.astype(np.float64)
    err = np.abs(logits - ref).max() / np.sqrt(np.mean(ref * ref))
    assert err <= 1e-3, f"last-step logits: max |diff| / rms = {err:.3e}"
    return ids


def test_generate_matches_oracle_greedy(small):
    host, dev = small
    ref = O.RefModel(host.cfg, host.tensors)
    model = dev.model()
    try:
        prompt = np.random.default_rng(12).integers(0, host.cfg.vocab, 16)
        ids = check_greedy(model, ref, prompt, 24)
        # reset + replay gives the same ids (the captured step is reused)
        model.reset()
        again, _l, _ms = model.generate(prompt, 24)
        assert np.array_equal(again, ids)
    finally:
        model.close()


def test_generate_wraps_the_kv_cache():
    """Positions past max_seq reuse slots pos % max_seq (engine_test.go:194)."""
    cfg = synth.LlamaConfig(n_layers=2, dim=256, hidden=512, n_heads=4, n_kv_heads=4, vocab=512, max_seq=8)
    host = synth.synth_model(cfg, seed=13)
    dev = synth.DeviceModel(host)
    model = dev.model()
    try:
        check_greedy(model, O.RefModel(cfg, host.tensors), [5, 77, 300, 12, 9], 12)
    finally:
        model.close()
        dev.close()


def test_synthetic_engine_model():
    """engine_test.go:159-192's model (all-0.1 F32 weights, dim 16, vocab 6)."""
    cfg = synth.LlamaConfig(n_layers=1, dim=16, hidden=32, n_heads=2, n_kv_heads=2, vocab=6, max_seq=32,
                            rope_theta=500000.0)
    T = {}
    for name, (r, c) in [("token_embd.weight", (cfg.vocab, cfg.dim)), ("output.weight", (cfg.vocab, cfg.dim))]:
        T[name] = (G.TYPE_F32, np.full((r, c), 0.1, np.float32))
    for name, (r, c) in synth.layer_shapes(cfg).items():
        T[synth.layer_tensor(0, name)] = (G.TYPE_F32, np.full((r, c), 0.1, np.float32))
    for name in ("blk.0.attn_norm.weight", "blk.0.ffn_norm.weight", "output_norm.weight"):
        T[name] = (G.TYPE_F32, np.full(cfg.dim, 0.1, np.float32))
    dev = synth.DeviceModel(synth.HostModel(cfg, T))
    model = dev.model()
    try:
        ids = check_greedy(model, O.RefModel(cfg, T, nthreads=1), [1, 3, 4], 3)
        assert list(ids) == [0, 0, 0]
    finally:
        model.close()
        dev.close()


def test_model_rejects_bad_arguments(small):
    _host, dev = small
    model = dev.model(max_pos=40)
    try:
        with pytest.raises(G.GoInferCudaError) as e:
            model.generate([1, 2, 3], 40)  # positions 0..41 > max_pos 40
        assert e.value.code == G.ERR_SHAPE
        with pytest.raises(G.GoInferCudaError):
            model.generate([SMALL.vocab], 1)  # token id out of range
    finally:
        model.close()


def golden_decode(which, persistent=False, tol=2e-3):
    """A whole-model golden (tests/golden/make_decode_golden.py): the model
    drawn on the device by gi_synth_weights (the bytes gi_quantize_seeded
    gave the oracle on the host, checked through the digest), the prompt,
    then 64 greedy steps: ids identical to the CPU oracle's Engine.Forward."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_decode_golden as MG
    cfg, seed, _ps, _pl, steps, fname = MG.GOLDENS[which]
    path = os.path.join(os.path.dirname(__file__), "golden", fname)
    if not os.path.exists(path):
        pytest.skip(f"{fname} not generated (python tests/golden/make_decode_golden.py {which})")
    gold = np.load(path)
    assert int(gold["seed"]) == seed
    dev = synth.DeviceModel.synth_on_device(cfg, seed=seed)
    model = None
    try:
        assert MG.device_model_digest(dev) == str(gold["digest"]), "the device-drawn weights differ from the golden's"
        model = dev.model()
        if persistent:
            model.set_persistent(True)
        ids, logits, _ms = model.generate(gold["prompt"], steps, want_logits=True)
        if not np.array_equal(ids, gold["ids"]):
            i = int(np.argmax(ids != gold["ids"]))
            pytest.fail(f"{which} greedy ids differ first at step {i}: gpu {ids[i]} vs oracle {gold['ids'][i]} "
                        f"(oracle top-2 margin {gold['margins'][i]:.3e})")
        # After every layer and every position the float32 summation-order
        # noise of the residual stream is larger than one GEMV's: the logits
        # are held to a normwise bar, max |gpu - oracle| <= tol * rms(oracle).
        ref = gold["last_logits"].astype(np.float64)
        dev_err = np.abs(logits - ref).max() / np.sqrt(np.mean(ref * ref))
        print(f"{which}: 64 ids identical to the oracle; smallest oracle top-2 margin "
              f"{gold['margins'].min():.3e}; last logits max |diff| / rms = {dev_err:.3e}")
        assert dev_err <= tol, f"{which} last logits: max |diff| / rms = {dev_err:.3e}"
    finally:
        if model is not None:
            model.close()
        dev.close()


def test_config4_greedy_matches_oracle_golden():
    """Config 4 (Llama-2-7B shape, Q4_K / Q6_K lm_head): 128-token prompt then
    64 greedy steps, ids identical to the CPU oracle's."""
    golden_decode("7b")


def test_config5_greedy_matches_oracle_golden():
    """Config 5 (Llama-3-70B shape, 80 layers, every matrix Q4_K) on one GPU:
    512-token prompt then 64 greedy steps, ids identical to the CPU oracle's."""
    golden_decode("70b")


@pytest.mark.parametrize("qt", [G.TYPE_Q4_K, G.TYPE_Q6_K, G.TYPE_Q8_0, G.TYPE_F32])
def test_device_generator_matches_host_bytes(qt):
    """gi_synth_weights (device) and gi_quantize_seeded (host) draw the same
    seeded matrix byte for byte, whole or as a shard (row and column offset)."""
    for rows, cols, row0, col0 in ((37, 1024, 0, 0), (5, 4096, 1000, 2048), (300, 256, 7, 256)):
        host = G.quantize_seeded(qt, 123, 0.02, rows, cols, row0=row0, col0=col0)
        buf = G.synth_buffer(qt, 123, 0.02, rows, cols, row0=row0, col0=col0)
        try:
            dev = G.read_buffer(buf)[:host.size]
        finally:
            G.ReleaseBuffer(buf)
        assert np.array_equal(dev, host), f"type {qt} {rows}x{cols} at ({row0}, {col0})"


def test_70b_widths_two_layers_match_oracle():
    """Config 5's widths (d=8192, 64 query / 8 KV heads, FFN 28672, vocab
    128256, RoPE base 500000) on two layers, weights drawn on the device and
    read back for the oracle: greedy ids identical to Engine.Forward's."""
    import dataclasses
    cfg = dataclasses.replace(synth.LLAMA3_70B, n_layers=2, max_seq=64)
    dev = synth.DeviceModel.synth_on_device(cfg, seed=70)
    model = dev.model()
    try:
        tensors = {name: (dev.types[name], dev.raw(name)) for name in dev.bufs}
        ref = O.RefModel(cfg, tensors)
        prompt = np.random.default_rng(71).integers(0, cfg.vocab, 12)
        check_greedy(model, ref, prompt, 8)
    finally:
        model.close()
        dev.close()


def test_model_from_gguf_file(tmp_path):
    """A model read from a GGUF file (go-infer_b200/gguf.py, the format of
    pkg/gguf) decodes the same ids as the in-memory synthetic model it was
    written from, and as the oracle."""
    import gguf
    host = synth.synth_model(SMALL, seed=15)
    path = str(tmp_path / "small.gguf")
    gguf.save_model(host, path)
    prompt = np.random.default_rng(16).integers(0, SMALL.vocab, 8)
    with gguf.GGUFReader(path) as r:
        dev = synth.DeviceModel(gguf.host_model(r))
    model = dev.model()
    try:
        ids = check_greedy(model, O.RefModel(host.cfg, host.tensors), prompt, 8)
        mem = synth.DeviceModel(host)
        m2 = mem.model()
        try:
            ids2, _l, _ms = m2.generate(prompt, 8)
        finally:
            m2.close()
            mem.close()
        assert np.array_equal(ids, ids2)
    finally:
        model.close()
        dev.close()


def test_qkv_biases_match_oracle():
    """Qwen 2-style Q/K/V biases (forward.go:211-225) through the device
    decode loop: ids identical to the oracle's, logits within the bar, and
    the biases change the logits."""
    cfg = synth.LlamaConfig(n_layers=2, dim=512, hidden=1024, n_heads=8, n_kv_heads=2, vocab=1000, max_seq=64)
    host = synth.synth_model(cfg, seed=31)
    rng = np.random.default_rng(32)
    for l in range(cfg.n_layers):
        for name, n in (("attn_q", cfg.q_dim), ("attn_k", cfg.kv_dim), ("attn_v", cfg.kv_dim)):
            host.tensors[f"blk.{l}.{name}.bias"] = (G.TYPE_F32, rng.normal(0, 0.3, n).astype(np.float32))
    dev = synth.DeviceModel(host)
    model = dev.model()
    try:
        prompt = rng.integers(0, cfg.vocab, 6)
        check_greedy(model, O.RefModel(cfg, host.tensors), prompt, 8)
        plain = {k: v for k, v in host.tensors.items() if not k.endswith(".bias")}
        _w, _m, plain_logits = O.RefModel(cfg, plain).greedy(prompt, 8)
        _w, _m, bias_logits = O.RefModel(cfg, host.tensors).greedy(prompt, 8)
        assert not np.allclose(plain_logits, bias_logits)
    finally:
        model.close()
        dev.close()


PERSISTENT_CASES = {
    # name: (config, seed, prompt length, greedy steps, draw on the device)
    "small": (SMALL, 11, 16, 24, False),
    "kv_wrap": (synth.LlamaConfig(n_layers=2, dim=256, hidden=512, n_heads=4, n_kv_heads=4, vocab=512, max_seq=8),
                13, 5, 12, False),
    "70b_widths": (None, 70, 12, 8, True),
}


@pytest.mark.parametrize("case", sorted(PERSISTENT_CASES))
def test_persistent_layers_match_oracle(case):
    """gi_cuda_model_set_persistent: every layer of a step in one cooperative
    launch.  Greedy ids identical to the oracle's Engine.Forward, logits
    within the per-layer launches' bar of the oracle and of the per-layer
    launches themselves, and the same bits when run twice."""
    import dataclasses
    cfg, seed, plen, n_gen, on_device = PERSISTENT_CASES[case]
    if cfg is None:
        cfg = dataclasses.replace(synth.LLAMA3_70B, n_layers=2, max_seq=64)
    dev = synth.DeviceModel.synth_on_device(cfg, seed=seed) if on_device else \
        synth.DeviceModel(synth.synth_model(cfg, seed=seed))
    model = dev.model()
    try:
        tensors = {name: (dev.types[name], dev.raw(name)) for name in dev.bufs}
        ref = O.RefModel(cfg, tensors)
        prompt = np.random.default_rng(seed + 100).integers(0, cfg.vocab, plen)
        ids_layer, logits_layer, _ms = model.generate(prompt, n_gen, want_logits=True)
        model.reset()
        model.set_persistent(True)
        ids = check_greedy(model, ref, prompt, n_gen)
        assert np.array_equal(ids, ids_layer)
        model.reset()
        ids2, logits_p, _ms = model.generate(prompt, n_gen, want_logits=True)
        model.reset()
        ids3, logits_p2, _ms = model.generate(prompt, n_gen, want_logits=True)
        assert np.array_equal(ids2, ids) and np.array_equal(ids3, ids)
        assert np.array_equal(logits_p.view(np.uint32), logits_p2.view(np.uint32))
        base = logits_layer.astype(np.float64)
        err = np.abs(logits_p - base).max() / np.sqrt(np.mean(base * base))
        print(f"{case}: persistent vs per-layer launches, last logits max |diff| / rms = {err:.3e}")
        assert err <= 1e-3
    finally:
        model.close()
        dev.close()


def test_persistent_config4_matches_oracle_golden():
    """Config 4 with every layer of a step in one persistent launch: ids
    identical to the CPU oracle's for 64 steps."""
    golden_decode("7b", persistent=True)
