"""CPU tests of the oracle's whole-model decode (oracle/goinfer_ref.c
ref_forward and its kernels).

Mirrors go-infer's own tests of these functions: pkg/math/kernels_test.go
(RMSNorm, Softmax, ApplyRoPE, SwiGLU), pkg/engine/engine_test.go:194-217
(rolling KV cache) and :159-192 (the 1-layer, dim-16, all-0.1 F32 synthetic
model), and pins ref_forward against an independent pure-Python
restatement of Engine.Forward (forward.go:140-297) on a small model.
"""
import math

import numpy as np
import pytest

import goinfer_cuda as G
import oracle as O
import synth


def test_rmsnorm_kat():  # kernels_test.go:8-21
    out = O.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    assert abs(out[0] - np.float32(1.0 / math.sqrt(7.5 + 1e-5))) <= 1e-4


def test_softmax_kat():  # kernels_test.go:23-37
    x = O.softmax(np.array([1, 2, 3], np.float32))
    assert abs(float(x.sum(dtype=np.float32)) - 1.0) <= 1e-5
    assert x[2] > x[1] > x[0]


def test_rope_pos0_is_identity():  # kernels_test.go:39-46
    v = O.apply_rope(np.array([1, 0, 0, 1], np.float32), 0, 10000.0)
    assert list(v) == [1.0, 0.0, 0.0, 1.0]


def test_swiglu_kat():  # kernels_test.go:48-61
    g = O.swiglu(np.array([0.0, 2.0], np.float32), np.array([3.0, 4.0], np.float32))
    assert g[0] == 0.0 and 6.0 < g[1] < 8.0


def test_attn_scale_newton_sqrt():  # forward.go:33, 771-780
    # Ten Newton steps land within an ulp of sqrt (here one ulp off for 128),
    # which the float32 attention scale does not see.
    for hd in (16, 64, 128, 256):
        z = O.math_sqrt(float(hd))
        assert abs(z - math.sqrt(hd)) <= 2 * math.ulp(math.sqrt(hd))
        assert np.float32(1.0 / z) == np.float32(1.0 / math.sqrt(hd))
    assert O.math_sqrt(0.0) == 0.0 and O.math_sqrt(-1.0) == 0.0


def f32(v):
    return np.float32(v)


def py_dot(x, w):  # quant.go:548-566, 8-term groups
    s = f32(0)
    n = len(x)
    i = 0
    while i + 8 <= n:
        g = f32(x[i] * w[i])
        for j in range(1, 8):
            g = f32(g + f32(x[i + j] * w[i + j]))
        s = f32(s + g)
        i += 8
    while i < n:
        s = f32(s + f32(x[i] * w[i]))
        i += 1
    return s


def py_forward(cfg, W, kc, vc, token, pos):
    """Engine.Forward's CPU branch, one float32 rounding per Go operation."""
    dim, hd = cfg.dim, cfg.head_dim
    kv_mul = cfg.n_heads // cfg.n_kv_heads
    x = [f32(v) for v in W["token_embd.weight"][1].reshape(cfg.vocab, dim)[token]]

    def rms(v, w):
        s = f32(0)
        for a in v:
            s = f32(s + f32(a * a))
        mean = f32(s / f32(len(v)))
        sc = f32(1.0 / math.sqrt(float(f32(mean + f32(cfg.eps)))))
        return [f32(f32(a * sc) * f32(b)) for a, b in zip(v, w)]

    def mm(name, v, rows):
        w = W[name][1].reshape(rows, -1)
        return [py_dot(v, w[r]) for r in range(rows)]

    def rope(v, p):
        half = hd // 2
        for i in range(half):
            freq = 1.0 / math.pow(float(f32(cfg.rope_theta)), (2 * i) / hd)
            c, s = f32(math.cos(p * freq)), f32(math.sin(p * freq))
            a, b = v[i], v[i + half]
            v[i] = f32(f32(a * c) - f32(b * s))
            v[i + half] = f32(f32(a * s) + f32(b * c))

    active = min(pos + 1, cfg.max_seq)
    scale = f32(1.0 / O.math_sqrt(float(hd)))
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        xb = rms(x, W[p + "attn_norm.weight"][1])
        q = mm(p + "attn_q.weight", xb, cfg.q_dim)
        k = mm(p + "attn_k.weight", xb, cfg.kv_dim)
        v = mm(p + "attn_v.weight", xb, cfg.kv_dim)
        for vec, bname in ((q, "attn_q.bias"), (k, "attn_k.bias"), (v, "attn_v.bias")):  # forward.go:211-225
            if p + bname in W:
                for i, b in enumerate(W[p + bname][1]):
                    vec[i] = f32(vec[i] + f32(b))
        for h in range(cfg.n_heads):
            seg = q[h * hd:(h + 1) * hd]; rope(seg, pos); q[h * hd:(h + 1) * hd] = seg
        for h in range(cfg.n_kv_heads):
            seg = k[h * hd:(h + 1) * hd]; rope(seg, pos); k[h * hd:(h + 1) * hd] = seg
        slot = pos % cfg.max_seq
        kc[l][slot] = k
        vc[l][slot] = v
        att = [f32(0)] * cfg.q_dim
        for h in range(cfg.n_heads):
            g = h // kv_mul
            sc = [f32(py_dot(q[h * hd:(h + 1) * hd], kc[l][t][g * hd:(g + 1) * hd]) * scale) for t in range(active)]
            m = sc[0]
            for s in sc[1:]:
                if s > m:
                    m = s
            tot = f32(0)
            for t in range(active):
                sc[t] = f32(math.exp(float(f32(sc[t] - m))))
                tot = f32(tot + sc[t])
            inv = f32(f32(1.0) / tot)
            sc = [f32(s * inv) for s in sc]
            for t in range(active):
                for d in range(hd):
                    att[h * hd + d] = f32(att[h * hd + d] + f32(sc[t] * vc[l][t][g * hd + d]))
        proj = mm(p + "attn_output.weight", att, dim)
        x = [f32(a + b) for a, b in zip(x, proj)]
        xb = rms(x, W[p + "ffn_norm.weight"][1])
        gt = mm(p + "ffn_gate.weight", xb, cfg.hidden)
        up = mm(p + "ffn_up.weight", xb, cfg.hidden)
        gt = [f32(f32(a / f32(f32(1.0) + f32(math.exp(-float(a))))) * b) for a, b in zip(gt, up)]
        down = mm(p + "ffn_down.weight", gt, dim)
        x = [f32(a + b) for a, b in zip(x, down)]
    xb = rms(x, W["output_norm.weight"][1])
    return np.array(mm("output.weight", xb, cfg.vocab), np.float32)


def f32_model(cfg, seed):
    """A model with float32 tensors drawn like synth_model's."""
    rng = np.random.default_rng(seed)
    T = {"token_embd.weight": (G.TYPE_F32, rng.normal(0, 0.5, (cfg.vocab, cfg.dim)).astype(np.float32))}
    for l in range(cfg.n_layers):
        for name, (r, c) in synth.layer_shapes(cfg).items():
            T[synth.layer_tensor(l, name)] = (G.TYPE_F32, rng.normal(0, 0.2, (r, c)).astype(np.float32))
        for name in ("attn_norm", "ffn_norm"):
            T[f"blk.{l}.{name}.weight"] = (G.TYPE_F32, rng.uniform(0.5, 1.5, cfg.dim).astype(np.float32))
    T["output_norm.weight"] = (G.TYPE_F32, np.ones(cfg.dim, np.float32))
    T["output.weight"] = (G.TYPE_F32, rng.normal(0, 0.2, (cfg.vocab, cfg.dim)).astype(np.float32))
    return T


def test_forward_matches_python_restatement():
    cfg = synth.LlamaConfig(n_layers=2, dim=16, hidden=24, n_heads=4, n_kv_heads=2, vocab=11, max_seq=4,
                            rope_theta=10000.0)
    W = f32_model(cfg, 3)
    ref = O.RefModel(cfg, W, nthreads=2)
    kc = [[[f32(0)] * cfg.kv_dim for _ in range(cfg.max_seq)] for _ in range(cfg.n_layers)]
    vc = [[[f32(0)] * cfg.kv_dim for _ in range(cfg.max_seq)] for _ in range(cfg.n_layers)]
    for pos, tok in enumerate([1, 5, 7, 2, 9, 3]):  # wraps the 4-slot cache
        got = ref.forward(tok, pos)
        want = py_forward(cfg, W, kc, vc, tok, pos)
        assert np.array_equal(got, want), f"pos {pos}: max diff {np.abs(got - want).max()}"


def test_forward_with_qkv_biases_matches_python_restatement():
    """Qwen 2-style Q/K/V biases (forward.go:211-225), added after the
    projections in both restatements; they change the logits."""
    cfg = synth.LlamaConfig(n_layers=2, dim=16, hidden=24, n_heads=4, n_kv_heads=2, vocab=11, max_seq=4,
                            rope_theta=10000.0)
    W = f32_model(cfg, 6)
    rng = np.random.default_rng(8)
    plain = O.RefModel(cfg, dict(W), nthreads=1)
    for l in range(cfg.n_layers):
        for name, n in (("attn_q", cfg.q_dim), ("attn_k", cfg.kv_dim), ("attn_v", cfg.kv_dim)):
            W[f"blk.{l}.{name}.bias"] = (G.TYPE_F32, rng.normal(0, 0.5, n).astype(np.float32))
    ref = O.RefModel(cfg, W, nthreads=2)
    kc = [[[f32(0)] * cfg.kv_dim for _ in range(cfg.max_seq)] for _ in range(cfg.n_layers)]
    vc = [[[f32(0)] * cfg.kv_dim for _ in range(cfg.max_seq)] for _ in range(cfg.n_layers)]
    for pos, tok in enumerate([4, 1, 9, 3, 0]):
        got = ref.forward(tok, pos)
        want = py_forward(cfg, W, kc, vc, tok, pos)
        assert np.array_equal(got, want), f"pos {pos}: max diff {np.abs(got - want).max()}"
        assert not np.array_equal(got, plain.forward(tok, pos))
    bad = dict(W)
    bad["blk.0.attn_k.bias"] = (G.TYPE_F32, np.zeros(cfg.kv_dim + 1, np.float32))
    with pytest.raises(ValueError):
        O.RefModel(cfg, bad)


def test_kv_cache_wrap_slot():  # engine_test.go:194-217: pos 9 of a 4-slot cache lands in slot 1
    cfg = synth.LlamaConfig(n_layers=1, dim=16, hidden=16, n_heads=2, n_kv_heads=2, vocab=6, max_seq=4)
    ref = O.RefModel(cfg, f32_model(cfg, 4), nthreads=1)
    for pos in range(10):
        before = ref.key.reshape(cfg.max_seq, cfg.kv_dim).copy()
        ref.forward(pos % cfg.vocab, pos)
        after = ref.key.reshape(cfg.max_seq, cfg.kv_dim)
        changed = [s for s in range(cfg.max_seq) if not np.array_equal(before[s], after[s])]
        assert changed == [pos % cfg.max_seq]


def synthetic_engine_model():
    """engine_test.go:16-157: 1 layer, dim 16, FFN 32, 2 heads (2 KV), vocab 6,
    every weight 0.1 (F32); no rope.freq_base, so the loader's 500000
    (engine.go:112)."""
    cfg = synth.LlamaConfig(n_layers=1, dim=16, hidden=32, n_heads=2, n_kv_heads=2, vocab=6, max_seq=32,
                            rope_theta=500000.0)
    T = {}
    for name, (r, c) in [("token_embd.weight", (cfg.vocab, cfg.dim)), ("output.weight", (cfg.vocab, cfg.dim))]:
        T[name] = (G.TYPE_F32, np.full((r, c), 0.1, np.float32))
    for name, (r, c) in synth.layer_shapes(cfg).items():
        T[synth.layer_tensor(0, name)] = (G.TYPE_F32, np.full((r, c), 0.1, np.float32))
    for name in ("blk.0.attn_norm.weight", "blk.0.ffn_norm.weight", "output_norm.weight"):
        T[name] = (G.TYPE_F32, np.full(cfg.dim, 0.1, np.float32))
    return cfg, T


def test_synthetic_engine_model_generates():  # engine_test.go:159-192
    cfg, T = synthetic_engine_model()
    ids, _m, logits = O.RefModel(cfg, T, nthreads=1).greedy([1, 2, 3], 3)
    assert len(ids) == 3 and np.isfinite(logits).all()
    assert list(ids) == [0, 0, 0]  # identical logits: the first maximum wins
