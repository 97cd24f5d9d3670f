"""Generates the whole-model greedy-decode goldens: the CPU oracle's
Engine.Forward (oracle/, the restatement of pkg/engine/forward.go's CPU
branch) run over a seeded synthetic model, prompt token by token, then
greedy steps.

  7b   tests/golden/decode_llama7b.npz   config 4: Llama-2-7B shape (32
       layers, d=4096, 32 heads, FFN 11008, vocab 32000, RoPE base 10000,
       eps 1e-5), Q4_K layers and token table, Q6_K lm_head, unit norms;
       synth.synth_model(seed=4); 128-token prompt (numpy seed 40), 64 steps.
  70b  tests/golden/decode_llama70b.npz  config 5: Llama-3-70B shape (80
       layers, d=8192, 64 query / 8 KV heads, FFN 28672, vocab 128256, RoPE
       base 500000), every matrix Q4_K; synth.synth_model(seed=5); 512-token
       prompt (numpy seed 50), 64 steps.

Each file stores the prompt, the 64 ids, the oracle's top-2 logit margin at
each step, the last step's logits and a digest of the model bytes (to catch
a changed generator).  The weights come from gi_quantize_seeded, whose bytes
gi_synth_weights reproduces on the GPU, so the GPU tests draw the same model
on the device.  Run from the repository root:
    python tests/golden/make_decode_golden.py 7b    (a few minutes on 8 cores)
    python tests/golden/make_decode_golden.py 70b   (about 2.3 hours on 8
                                                      cores, 40 GB of memory)"""
import hashlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "go-infer_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
import synth  # noqa: E402

# name: (config, weight seed, prompt seed, prompt length, greedy steps, file)
GOLDENS = {
    "7b": (synth.LLAMA2_7B, 4, 40, 128, 64, "decode_llama7b.npz"),
    "70b": (synth.LLAMA3_70B, 5, 50, 512, 64, "decode_llama70b.npz"),
}


def draw_order(cfg) -> list:
    """The model's tensor names in the order synth_model draws them (token
    table, each layer's seven matrices and two norms, output norm, head)."""
    names = ["token_embd.weight"]
    for l in range(cfg.n_layers):
        names += [synth.layer_tensor(l, role) for role in synth.LAYER_MATS]
        names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight"]
    return names + ["output_norm.weight", "output.weight"]


def digest_update(h, qt: int, raw: np.ndarray) -> None:
    h.update(np.int64(qt).tobytes())
    h.update(np.ascontiguousarray(raw).view(np.uint8).reshape(-1)[:: 4099].tobytes())


def model_digest(host) -> str:
    """SHA-256 over every 4099th byte of each tensor, tensors in draw order.
    Names are not hashed, so renaming tensors keeps the digest; changed
    weight bytes, types or shapes change it."""
    h = hashlib.sha256()
    for name in draw_order(host.cfg):
        qt, arr = host.tensors[name]
        digest_update(h, qt, arr)
    return h.hexdigest()


def device_model_digest(dev) -> str:
    """model_digest of a synth.DeviceModel, reading one tensor back at a time."""
    h = hashlib.sha256()
    for name in draw_order(dev.cfg):
        digest_update(h, dev.types[name], dev.raw(name))
    return h.hexdigest()


def prompt_of(which: str) -> np.ndarray:
    cfg, _seed, pseed, plen, _steps, _f = GOLDENS[which]
    return np.random.default_rng(pseed).integers(0, cfg.vocab, plen).astype(np.int32)


def main(which: str):
    cfg, seed, _pseed, _plen, steps, fname = GOLDENS[which]
    t0 = time.time()
    host = synth.synth_model(cfg, seed=seed, threads=os.cpu_count() or 1)
    digest = model_digest(host)
    t1 = time.time()
    print(f"model drawn in {t1 - t0:.1f} s, digest {digest}", flush=True)
    prompt = prompt_of(which)
    ref = O.RefModel(cfg, host.tensors)
    ids, margins, logits = ref.greedy(prompt, steps, progress=lambda i, n: print(
        f"  forward {i}/{n} ({time.time() - t1:.0f} s)", flush=True) if i % 16 == 0 else None)
    t2 = time.time()
    out = os.path.join(ROOT, "tests", "golden", fname)
    np.savez_compressed(out, prompt=prompt, ids=ids, margins=margins, last_logits=logits,
                        digest=np.array(digest), seed=np.array(seed), prompt_seed=np.array(_pseed))
    print(f"model {t1 - t0:.1f} s, oracle {t2 - t1:.1f} s for {len(prompt) + steps - 1} forward steps; "
          f"min margin {margins.min():.4g}; wrote {out}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "7b")
