"""Generates tests/golden/decode_llama7b.npz: the CPU oracle's greedy decode
of the config-4 model (Llama-2-7B shape: 32 layers, d=4096, 32 heads, FFN
11008, vocab 32000, RoPE base 10000, eps 1e-5; weights N(0, 0.02) from
synth.synth_model(seed=4): Q4_K layers and token table, Q6_K lm_head, unit
norms) for a 128-token prompt drawn with numpy seed 40, then 64 greedy
steps.  Stores the prompt, the 64 ids, the oracle's top-2 logit margin at
each step, the last step's logits and a digest of the model bytes (to catch
a changed generator).  Run from the repository root:
    python tests/golden/make_decode_golden.py
(about 1-2 s per token per 8 host cores)."""
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


def draw_order(cfg) -> list:
    """The model's tensor names in the order synth_model draws them (token
    table, each layer's seven matrices and two norms, output norm, head)."""
    names = ["token_embd.weight"]
    for l in range(cfg.n_layers):
        names += [synth.layer_tensor(l, role) for role in synth.LAYER_MATS]
        names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight"]
    return names + ["output_norm.weight", "output.weight"]


def model_digest(host) -> str:
    """SHA-256 over every 4099th byte of each tensor, tensors in draw order.
    Names are not hashed, so renaming tensors keeps the digest; changed
    weight bytes, types or shapes change it."""
    h = hashlib.sha256()
    for name in draw_order(host.cfg):
        qt, arr = host.tensors[name]
        h.update(np.int64(qt).tobytes())
        h.update(np.ascontiguousarray(arr).view(np.uint8)[:: 4099].tobytes())
    return h.hexdigest()


def main():
    cfg = synth.LLAMA2_7B
    t0 = time.time()
    host = synth.synth_model(cfg, seed=4)
    digest = model_digest(host)
    t1 = time.time()
    prompt = np.random.default_rng(40).integers(0, cfg.vocab, 128).astype(np.int32)
    ids, margins, logits = O.RefModel(cfg, host.tensors).greedy(prompt, 64)
    t2 = time.time()
    out = os.path.join(ROOT, "tests", "golden", "decode_llama7b.npz")
    np.savez_compressed(out, prompt=prompt, ids=ids, margins=margins, last_logits=logits,
                        digest=np.array(digest), seed=np.array(4), prompt_seed=np.array(40))
    print(f"model {t1 - t0:.1f} s, oracle {t2 - t1:.1f} s for {len(prompt) + 63} forward steps; "
          f"min margin {margins.min():.4f}; wrote {out}")


if __name__ == "__main__":
    main()
