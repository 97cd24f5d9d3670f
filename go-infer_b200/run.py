"""Command-line runner: greedy decode of a synthetic Llama-shaped model, or
one prefill dequant-GEMM, on one GPU.

The counterpart of go-infer's `go-infer run` for this engine's path: it
builds the model from seeded synthetic GGUF tensors (no checkpoints are
available), runs `--prompt` prompt tokens and `--steps` greedy steps through
the device-resident decode loop and prints the ids and the device time per
generated token.

    python go-infer_b200/run.py decode --model llama2-7b --prompt 128 --steps 64
    python go-infer_b200/run.py decode --model llama3-70b --prompt 40 --steps 2
    python go-infer_b200/run.py decode --gguf model.gguf --prompt 16 --steps 32
    python go-infer_b200/run.py export --model llama2-7b --layers 2 --out small.gguf
    python go-infer_b200/run.py prefill --type q4_k --rows 4096 --cols 4096 --batch 512 --reps 3
    python go-infer_b200/run.py gemv --type q6_k --rows 32000 --cols 4096 --reps 20
"""
from __future__ import annotations

import argparse
import dataclasses
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import goinfer_cuda as G  # noqa: E402
import synth  # noqa: E402

MODELS = {"llama2-7b": synth.LLAMA2_7B, "llama3-70b": synth.LLAMA3_70B}
TYPES = {"q4_k": G.TYPE_Q4_K, "q6_k": G.TYPE_Q6_K, "q8_0": G.TYPE_Q8_0}


def decode(args) -> None:
    if args.gguf:  # a GGUF file (Q4_K / Q6_K / Q8_0 / F32 tensors under go-infer's names)
        import gguf
        with gguf.GGUFReader(args.gguf) as r:
            host = gguf.host_model(r, max_seq=args.prompt + args.steps)
            dev = synth.DeviceModel(host)
        cfg = dev.cfg
    else:
        cfg = MODELS[args.model]
        if args.layers:
            cfg = dataclasses.replace(cfg, n_layers=args.layers)
        cfg = dataclasses.replace(cfg, max_seq=max(cfg.max_seq, args.prompt + args.steps))
        dev = synth.DeviceModel.synth_on_device(cfg, seed=args.seed)
    model = dev.model()
    try:
        if args.persistent:
            model.set_persistent(True)
        prompt = np.random.default_rng(args.seed * 10).integers(0, cfg.vocab, args.prompt).astype(np.int32)
        ids, _logits, ms = model.generate(prompt, args.steps)
        per = ms / max(args.steps - 1, 1)
        print(f"ids {ids.tolist()}")
        print(f"decode {per * 1e3:.1f} us/token ({1e3 / per:.1f} tok/s) over {args.steps - 1} steps")
    finally:
        model.close()
        dev.close()


def export(args) -> None:
    """Write the seeded synthetic model (drawn on the host) as a GGUF file."""
    import gguf
    cfg = MODELS[args.model]
    if args.layers:
        cfg = dataclasses.replace(cfg, n_layers=args.layers)
    gguf.save_model(synth.synth_model(cfg, seed=args.seed), args.out)
    print(f"wrote {args.out}")


def prefill(args) -> None:
    import torch
    qt = TYPES[args.type]
    wb = G.synth_buffer(qt, args.seed, 0.02, args.rows, args.cols)
    x = torch.randn(args.batch, args.cols, device="cuda")
    y = torch.empty(args.batch, args.rows, device="cuda")
    st = torch.cuda.Stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    G.set_prefill_pair(args.pair)

    def run():
        G.gemm_dev(qt, y.data_ptr(), x.data_ptr(), wb.device_ptr, wb.nbytes, args.batch, args.rows, args.cols,
                   st.cuda_stream)

    try:
        run()  # the first call sizes the library's workspace
        st.synchronize()
        with torch.cuda.stream(st):
            e0.record()
            for _ in range(args.reps):
                run()
            e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.reps
        print(f"prefill {args.type} {args.batch}x{args.rows}x{args.cols}{' (CTA pairs)' if args.pair else ''}: "
              f"{us:.1f} us ({2 * args.batch * args.rows * args.cols / us / 1e6:.1f} TFLOP/s)")
    finally:
        G.set_prefill_pair(False)
        G.ReleaseBuffer(wb)


def gemv(args) -> None:
    """Decode GEMVs y = W x of one shape, rotating over enough weight copies
    that every launch streams its matrix from HBM (> 2 x the 126 MB L2)."""
    import torch
    qt = TYPES[args.type]
    nbytes = args.rows * G.row_bytes(qt, args.cols)
    ncopy = max(1, -(-252_000_000 // nbytes))
    bufs = [G.synth_buffer(qt, args.seed + c, 0.02, args.rows, args.cols) for c in range(ncopy)]
    x = torch.randn(args.cols, device="cuda")
    y = torch.empty(args.rows, device="cuda")
    st = torch.cuda.Stream()
    G.set_q6k_mma(not args.cuda_cores)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def run(i):
        b = bufs[i % ncopy]
        G.gemv_dev(qt, y.data_ptr(), x.data_ptr(), b.device_ptr, b.nbytes, args.rows, args.cols, st.cuda_stream)

    try:
        for i in range(3):
            run(i)
        st.synchronize()
        with torch.cuda.stream(st):
            e0.record()
            for i in range(args.reps):
                run(i)
            e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.reps
        print(f"gemv {args.type} {args.rows}x{args.cols}: {us:.2f} us per launch "
              f"({(nbytes + 4 * (args.rows + args.cols)) / us / 1e3:.1f} GB/s, {ncopy} weight copies)")
    finally:
        G.set_q6k_mma(True)
        for b in bufs:
            G.ReleaseBuffer(b)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    d = sub.add_parser("decode")
    d.add_argument("--model", choices=sorted(MODELS), default="llama2-7b")
    d.add_argument("--layers", type=int, default=0, help="override the layer count")
    d.add_argument("--prompt", type=int, default=128)
    d.add_argument("--steps", type=int, default=64)
    d.add_argument("--seed", type=int, default=4)
    d.add_argument("--gguf", default="", help="decode the model of this GGUF file instead")
    d.add_argument("--persistent", action="store_true", help="every layer of a step in one persistent launch")
    x = sub.add_parser("export")
    x.add_argument("--model", choices=sorted(MODELS), default="llama2-7b")
    x.add_argument("--layers", type=int, default=0, help="override the layer count")
    x.add_argument("--seed", type=int, default=4)
    x.add_argument("--out", required=True)
    p = sub.add_parser("prefill")
    p.add_argument("--type", choices=sorted(TYPES), default="q4_k")
    p.add_argument("--rows", type=int, default=4096)
    p.add_argument("--cols", type=int, default=4096)
    p.add_argument("--batch", type=int, default=512)
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--seed", type=int, default=8)
    p.add_argument("--pair", action="store_true", help="CTA pairs (cta_group::2 MMAs) instead of single CTAs")
    v = sub.add_parser("gemv")
    v.add_argument("--type", choices=sorted(TYPES), default="q4_k")
    v.add_argument("--rows", type=int, default=11008)
    v.add_argument("--cols", type=int, default=4096)
    v.add_argument("--reps", type=int, default=20)
    v.add_argument("--seed", type=int, default=20)
    v.add_argument("--cuda-cores", action="store_true", help="Q6_K on the CUDA-core kernel")
    args = ap.parse_args()
    if args.cmd == "export":  # host only
        export(args)
        return
    G.Init(0)
    if not G.IsAvailable():
        raise SystemExit("libgoinfer_cuda: no CUDA device")
    {"decode": decode, "prefill": prefill, "gemv": gemv}[args.cmd](args)


if __name__ == "__main__":
    main()
