"""Benchmark of the B200 quantised-GEMV engine on BASELINE.json's headline config.

Workload: Q4_K GEMV, batch 1, Llama-7B FFN shapes.
One step = the three FFN projections of one layer: gate and up
(11008x4096) on the same activation, then down (4096x11008) -- 3 x
25,422,848 algorithmic bytes (raw Q4_K weights + fp32 x + fp32 y).
Weights are seeded N(0, 0.02) fp32 quantised by the library's Q4_K
quantiser; activations seeded N(0, 1).  Steps rotate over 8 copies of the
layer's weights (610 MB > the 126 MB L2), so every launch streams its
matrix from HBM.

  value    device-timed throughput (CUDA events, max over ranks) of K steps
           captured in one CUDA graph, inputs resident in HBM;
  e2e      the same metric through the reference-facing C-ABI call
           (gi_cuda_gemv_buf, metal_gemv_buf's counterpart) with x copied in
           from pinned host memory and y read back every call;
  roofline the Q4_K GEMV kernel: algorithmic bytes per launch / average
           launch time, against the measured HBM copy bandwidth;
  cpu_baseline  the CPU restatement of go-infer's GEMVEngine.MatMulQ4_K on
           the host cores (rank 0, N=1 only);
  step_distribution  p10 / p50 / p90 of the step time over 20 replays of a
           100-step graph, taken after the timed region (this rank).

--impl reference times go-infer's CPU path (the C restatement in oracle/;
the Go code cannot be built here) on the same workload and prints the same
line with "impl": "reference".

Multi-GPU: one process per GPU (torchrun).  At N > 1 the step is config
2's FFN block split Megatron-style across the ranks (gate/up rows and the
matching down columns, in whole 256-column Q4_K blocks), the all-reduce of
the down partials fused into the down GEMV's epilogue over NVLink
(gi_cuda_ffn_dev): strong scaling, value = the FFN's bytes / max rank time.
At N=1 ffn_block times the same FFN block on one GPU, the reference point of
those lines.

decode   (the metric's second half) greedy decode tokens/s of the Llama-
         shaped synthetic models, device-timed (CUDA events around the
         generation steps, max over ranks): config 5 (Llama-3-70B shape,
         512-token prompt, 64 steps) tensor-parallel over the N ranks, and at
         N=1 config 4 (Llama-2-7B shape, 128-token prompt, 64 steps) with a
         bounded CPU-oracle sample of the same decode step; prefill (config
         3, 512 tokens x 4096 columns) at N=1.  "persistent" holds the same
         generations with every layer of a step in one persistent launch
         (gi_cuda_model_set_persistent) -- for config 5 always at N > 1, and
         with --persistent also at N=1 and for config 4 -- and whether
         their ids equal the per-layer launches'.  gemv_other times the Q6_K
         lm_head shapes on both Q6_K kernels (the int8 tensor-core default and
         "_cuda_cores").
--e2e-batch  runs the e2e step's three calls inside gi_cuda_begin_batch /
         gi_cuda_end_batch (go-infer's metal.BeginBatch/EndBatch: one wait
         per step), after checking that it reproduces the call-by-call step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "go-infer_b200"))

METRIC = "Q4_K GEMV HBM GB/s (% of 8 TB/s); decode tokens/s at 1/2/4/8 B200"
GATE = (11008, 4096)
DOWN = (4096, 11008)
NCOPIES = 8
Q4K_ROW = {4096: 16 * 144, 11008: 43 * 144}


def gemv_bytes(rows, cols):
    return rows * Q4K_ROW[cols] + 4 * (rows + cols)


STEP_BYTES = 2 * gemv_bytes(*GATE) + gemv_bytes(*DOWN)  # 76,268,544
WORKLOAD = ("config2: Q4_K GEMV batch 1, Llama-7B FFN shapes; step = gate and up 11008x4096 "
            "(one launch, shared activation) and down 4096x11008 (second launch)")


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def seeded(seed, shape, std):
    return np.random.default_rng(seed).normal(0.0, std, size=shape).astype(np.float32)


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks rather than fail
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.005)

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if mask & bit and bit != 0x1:
                    self.reasons.add(name)
        except Exception:
            pass

    def __enter__(self):
        if self.nv:
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.nv:
            self._stop.set()
            self.t.join()
            self._sample()

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the Q4_K GEMV from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemv_q4k_config2.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


def cpu_matrices(row_frac=1.0):
    """The step's three Q4_K matrices (their first row_frac of the rows) for
    the CPU legs, quantised by oracle/quantize_np.py, the byte-identical
    numpy restatement of the library's Q4_K quantiser: no CPU leg loads the
    product library."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import quantize_np
    mats = []
    for seed, (rows, cols) in ((3, GATE), (4, GATE), (5, DOWN)):
        r = max(16, int(rows * row_frac))
        mats.append((quantize_np.quantize_q4_k(seeded(seed, (rows, cols), 0.02)[:r]), r, cols))
    return mats


def cpu_port_gemv_gbs(budget_s, row_frac=1.0):
    """go-infer's CPU path (oracle restatement), all host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build() if not os.path.exists(O.LIB_PATH) else None
    threads = os.cpu_count() or 1
    mats = cpu_matrices(row_frac)
    xg, xd = seeded(101, GATE[1], 1.0), seeded(102, DOWN[1], 1.0)
    done_bytes, t0, steps = 0, time.perf_counter(), 0
    while True:
        for (raw, r, cols), x in zip(mats, (xg, xg, xd)):
            O.matmul(O.GGML_Q4_K, x, raw, r, cols, nthreads=threads)
            done_bytes += r * Q4K_ROW[cols] + 4 * (r + cols)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    sample = (f"{steps} FFN steps (gate+up+down) over {row_frac:.0%} of the rows, "
              f"{el:.1f} s, {threads} threads")
    return done_bytes / el / 1e9, threads, sample


TP_WORKLOAD = ("config2 FFN block, Llama-7B shapes, Megatron-split: x += down(SwiGLU(gate(n), up(n))), "
               "n = RMSNorm(x); gate/up 11008x4096 column-split and down 4096x11008 row-split in whole 256-column "
               "blocks; two launches per rank, the all-reduce of the down partials fused into its epilogue")


def step_config(world):
    """The line's config, the same in both arms."""
    return {"workload": WORKLOAD if world == 1 else TP_WORKLOAD,
            "parallelism": f"tensor parallel x{world}" if world > 1 else "single",
            "l2": (f"inputs larger than L2: GPU arm {NCOPIES} rotating weight copies "
                   f"({NCOPIES * STEP_BYTES / 1e6:.0f} MB > 126 MB L2); CPU arm {STEP_BYTES / 1e6:.0f} MB per step"),
            "graph": "GPU arm: K steps in one CUDA graph, programmatic dependent launch; CPU arm: one call per matrix"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    # size the sample so warmup + steps finish within ~2 minutes
    probe, _, _ = cpu_port_gemv_gbs(0.0, 1.0)
    t_step = STEP_BYTES / (probe * 1e9)
    frac = min(1.0, 120.0 / max(1e-9, t_step * (args.steps + args.warmup)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    mats = cpu_matrices(frac)
    xg, xd = seeded(101, GATE[1], 1.0), seeded(102, DOWN[1], 1.0)
    for _ in range(args.warmup):
        for (raw, r, cols), x in zip(mats, (xg, xg, xd)):
            O.matmul(O.GGML_Q4_K, x, raw, r, cols, nthreads=threads)
    nbytes = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for (raw, r, cols), x in zip(mats, (xg, xg, xd)):
            O.matmul(O.GGML_Q4_K, x, raw, r, cols, nthreads=threads)
            nbytes += r * Q4K_ROW[cols] + 4 * (r + cols)
    el = time.perf_counter() - t0
    gbs = nbytes / el / 1e9
    sample = (f"{args.steps} steps, each gate+up+down over {frac:.1%} of the rows "
              f"(GEMVEngine.MatMulQ4_K restated in C, contiguous row chunks, {threads} threads)")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded)", "config": step_config(world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample, "rows_sampled": round(frac, 4), "nproc": os.cpu_count(),
                         "cpu_model": cpu_model()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_section(args, world, rank, local, pg):
    """Config 5 on all ranks (tensor parallel), config 4 / prefill / CPU sample at N=1."""
    import dataclasses
    import torch
    import goinfer_cuda as G
    import synth
    import tp

    dev = torch.device("cuda", local)
    out = {}

    def max_over_ranks(v):
        t = torch.tensor([float(v)], device=dev)
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    def persistent_run(model, prompt, ids_ref):
        """The same generation with every layer of a step in one persistent
        launch.  A failure (a shape the plan does not take, a bounded wait
        that gave up: the same on every rank) is reported in the line; the
        per-layer numbers stand."""
        try:
            model.set_persistent(True)
            model.reset()
            model.generate(prompt, 64)
            model.reset()
            ids_p, _l, ms_p = model.generate(prompt, 64)
        except G.GoInferCudaError as exc:
            try:
                model.set_persistent(False)
            except G.GoInferCudaError:
                pass
            model.reset()
            return {"error": str(exc)[:200]}
        ms_p = max_over_ranks(ms_p)
        model.set_persistent(False)
        return {"tok_s": round(63 / (ms_p / 1e3), 2), "ms_per_token": round(ms_p / 63, 4),
                "ids_equal_per_layer": bool(np.array_equal(ids_p, ids_ref))}

    # config 5: Llama-3-70B shape, weights drawn on the device (seeded)
    cfg5 = synth.LLAMA3_70B
    if world > 1:
        tp.connect(rank, world, cfg5.dim)
    dm = synth.DeviceModel.synth_on_device(cfg5, seed=5, rank=rank, world=world)
    model = dm.model(tp_rank=rank, tp_world=world)
    prompt5 = np.random.default_rng(50).integers(0, cfg5.vocab, 512).astype(np.int32)
    ids, _l, ms = model.generate(prompt5, 64)
    model.reset()
    ids, _l, ms = model.generate(prompt5, 64)
    ms = max_over_ranks(ms)
    w_bytes = sum(b.nbytes for b in dm.bufs.values()) - dm.bufs["token_embd.weight"].nbytes
    # Under tensor parallelism the persistent kernel is always timed too (on
    # B200 it was ahead of the per-layer launches at TP2 and 22 % ahead at TP4).
    pers5 = persistent_run(model, prompt5, ids) if (args.persistent or world > 1) else None
    model.close()
    dm.close()
    if world > 1:
        pg.barrier()
        G.tp_close()
    out["config5"] = {"model": "Llama-3-70B shape (80 x d8192, 64/8 heads, FFN 28672, vocab 128256), every matrix Q4_K",
                      "parallelism": f"tensor parallel x{world}" if world > 1 else "single GPU",
                      "prompt": 512, "steps": 64, "tok_s": round(63 / (ms / 1e3), 2),
                      "ms_per_token": round(ms / 63, 4),
                      "weight_bytes_per_token_per_gpu": int(w_bytes),
                      "ids_head": [int(i) for i in ids[:8]]}
    if pers5:
        out["config5"]["persistent"] = pers5
    if world > 1:
        return out
    # config 4: Llama-2-7B shape
    cfg4 = synth.LLAMA2_7B
    dm = synth.DeviceModel.synth_on_device(cfg4, seed=4)
    model = dm.model()
    prompt4 = np.random.default_rng(40).integers(0, cfg4.vocab, 128).astype(np.int32)
    model.generate(prompt4, 64)
    model.reset()
    ids4, _l, ms4 = model.generate(prompt4, 64)
    w_bytes = sum(b.nbytes for b in dm.bufs.values()) - dm.bufs["token_embd.weight"].nbytes
    out["config4"] = {"model": "Llama-2-7B shape (32 x d4096, 32 heads, FFN 11008, vocab 32000), Q4_K + Q6_K head",
                      "prompt": 128, "steps": 64, "tok_s": round(63 / (ms4 / 1e3), 2),
                      "ms_per_token": round(ms4 / 63, 4), "weight_bytes_per_token": int(w_bytes),
                      "effective_gbs": round(w_bytes / (ms4 / 63 / 1e3) / 1e9, 1)}
    if args.persistent:
        out["config4"]["persistent"] = persistent_run(model, prompt4, ids4)
    if not args.no_cpu_baseline:
        # the CPU restatement of Engine.Forward on the same bytes, a bounded sample
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        tensors = {name: (dm.types[name], dm.raw(name)) for name in dm.bufs}
        ref = O.RefModel(cfg4, tensors)
        t0 = time.perf_counter()
        nsteps = 0
        while nsteps < 2 or (time.perf_counter() - t0 < args.cpu_seconds and nsteps < 8):
            ref.forward(int(prompt4[nsteps]), nsteps)
            nsteps += 1
        cpu_s = (time.perf_counter() - t0) / nsteps
        out["config4"]["cpu_baseline"] = {"tok_s": round(1.0 / cpu_s, 4), "cores": os.cpu_count(), "kind": "port",
                                          "sample": f"{nsteps} decode steps of the same model (oracle ref_forward)",
                                          "cpu_model": cpu_model()}
        del tensors, ref
    model.close()
    dm.close()
    # config 1 (Q8_0 4096x4096) and the Q6_K lm_head shapes: HBM GB/s of the
    # plain decode GEMV, rotating weight copies past the L2, graph + PDL
    peak, _kind = measured_peak()
    other = {}
    # Q6_K: the int8 tensor-core kernel (the default) and the CUDA-core one
    shapes = [("q8_0_config1_4096x4096", G.TYPE_Q8_0, 4096, 4096, True),
              ("q6_k_lm_head_32000x4096", G.TYPE_Q6_K, 32000, 4096, True),
              ("q6_k_lm_head_128256x8192", G.TYPE_Q6_K, 128256, 8192, True)]
    shapes += [(n + "_cuda_cores", qt, r, c, False) for n, qt, r, c, _m in shapes if qt == G.TYPE_Q6_K]
    for name, qt, rows, cols, mma in shapes:
        G.set_q6k_mma(mma)
        wbytes = rows * G.row_bytes(qt, cols)
        ncopy = max(2, int(2 * 126e6 / wbytes) + 1)
        bufs = [G.synth_buffer(qt, 20 + c, 0.02, rows, cols) for c in range(ncopy)]
        xv = torch.randn(cols, device=dev)
        yv = torch.empty(rows, device=dev)
        nl = 200
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream().cuda_stream
            for i in range(nl):
                b = bufs[i % ncopy]
                G.gemv_dev(qt, yv.data_ptr(), xv.data_ptr(), b.device_ptr, b.nbytes, rows, cols, cs)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / nl
        gbs = (wbytes + 4 * (rows + cols)) / us / 1e3
        other[name] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        del graph
        for b in bufs:
            G.ReleaseBuffer(b)
    G.set_q6k_mma(True)
    out["gemv_other"] = other
    # config 3: prefill dequant-GEMM (512 tokens x 4096 columns)
    x = torch.randn(512, 4096, device=dev)
    st = torch.cuda.Stream()
    pre = {}
    for name, qt, rows, seed in (("q4k_4096", G.TYPE_Q4_K, 4096, 8), ("q4k_11008", G.TYPE_Q4_K, 11008, 9),
                                 ("q6k_32000", G.TYPE_Q6_K, 32000, 10), ("q8_0_4096", G.TYPE_Q8_0, 4096, 1)):
        wb = G.synth_buffer(qt, seed, 0.02, rows, 4096)
        y = torch.empty(512, rows, device=dev)
        run = lambda: G.gemm_dev(qt, y.data_ptr(), x.data_ptr(), wb.device_ptr, wb.nbytes, 512, rows, 4096,
                                 st.cuda_stream)
        for _ in range(3):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record()
            for _ in range(10):
                run()
            e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 100.0
        pre[name] = {"us": round(us, 1), "tflops": round(2 * 512 * rows * 4096 / us / 1e6, 1)}
        G.ReleaseBuffer(wb)
    out["prefill_config3"] = pre
    return out


def cpu_model() -> str:
    """The host CPU's model name (recorded beside every CPU baseline)."""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def step_distribution(capture, steps_per_replay=100, replays=20, pg=None, dev=None):
    """Spread of the step time, outside the timed region: `replays` replays
    of a graph of `steps_per_replay` steps, each timed with CUDA events on
    the launching stream (this rank).  With several ranks each replay's
    start event follows a one-element all-reduce, as in time_graph.  An
    optional statistic: a failure is reported in the line, never raised."""
    import torch
    try:
        g = capture(steps_per_replay)
        g.replay()
        torch.cuda.synchronize()
        rendezvous = torch.zeros(1, device=dev) if pg else None
        per_step = []
        for _ in range(replays):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if pg:
                pg.all_reduce(rendezvous)
            a.record()
            g.replay()
            b.record()
            b.synchronize()
            per_step.append(a.elapsed_time(b) * 1e3 / steps_per_replay)
        del g
        p10, p50, p90 = np.percentile(per_step, [10, 50, 90])
        return {"us_per_step_p10": round(float(p10), 3), "us_per_step_p50": round(float(p50), 3),
                "us_per_step_p90": round(float(p90), 3), "replays": replays, "steps_per_replay": steps_per_replay}
    except Exception as exc:  # noqa: BLE001
        return {"error": f"{type(exc).__name__}: {exc}"[:200]}


def ffn_shard(world, rank):
    """(h0, hn): rank's slice of the FFN hidden dimension under the Megatron
    split, in whole 256-column Q4_K blocks (11008 = 43 blocks, so slices
    differ by at most one block)."""
    nsb = GATE[0] // 256
    b0, b1 = nsb * rank // world, nsb * (rank + 1) // world
    return 256 * b0, 256 * (b1 - b0)


def time_graph(capture, steps, warmup, pg, local, dev):
    """Device time (ms, max over ranks) of `steps` steps captured in one
    CUDA graph, after `warmup` untimed steps and one untimed replay of the
    timed graph itself; barrier and synchronize on both sides; clocks
    sampled during the timed replay.

    With several ranks the start event is recorded behind a one-element
    all-reduce on the timing stream: the ranks' timed regions then begin
    together on the devices.  Without it, the host-side skew between the
    ranks leaving the barrier (and starting the clock sampler) is timed,
    since the first step's fused all-reduce waits for the last rank to
    start (measured on two B200s: 181 us per FFN step against 21 us)."""
    import torch
    g_warm = capture(max(warmup, 3))
    g_timed = capture(steps)
    for _ in range(2):
        g_warm.replay()
    g_timed.replay()  # uploads the timed graph: its first replay is not timed
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rendezvous = torch.zeros(1, device=dev)
    with ClockSampler(local) as clocks:
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        if pg:
            pg.all_reduce(rendezvous)
        start.record()
        g_timed.replay()
        stop.record()
        torch.cuda.synchronize()
    if pg:
        pg.barrier()
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    del g_timed, g_warm
    return float(t.item()), ms, clocks.summary()


def run_ours(args):
    import torch
    import goinfer_cuda as G

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    G.Init(local)
    dev = torch.device("cuda", local)
    G.set_pdl(True)
    stream_of = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731

    # ---- config 2's FFN block, Megatron-split over the ranks (any N) --------
    # x += down(SwiGLU(gate(n), up(n))), n = RMSNorm(x): gate/up rows
    # [h0, h0 + hn) and the same columns of down on this rank; the down
    # GEMV sums the ranks' partials in its epilogue (gi_cuda_ffn_dev).
    import tp
    if world > 1:
        tp.connect(rank, world, DOWN[0])
    h0, hn = ffn_shard(world, rank)
    fw = {"gate": G.quantize(G.TYPE_Q4_K, seeded(3, GATE, 0.02)[h0:h0 + hn]),
          "up": G.quantize(G.TYPE_Q4_K, seeded(4, GATE, 0.02)[h0:h0 + hn]),
          "down": G.quantize(G.TYPE_Q4_K, np.ascontiguousarray(seeded(5, DOWN, 0.02)[:, h0:h0 + hn]))}
    rank_bytes = sum(v.nbytes for v in fw.values())
    ncopy = max(NCOPIES, -(-300_000_000 // rank_bytes))  # > 2x the 126 MB L2 on every rank
    fcopies = {k: [torch.from_numpy(v).to(dev) for _ in range(ncopy)] for k, v in fw.items()}
    norm = torch.ones(DOWN[0], device=dev)
    x_ffn = torch.from_numpy(seeded(101, GATE[1], 1.0)).to(dev)
    h = torch.empty(hn, device=dev)

    def ffn_step(i, stream):
        c = i % ncopy
        wg, wu, wd = fcopies["gate"][c], fcopies["up"][c], fcopies["down"][c]
        G.ffn_dev(x_ffn.data_ptr(), norm.data_ptr(), wg.data_ptr(), wu.data_ptr(), wd.data_ptr(), wg.numel(),
                  wu.numel(), wd.numel(), h.data_ptr(), DOWN[0], hn, 1e-5, stream)

    def capture_ffn(nsteps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            s = stream_of()
            for i in range(nsteps):
                ffn_step(i, s)
        return g

    # ---- config 2 as BASELINE states it (N=1): gate and up (one launch,
    # shared activation), then down, all on N(0, 1) activations -------------
    if world == 1:
        raws = {"gate": G.quantize(G.TYPE_Q4_K, seeded(3, GATE, 0.02)),
                "up": G.quantize(G.TYPE_Q4_K, seeded(4, GATE, 0.02)),
                "down": G.quantize(G.TYPE_Q4_K, seeded(5, DOWN, 0.02))}
        copies = {k: [torch.from_numpy(v).to(dev) for _ in range(NCOPIES)] for k, v in raws.items()}
        xg = torch.from_numpy(seeded(101, GATE[1], 1.0)).to(dev)
        xd = torch.from_numpy(seeded(102, DOWN[1], 1.0)).to(dev)
        yg = torch.empty(GATE[0], device=dev)
        yu = torch.empty(GATE[0], device=dev)
        yd = torch.empty(DOWN[0], device=dev)

        def gemv_step(i, stream):
            c = i % NCOPIES
            wg, wu, wd = copies["gate"][c], copies["up"][c], copies["down"][c]
            G.gemv_multi_dev(G.TYPE_Q4_K, [yg.data_ptr(), yu.data_ptr()], xg.data_ptr(),
                             [wg.data_ptr(), wu.data_ptr()], [wg.numel(), wu.numel()], [GATE[0], GATE[0]], GATE[1],
                             stream)
            G.gemv_dev(G.TYPE_Q4_K, yd.data_ptr(), xd.data_ptr(), wd.data_ptr(), wd.numel(), DOWN[0], DOWN[1],
                       stream)

        def capture(nsteps):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                s = stream_of()
                for i in range(nsteps):
                    gemv_step(i, s)
            return g
    else:
        capture = capture_ffn

    ms_max, ms, clocks = time_graph(capture, args.steps, args.warmup, pg, local, dev)
    value = STEP_BYTES * args.steps / (ms_max / 1e3) / 1e9  # the whole step's bytes, over all ranks
    launch_bytes = (STEP_BYTES / 2) if world == 1 else rank_bytes / 2
    launch_ms = ms / (2 * args.steps)  # this rank's average Q4_K GEMV launch
    achieved = launch_bytes / (launch_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    dist = step_distribution(capture, pg=pg, dev=dev)
    ffn_block = None
    if world == 1:  # the FFN block at N=1: the reference point of the N>1 lines
        f_ms, _f, _c = time_graph(capture_ffn, args.steps, args.warmup, None, local, dev)
        ffn_block = {"gbs": round(STEP_BYTES * args.steps / (f_ms / 1e3) / 1e9, 2),
                     "us_per_step": round(f_ms * 1e3 / args.steps, 3),
                     "what": "gi_cuda_ffn_dev: RMSNorm + gate/up + SwiGLU (one launch), down + residual (second)"}

    # ---- e2e through the reference-facing C ABI: host x (and y), resident weights
    if world == 1:
        bufs = {k: G.CreateBuffer(v) for k, v in raws.items()}
        px_g = torch.from_numpy(seeded(101, GATE[1], 1.0)).pin_memory()
        px_d = torch.from_numpy(seeded(102, DOWN[1], 1.0)).pin_memory()
        py_g, py_u = torch.empty(GATE[0]).pin_memory(), torch.empty(GATE[0]).pin_memory()
        py_d = torch.empty(DOWN[0]).pin_memory()
        hx_g, hx_d = px_g.numpy(), px_d.numpy()
        hy_g, hy_u, hy_d = py_g.numpy(), py_u.numpy(), py_d.numpy()

        def e2e_calls():
            G.MatMulBuf(G.TYPE_Q4_K, hy_g, hx_g, bufs["gate"], *GATE)
            G.MatMulBuf(G.TYPE_Q4_K, hy_u, hx_g, bufs["up"], *GATE)
            G.MatMulBuf(G.TYPE_Q4_K, hy_d, hx_d, bufs["down"], *DOWN)

        def e2e_batched():  # metal.BeginBatch / EndBatch around the step: one wait per step
            G.BeginBatch()
            e2e_calls()
            G.EndBatch()

        e2e_step = e2e_batched if args.e2e_batch else e2e_calls
        if args.e2e_batch:  # the batched step must give the call-by-call outputs, bit for bit
            e2e_calls()
            want = [a.copy() for a in (hy_g, hy_u, hy_d)]
            for a in (hy_g, hy_u, hy_d):
                a.fill(np.nan)
            e2e_batched()
            if not all(np.array_equal(a.view(np.uint32), b.view(np.uint32))
                       for a, b in zip((hy_g, hy_u, hy_d), want)):
                raise RuntimeError("batched e2e step differs from the call-by-call step")
        h2d, d2h = 4 * (GATE[1] + DOWN[1]), 4 * (2 * GATE[0] + DOWN[0])
        api = ("gi_cuda_gemv_buf x3 inside gi_cuda_begin_batch/end_batch (host y/x, pinned)" if args.e2e_batch
               else "gi_cuda_gemv_buf (host y/x, pinned: x copied in, y stored by the kernel)")
    else:
        bufs = {k: G.CreateBuffer(v) for k, v in fw.items()}
        bufs["norm"] = G.CreateBuffer(np.ones(DOWN[0], np.float32))
        hx = torch.from_numpy(seeded(101, GATE[1], 1.0)).pin_memory().numpy()

        def e2e_step():
            G.FFNBuf(hx, bufs["norm"], bufs["gate"], bufs["up"], bufs["down"], DOWN[0], hn, 1e-5)

        h2d = d2h = 4 * DOWN[0]
        api = "gi_cuda_ffn_buf (host x, pinned: copied in and back; the down partials all-reduced on the GPUs)"

    for _ in range(max(3, args.warmup)):
        e2e_step()
    e2e_steps = max(10, min(args.steps, 2000))
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev)
    if pg:
        pg.all_reduce(te, op=pg.ReduceOp.MAX)
    e2e_gbs = STEP_BYTES * e2e_steps / float(te.item()) / 1e9
    for b in bufs.values():
        G.ReleaseBuffer(b)
    del fcopies
    if world > 1:
        pg.barrier()
        G.tp_close()

    decode = None if args.no_decode else decode_section(args, world, rank, local, pg)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, cores, sample = cpu_port_gemv_gbs(args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample,
               "nproc": os.cpu_count(), "cpu_model": cpu_model()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "fp32",
            "data": "synthetic (seeded N(0,0.02) weights -> Q4_K, N(0,1) activations)",
            "config": step_config(world),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": profiled_traffic() if world == 1 else None,
                         "peak_source": peak_kind, "kernel": "gemv_q4k_kernel",
                         "bytes_per_launch": int(launch_bytes)},
            "frac_of_8TBs": round(value / world / 8000.0, 4),
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": api, "steps": e2e_steps},
            "gpu_launches": 2 * args.steps,
            "step_distribution": dist,
            "ffn_block": ffn_block,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "decode": decode,
        }
        if world > 1:
            line["tp_shard"] = {"hidden_rows_per_rank": [ffn_shard(world, r)[1] for r in range(world)],
                                "weight_bytes_per_rank": int(rank_bytes), "rotating_copies": ncopy}
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode / prefill section")
    ap.add_argument("--e2e-batch", action="store_true",
                    help="e2e step inside BeginBatch/EndBatch (one wait per step), checked against call-by-call")
    ap.add_argument("--persistent", action="store_true",
                    help="also time configs 4 and 5 with the persistent layers kernel (Model.set_persistent)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
