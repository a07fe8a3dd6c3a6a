"""Benchmark of the Q8_0 linear hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the Q8_0 GEMM shape sweep): one step = one pass over the 18 GEMMs
M in {1, 16, 128, 1024, 4096, 16384} x (K, N) in {(1024, 3072), (1024, 4096), (4096, 1024)}: bf16 activations ~N(0,1),
weights ~N(0,0.02) quantized to Q8_0 on the device, fp32 accumulation, bf16 out, seeded synthetic data. Every GEMM of
a step has its own weights and activations; a step streams ~1.3 GB, so no operand is still in the 126 MB L2 when it
is used again one step later.

value      : whole-job TFLOP/s = sum over ranks of 2 M N K per step x K steps / max-over-ranks device time, with all
             operands resident in HBM (the K steps replay a CUDA graph of the 18 launches; timed by CUDA events).
e2e        : the same metric through the drop-in API (fused_linear over GGUF Q8_0 bytes) with each step's activations
             copied host->device from pinned memory and its outputs copied back inside the timed region; the copies of
             the independent GEMMs are pipelined with their compute over three streams.
roofline   : the GEMM kernel on the tensor-bound shapes (M >= 4096): 2 M N K per launch / CUDA-event duration, against
             the measured dense bf16 peak; roofline_small_m: the HBM-bound shapes (M <= 16), algorithmic bytes
             1.0625 N K + 2 M K + 2 M N + 4 N per launch against the measured HBM bandwidth.
gpu_baselines: on the same GPU, per shape, the reference's unfused PackedLinear path (torch dequantize + F.linear)
             and cuBLAS on dense bf16 weights, against the fused kernel's per-launch times (shapes[]).
cpu_baseline: the reference's own CPU kernel (src/kernels.cpp gemm_packed, float kernel, OpenMP, compiled into
             oracle/_ref) on a bounded sample (M capped at 256 rows per shape), rank 0 at N=1.
--impl reference: that CPU kernel alone, as the reference arm (rank 0 only under torchrun).
N > 1: one process per GPU (torchrun), each GPU runs the full sweep on its own data; the path shards by request with
no collective ("weak" scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MS = (1, 16, 128, 1024, 4096, 16384)
KNS = ((1024, 3072), (1024, 4096), (4096, 1024))
METRIC = "Q8_0 GEMM TFLOP/s (config 2 shape sweep)"
UNIT = "TFLOP/s"


def shapes():
    return [(m, k, n) for (k, n) in KNS for m in MS]


def flops(m, k, n):
    return 2.0 * m * n * k


def alg_bytes(m, k, n):
    return 1.0625 * n * k + 2.0 * m * k + 2.0 * m * n + 4.0 * n


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------------------------------ CPU (reference)
def cpu_reference_runner(m_cap=256):
    """Builds the reference's gemm_packed float kernel over the sweep with M capped at m_cap rows (operands made
    once) and returns sample(seconds) -> (TFLOP/s, cores, kind, sample description), each sample at least one pass."""
    from oracle import oracle as O
    kind = "reference" if O.have_ref() else "port"
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    cases = []
    for (m, k, n) in shapes():
        mm = min(m, m_cap)
        q8 = O.q8_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32))
        x = O.f32_to_bf16_round(rng.normal(0, 1, (mm, k)).astype(np.float32))
        b = np.zeros(n, np.float32)
        cases.append((mm, k, n, q8, x, b))
    if kind == "reference":
        O.ref_threads(cores)
        lins = [O.RefLinear(q8, b, n, k) for (mm, k, n, q8, x, b) in cases]
        run = lambda i: lins[i].gemm(cases[i][4], mode=0)  # noqa: E731
    else:
        cores = 1
        run = lambda i: O.gemm_q8(cases[i][4], cases[i][3], cases[i][5], cases[i][2], cases[i][1])  # noqa: E731
    for i in range(len(cases)):  # warm-up pass
        run(i)

    def sample(seconds):
        total_flops, passes, t0 = 0.0, 0, time.perf_counter()
        while True:
            for i, (mm, k, n, *_) in enumerate(cases):
                run(i)
                total_flops += flops(mm, k, n)
            passes += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        text = (f"{passes} passes of the 18-shape sweep with M capped at {m_cap} rows "
                f"({total_flops / passes / 1e9:.1f} GFLOP per pass), {'OpenMP' if kind == 'reference' else 'scalar'}")
        return total_flops / dt / 1e12, cores, kind, text

    return sample


def cpu_reference_sample(seconds=12.0, m_cap=256):
    """One bounded sample of the reference's CPU kernel over the sweep: (TFLOP/s, cores, kind, description)."""
    return cpu_reference_runner(m_cap)(seconds)


# ------------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    def __init__(self, gpus):
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])
        self.gpus = gpus
        self.proc = None

    def start(self):
        q = ("index,timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        self.t_start = time.time()

    def mark(self):
        return time.time()

    def stop(self, t0, t1):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
                ts = time.mktime(time.strptime(parts[1].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                rows.append((idx, ts, float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        rows = [r for r in rows if r[0] in self.gpus]
        inside = [r for r in rows if t0 - 1.0 <= r[1] <= t1 + 1.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v.lower() == "active"})
        self.path.unlink(missing_ok=True)
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(r[2] for r in inside), "sm_max_mhz": max(r[3] for r in inside),
                "reasons": reasons, "samples": len(inside)}


# ------------------------------------------------------------------------------------------------ GPU baselines
def dequantize_q8_torch(packed, n, k, dtype):
    """The reference's unfused GPU path for a Q8_0 matrix (tools/idol_packed.py:25-31,71-79 PackedLinear.dequantize):
    fp16 scale times int8 code in fp32 over the 34-byte blocks, then the activation dtype, in plain torch ops."""
    import torch
    blocks = packed.reshape(-1, 34)
    scale = blocks[:, :2].contiguous().view(torch.float16).float()
    codes = blocks[:, 2:].contiguous().view(torch.int8).float()
    return (codes * scale).reshape(n, k).to(dtype)


def measure_gpu_baselines(ops, stream, dev):
    """Per sweep shape, CUDA-event time of (a) the reference's unfused PackedLinear.forward on the GPU (dequantize the
    GGUF bytes to bf16, then F.linear = cuBLAS) and (b) cuBLAS alone on weights dequantized beforehand, each over R
    operand copies in one CUDA graph (as the per-launch timing of the fused kernel). Returns per-shape microseconds."""
    import torch
    import torch.nn.functional as F
    rows = []
    for o in ops:
        m, k, n = o["m"], o["k"], o["n"]
        per_copy = n * k * 2 + m * k * 2
        R = int(min(16, max(2, -(-256e6 // per_copy))))
        xs = [o["x"].clone() for _ in range(R)]
        packs = [o["packed"].clone() for _ in range(R)]
        dense = [dequantize_q8_torch(pk, n, k, torch.bfloat16) for pk in packs]
        res = {}
        for name in ("unfused", "cublas"):
            def run():
                for r in range(R):
                    w = dense[r] if name == "cublas" else dequantize_q8_torch(packs[r], n, k, torch.bfloat16)
                    F.linear(xs[r], w, o["bias_bf16"])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                run()
                with torch.cuda.graph(g, stream=stream):
                    run()
                g.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(3):
                    g.replay()
                e1.record(stream)
            stream.synchronize()
            res[name] = e0.elapsed_time(e1) * 1e3 / (3 * R)
            del g
        rows.append(res)
        del xs, packs, dense
        torch.cuda.empty_cache()
    return rows


# ------------------------------------------------------------------------------------------------------ ours
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, tc_peak, peak_kind = peaks()

    # Operands: one weight matrix and one activation batch per GEMM, resident in HBM.
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    ops = []
    for (m, k, n) in shapes():
        w = torch.randn((n, k), device=dev, generator=g) * 0.02
        packed = pkg.quantize(w)
        tiles = pkg.repack(packed, n, k)
        del w
        x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
        bias = (torch.randn(n, device=dev, generator=g) * 0.01)
        y = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
        ops.append(dict(m=m, k=k, n=n, packed=packed, tiles=tiles, x=x, bias=bias, y=y,
                        bias_bf16=bias.to(torch.bfloat16)))
    step_flops = sum(flops(o["m"], o["k"], o["n"]) for o in ops)
    stream = torch.cuda.Stream(device=dev)

    def launch_step():
        for o in ops:
            pkg.gemm_into(o["y"], o["x"], o["tiles"], o["bias"], o["n"], o["k"])

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 1)):
            launch_step()
    stream.synchronize()
    assert pkg._capi.device_status(local_rank) == 0

    # Region A (value): a CUDA graph of G whole steps, replayed; timed by events outside the graph.
    G = min(10, args.steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(G):
                launch_step()
    rest = args.steps % G
    graph_rest = None
    if rest:
        graph_rest = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph_rest, stream=stream):
                for _ in range(rest):
                    launch_step()
    with torch.cuda.stream(stream):
        graph.replay()  # warm the graph itself (not timed)
    stream.synchronize()
    assert pkg._capi.device_status(local_rank) == 0

    clocks = ClockSampler([local_rank] if world == 1 else list(range(world)))
    if rank == 0:
        clocks.start()
        time.sleep(0.5)
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.time()
    with torch.cuda.stream(stream):
        t_begin.record(stream)
        for _ in range(args.steps // G):
            graph.replay()
        if graph_rest is not None:
            graph_rest.replay()
        t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall1 = time.time()
    ms = t_begin.elapsed_time(t_end)
    status = pkg._capi.device_status(local_rank)

    # Region B (per-launch durations for the roofline): per shape, a graph of R back-to-back launches over R distinct
    # copies of its operands (R copies total > 256 MB, so each launch reads its operands from HBM), timed by events.
    mean_ms = []
    reps = []
    for o in ops:
        per_copy = o["tiles"].numel() + o["x"].numel() * 2
        R = int(min(32, max(2, -(-256e6 // per_copy))))
        copies = []
        for _ in range(R):
            copies.append((o["tiles"].clone(), o["x"].clone(), torch.empty_like(o["y"])))
        gs = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for (t_, x_, y_) in copies[:1]:
                pkg.gemm_into(y_, x_, t_, o["bias"], o["n"], o["k"])
            with torch.cuda.graph(gs, stream=stream):
                for (t_, x_, y_) in copies:
                    pkg.gemm_into(y_, x_, t_, o["bias"], o["n"], o["k"])
            gs.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(3):
                gs.replay()
            e1.record(stream)
        stream.synchronize()
        mean_ms.append(e0.elapsed_time(e1) / (3 * R))
        reps.append(R)
        del copies, gs
    torch.cuda.empty_cache()

    # GPU baselines on the same device (not part of the timed step): the reference's unfused PackedLinear path and
    # cuBLAS on dense bf16 weights, per shape.
    base_us = measure_gpu_baselines(ops, stream, dev) if not args.no_gpu_baselines else None

    # e2e through the drop-in API with host buffers
    host_x = [o["x"].cpu().pin_memory() for o in ops]
    host_y = [torch.empty(o["y"].shape, dtype=o["y"].dtype).pin_memory() for o in ops]
    dev_x = [torch.empty_like(o["x"]) for o in ops]
    e2e_steps = max(1, min(args.steps, 10))
    fused = pkg.fused_linear
    with torch.cuda.stream(stream):
        for i, o in enumerate(ops):  # warm: builds the tiled copies fused_linear caches
            fused(o["x"], o["packed"], (o["n"], o["k"]), 8, o["bias_bf16"])
    stream.synchronize()
    # The ops are independent, so the copies are pipelined as a user streaming them would: the host->device copy of
    # op i+1 runs on one stream and the device->host copy of op i-1 on another while op i computes (PCIe is full
    # duplex). Events order each op's copy-in -> compute -> copy-out; an op's device input is rewritten only after its
    # previous compute finished. The timed region spans every copy of every step.
    copy_in, copy_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in ops]
    ev_comp = [torch.cuda.Event() for _ in ops]
    outs = [None] * len(ops)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    copy_in.wait_event(e0)
    copy_out.wait_event(e0)
    for step in range(e2e_steps):
        for i, o in enumerate(ops):
            with torch.cuda.stream(copy_in):
                if step > 0:
                    copy_in.wait_event(ev_comp[i])
                dev_x[i].copy_(host_x[i], non_blocking=True)
                ev_in[i].record(copy_in)
            with torch.cuda.stream(stream):
                stream.wait_event(ev_in[i])
                outs[i] = fused(dev_x[i], o["packed"], (o["n"], o["k"]), 8, o["bias_bf16"])
                ev_comp[i].record(stream)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_comp[i])
                outs[i].record_stream(copy_out)
                host_y[i].copy_(outs[i], non_blocking=True)
    stream.wait_stream(copy_out)
    stream.wait_stream(copy_in)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    h2d = sum(t.numel() * t.element_size() for t in host_x)
    d2h = sum(t.numel() * t.element_size() for t in host_y)

    # Config 3 (denoiser-block steps) and config 4 (Gaussian MLP) on this GPU's own data (shard by request).
    block_steps = max(3, min(args.steps, 30))
    block_ms = measure_block(pkg, dev, stream, block_steps, world)
    mlp_steps = max(3, min(args.steps, 30))
    mlp_ms = measure_mlp(pkg, dev, stream, mlp_steps, world)
    gs_steps = max(3, min(args.steps, 20))
    gs_ms = measure_gs_block(pkg, dev, stream, gs_steps, world)
    dec_steps = max(3, min(args.steps, 5))
    dec_ms = measure_gs_decoder(pkg, dev, stream, dec_steps, world)
    full_steps = 3
    full_ms = measure_decode(pkg, dev, stream, full_steps, world)
    status = max(status, pkg._capi.device_status(local_rank))

    if world > 1:
        t = torch.tensor([ms, e2e_ms, float(status), block_ms, mlp_ms, gs_ms, dec_ms, full_ms], device=dev,
                         dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, status, block_ms, mlp_ms = float(t[0]), float(t[1]), int(t[2]), float(t[3]), float(t[4])
        gs_ms, dec_ms, full_ms = float(t[5]), float(t[6]), float(t[7])
    clk = clocks.stop(wall0, wall1) if rank == 0 else None
    if rank != 0:
        return

    value = step_flops * args.steps * world / (ms / 1e3) / 1e12
    e2e_value = step_flops * e2e_steps * world / (e2e_ms / 1e3) / 1e12
    shape_rows = []
    for i, o in enumerate(ops):
        t = mean_ms[i] / 1e3
        tf = flops(o["m"], o["k"], o["n"]) / t / 1e12
        gb = alg_bytes(o["m"], o["k"], o["n"]) / t / 1e9
        row = {"M": o["m"], "K": o["k"], "N": o["n"], "copies": reps[i], "us": round(mean_ms[i] * 1e3, 2),
               "tflops": round(tf, 1), "gbs": round(gb, 1), "frac_tensor": round(tf / tc_peak, 3),
               "frac_hbm": round(gb / hbm_peak, 3)}
        if base_us is not None:
            row["us_unfused"] = round(base_us[i]["unfused"], 2)
            row["us_cublas_dense"] = round(base_us[i]["cublas"], 2)
        shape_rows.append(row)
    big = [i for i, o in enumerate(ops) if o["m"] >= 4096]
    small = [i for i, o in enumerate(ops) if o["m"] <= 16]
    ach_t = sum(flops(ops[i]["m"], ops[i]["k"], ops[i]["n"]) for i in big) / (sum(mean_ms[i] for i in big) / 1e3) / 1e12
    ach_b = sum(alg_bytes(ops[i]["m"], ops[i]["k"], ops[i]["n"]) for i in small) / (
        sum(mean_ms[i] for i in small) / 1e3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "q8_gemm_traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("bytes_per_launch_tensor_bound")

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded normal activations, Q8_0 of normal weights)",
        "config": {"workload": "config2_q8_0_gemm_sweep", "M": list(MS), "KN": [list(kn) for kn in KNS],
                   "operands": "resident in HBM", "l2": "each operand used once per step; a step streams "
                   f"{sum(o['x'].numel() * 2 + o['tiles'].numel() + o['y'].numel() * 2 for o in ops) / 1e9:.2f} GB "
                   "> 126 MB L2", "timing": f"CUDA graph of {G} steps replayed; CUDA events",
                   "per_launch_timing": "per shape, a CUDA graph of R launches over R operand copies (> 256 MB in "
                   "total) replayed 3 times between CUDA events; R per shape in shapes[].copies",
                   "parallelism": f"replicas x{world} (shard by request, no collective)"},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "fused_linear(value, packed, shape, 8, bias) on host-pinned inputs; per op H2D copy, compute and "
                       "D2H copy pipelined over three streams (the ops are independent)"},
        "roofline": {"bound": "tensor", "achieved": round(ach_t, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(ach_t / tc_peak, 3), "traffic": traffic,
                     "peak_source": f"{peak_kind} bf16 burst", "launches": "M in {4096, 16384}"},
        "roofline_small_m": {"bound": "hbm", "achieved": round(ach_b, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(ach_b / hbm_peak, 3), "peak_source": f"{peak_kind} copy",
                             "launches": "M in {1, 16}"},
        "shapes": shape_rows,
        "gpu_launches": len(ops) * args.steps,
        "device_status": status,
        "clocks": clk,
        "block": {"metric": "denoiser-block steps/s (config 3: 2 images x 4096 tokens, D 1024, 16 heads x 64, "
                            "Q8_0 QKV/out/MLP 1024->4096->1024, GELU tanh, fp32 residual)",
                  "value": round(block_steps * world / (block_ms / 1e3), 2), "unit": "block-steps/s",
                  "ms_per_step": round(block_ms / block_steps, 3), "steps": block_steps,
                  "tflops": round(BLOCK_FLOPS * block_steps * world / (block_ms / 1e3) / 1e12, 1),
                  "frac_tensor": round(BLOCK_FLOPS / (block_ms / block_steps / 1e3) / 1e12 / tc_peak, 3),
                  "scaling": "weak (each GPU runs its own images; no collective)",
                  "work": "343.6 GFLOP per step (206.2 linears + 137.4 attention)"},
        "gaussian_block": {"metric": "Gaussian-decoder block steps/s (src/decoders.cpp:296-313: 8192 anchors, "
                                     "self-attention, cross-attention to 8192 latent tokens x 16 conditions, MLP "
                                     "1024->4096->1024, D 1024, 16 heads, fp32 residual)",
                           "value": round(gs_steps * world / (gs_ms / 1e3), 2), "unit": "block-steps/s",
                           "ms_per_step": round(gs_ms / gs_steps, 3), "steps": gs_steps,
                           "tflops": round(GS_FLOPS * gs_steps * world / (gs_ms / 1e3) / 1e12, 1),
                           "work": f"{GS_FLOPS / 1e9:.1f} GFLOP per step"},
        "gaussian_decoder": {"metric": "Gaussian decodes/s (Decoders::gaussian_features + to_gaussians: 8192 "
                                       "anchors -> 262,144 Gaussians, 16 blocks, 8192 latent tokens x 16, D 1024)",
                             "value": round(dec_steps * world / (dec_ms / 1e3), 3), "unit": "decodes/s",
                             "ms_per_step": round(dec_ms / dec_steps, 3), "steps": dec_steps,
                             "gaussians_per_s": round(GS_ANCHORS * 32 * dec_steps * world / (dec_ms / 1e3), 0),
                             "tflops": round(GS_FLOPS * GS_BLOCKS * dec_steps * world / (dec_ms / 1e3) / 1e12, 1)},
        "decode": {"metric": "Decoders::decode calls/s (latent 8192 x 16 -> sample_anchors to level 7 through the "
                             "octree decoder, 4 blocks -> Gaussian decoder, 16 blocks -> 262,144 activated Gaussians; "
                             "D 1024)", "value": round(full_steps * world / (full_ms / 1e3), 3), "unit": "decodes/s",
                   "ms_per_step": round(full_ms / full_steps, 2), "steps": full_steps,
                   "reference_published": "36.99 s on 8 threads and 0.34 s with the upstream GPU modules on an RTX "
                                          "4090, both octree + Gaussian decoders at 262,144 Gaussians "
                                          "(docs/data/decoder-cpu-vs-gpu.json); context only, other hardware"},
        "gaussian_mlp": {"metric": "Gaussian MLP points/s (config 4: 262,144 points, Q8_0 128->512->512->14, SiLU, "
                                   "heads)", "value": round(MLP_POINTS * mlp_steps * world / (mlp_ms / 1e3), 0),
                         "unit": "points/s", "ms_per_step": round(mlp_ms / mlp_steps, 3), "steps": mlp_steps,
                         "tflops": round(MLP_FLOPS * mlp_steps * world / (mlp_ms / 1e3) / 1e12, 1)},
    }
    if base_us is not None:
        sweep_unfused = sum(r["unfused"] for r in base_us) / 1e6
        sweep_cublas = sum(r["cublas"] for r in base_us) / 1e6
        sweep_ours = sum(mean_ms) / 1e3
        line["gpu_baselines"] = {
            "unit": UNIT, "timing": "per shape, R operand copies in one CUDA graph, CUDA events (as shapes[].us)",
            "sweep_ours": round(step_flops / sweep_ours / 1e12, 1),
            "packedlinear_unfused": {
                "value": round(step_flops / sweep_unfused / 1e12, 1),
                "what": "the reference's GPU path without the fused kernel (tools/idol_packed.py:71-79): dequantize "
                        "the GGUF Q8_0 bytes to bf16 with torch ops every call, then F.linear (cuBLAS)"},
            "cublas_bf16_dense": {
                "value": round(step_flops / sweep_cublas / 1e12, 1),
                "what": "F.linear (cuBLAS) on bf16 weights dequantized beforehand: 2 bytes per weight instead of "
                        "1.0625, no dequantization in the call"}}
    if world == 1 and not args.no_cpu_baseline:
        v, cores, kind, sample = cpu_reference_sample()
        line["cpu_baseline"] = {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample}
    print(json.dumps(line), flush=True)


def run_profile_shape(args):
    """One GEMM shape (or the block / MLP composition), launched warmup + steps times back to back: the small case an
    ncu capture targets."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    if args.profile_shape in ("block", "mlp"):
        dev = torch.device("cuda", 0)
        stream = torch.cuda.Stream(device=dev)
        fn = measure_block if args.profile_shape == "block" else measure_mlp
        ms = fn(pkg, dev, stream, args.steps, 1)
        print(json.dumps({"profile": args.profile_shape, "ms_per_step": round(ms / args.steps, 3),
                          "device_status": pkg._capi.device_status(0)}))
        return
    m, k, n = (int(v) for v in args.profile_shape.split(","))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    packed = pkg.quantize(torch.randn((n, k), device=dev, generator=g) * 0.02)
    tiles = pkg.repack(packed, n, k)
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device=dev, generator=g) * 0.01
    y = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
    for _ in range(args.warmup):
        pkg.gemm_into(y, x, tiles, bias, n, k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        pkg.gemm_into(y, x, tiles, bias, n, k)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"profile_shape": [m, k, n], "us_per_launch": round(us, 2),
                      "tflops": round(flops(m, k, n) / us / 1e6, 1), "device_status": pkg._capi.device_status(0)}))


BLOCK_IMAGES, BLOCK_TOKENS, BLOCK_D, BLOCK_HEADS, BLOCK_H = 2, 4096, 1024, 16, 4096
BLOCK_FLOPS = (2.0 * BLOCK_IMAGES * BLOCK_TOKENS * (3 * BLOCK_D * BLOCK_D + BLOCK_D * BLOCK_D + 2 * BLOCK_H * BLOCK_D)
               + 4.0 * BLOCK_TOKENS ** 2 * BLOCK_D * BLOCK_IMAGES)
GS_ANCHORS, GS_LATENTS, GS_COND, GS_BLOCKS, OCT_BLOCKS, DECODE_LEVEL = 8192, 8192, 16, 16, 4, 7
GS_FLOPS = (2.0 * GS_ANCHORS * (3 + 1 + 1 + 1 + 2 * BLOCK_H // BLOCK_D) * BLOCK_D * BLOCK_D
            + 4.0 * GS_ANCHORS * GS_ANCHORS * BLOCK_D + 4.0 * GS_ANCHORS * GS_LATENTS * BLOCK_D
            + 2.0 * GS_LATENTS * GS_COND * 2 * BLOCK_D)
MLP_POINTS = 262144
MLP_FLOPS = 2.0 * MLP_POINTS * (128 * 512 + 512 * 512 + 512 * 14)


def _graph_ms(torch, stream, fn, steps, world):
    """Capture `fn` (one step) in a CUDA graph, warm it, then time `steps` replays with CUDA events."""
    import torch.distributed as dist
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            fn()
        g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def measure_block(pkg, dev, stream, steps, world):
    """Config 3: one denoiser block over 2 images x 4096 tokens (fp32 residual stream updated in place)."""
    import torch
    from idol_b200.block import DenoiserBlock, Q8Weight
    g = torch.Generator(device=dev).manual_seed(77)
    D, H = BLOCK_D, BLOCK_H
    w = {}
    for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "ff1": (H, D), "ff2": (D, H)}.items():
        w[name] = Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * 0.02,
                                      torch.randn(n, device=dev, generator=g) * 0.01)
    blk = DenoiserBlock(w["qkv"], w["out"], w["ff1"], w["ff2"], 1 + 0.1 * torch.randn(D, device=dev, generator=g),
                        1 + 0.1 * torch.randn(D, device=dev, generator=g), BLOCK_HEADS)
    x = torch.randn((BLOCK_IMAGES * BLOCK_TOKENS, D), device=dev, generator=g)
    blk.forward_(x, images=BLOCK_IMAGES)  # sizes the workspace outside the graph
    return _graph_ms(torch, stream, lambda: blk.forward_(x, images=BLOCK_IMAGES), steps, world)


def _random_gs_block(dev, g):
    """A Gaussian-decoder block of the real model's shape with seeded random weights (Q8_0 on the device)."""
    import torch
    from idol_b200.block import GaussianBlock, Q8Weight
    D, H = BLOCK_D, BLOCK_H
    w = {}
    for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "cq": (D, D), "co": (D, D), "ff1": (H, D),
                         "ff2": (D, H)}.items():
        w[name] = Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * 0.02,
                                      torch.randn(n, device=dev, generator=g) * 0.01)
    vec = [1 + 0.1 * torch.randn(D, device=dev, generator=g) for _ in range(5)] + [
        0.1 * torch.randn(D, device=dev, generator=g)]
    return GaussianBlock(w["qkv"], w["out"], w["cq"], w["co"], w["ff1"], w["ff2"], *vec,
                         torch.randn((2 * D, GS_COND), device=dev, generator=g) * 0.25,
                         torch.randn(2 * D, device=dev, generator=g) * 0.01, BLOCK_HEADS)


def measure_gs_block(pkg, dev, stream, steps, world):
    """The real Gaussian decoder's block (src/decoders.cpp:296-313) at its model size: 8192 anchors attending to
    themselves and to 8192 latent tokens of 16 conditions, D 1024, 16 heads, fp32 residual stream in place."""
    import torch
    g = torch.Generator(device=dev).manual_seed(78)
    blk = _random_gs_block(dev, g)
    D = BLOCK_D
    x = torch.randn((GS_ANCHORS, D), device=dev, generator=g)
    cond = torch.randn((GS_LATENTS, GS_COND), device=dev, generator=g)
    blk.forward_(x, cond)  # sizes the workspace outside the graph
    return _graph_ms(torch, stream, lambda: blk.forward_(x, cond), steps, world)


def _random_gaussian_decoder(dev, g):
    import torch
    from idol_b200.block import Q8Weight
    from idol_b200.native import GaussianDecoder
    D, G = BLOCK_D, 32
    blocks = [_random_gs_block(dev, g) for _ in range(GS_BLOCKS)]
    return GaussianDecoder(blocks, torch.randn((D, 3), device=dev, generator=g) * 0.5,
                           torch.randn(D, device=dev, generator=g) * 0.01,
                           Q8Weight.from_float(torch.randn((D, D), device=dev, generator=g) * 0.03),
                           Q8Weight.from_float(torch.randn((15 * G, D), device=dev, generator=g) * 0.03),
                           2.0 ** torch.linspace(0, 10, D // 6), G, torch.randn(3 * G, device=dev, generator=g) * 0.1,
                           -1.0)


def _random_octree_decoder(dev, g):
    """The octree decoder of the real model's shape (4 blocks, D 1024) with seeded random weights."""
    import torch
    from idol_b200.block import Q8Weight
    from idol_b200.native import OctreeDecoder
    D, H = BLOCK_D, BLOCK_H

    def q8(n, k, sd=0.02):
        return Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * sd,
                                   torch.randn(n, device=dev, generator=g) * 0.01)

    blocks = [{"cq": q8(D, D), "co": q8(D, D), "ff1": q8(H, D), "ff2": q8(D, H),
               "kv_w": torch.randn((2 * D, GS_COND), device=dev, generator=g) * 0.25,
               "kv_b": torch.randn(2 * D, device=dev, generator=g) * 0.01,
               "cq_gamma": 1 + 0.1 * torch.randn(D, device=dev, generator=g),
               "ck_gamma": 1 + 0.1 * torch.randn(D, device=dev, generator=g)} for _ in range(OCT_BLOCKS)]
    return OctreeDecoder(blocks, torch.randn((D, 3), device=dev, generator=g) * 0.5,
                         torch.randn(D, device=dev, generator=g) * 0.01, q8(D, D, 0.03), q8(D, 256, 0.1),
                         q8(D, D, 0.03), q8(6 * D, D, 0.03), q8(8, D, 0.1), 2.0 ** torch.linspace(0, 10, D // 6),
                         torch.exp(-torch.log(torch.tensor(1024.0)) * torch.arange(128) / 128), BLOCK_HEADS)


def measure_decode(pkg, dev, stream, steps, world):
    """Decoders::decode at the real model's size: sample_anchors through the octree decoder (4 blocks) down to level
    DECODE_LEVEL for 8192 anchors, the Gaussian decoder (16 blocks) and to_gaussians: 262,144 Gaussians from 8192
    latent tokens x 16. The octree levels synchronise the stream (the host resamples between them), so the decode is
    timed by CUDA events around whole calls rather than replayed from a graph."""
    import torch
    import torch.distributed as dist
    from idol_b200.native import decode
    g = torch.Generator(device=dev).manual_seed(80)
    octree, gaussian = _random_octree_decoder(dev, g), _random_gaussian_decoder(dev, g)
    cond = torch.randn((GS_LATENTS, GS_COND), device=dev, generator=g)
    with torch.cuda.stream(stream):
        for _ in range(2):
            decode(octree, gaussian, cond, GS_ANCHORS * 32, DECODE_LEVEL, 7)
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(steps):
            decode(octree, gaussian, cond, GS_ANCHORS * 32, DECODE_LEVEL, 7 + i)
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def measure_gs_decoder(pkg, dev, stream, steps, world):
    """The whole Gaussian decoder (Decoders::gaussian_features + to_gaussians, src/decoders.cpp:284-316, 393-433) at
    the real model's size: 8192 anchors (262,144 Gaussians), 16 blocks, 8192 latent tokens x 16, D 1024, 480 raw
    features per anchor."""
    import torch
    g = torch.Generator(device=dev).manual_seed(79)
    dec = _random_gaussian_decoder(dev, g)
    pts = torch.rand((GS_ANCHORS, 3), device=dev, generator=g)
    cond = torch.randn((GS_LATENTS, GS_COND), device=dev, generator=g)

    def step():
        dec.to_gaussians(pts, dec.features(pts, cond))

    step()  # sizes the workspace outside the graph
    return _graph_ms(torch, stream, step, steps, world)


def measure_mlp(pkg, dev, stream, steps, world):
    """Config 4: the Gaussian MLP over 262,144 points."""
    import torch
    from idol_b200.block import GaussianMLP, Q8Weight
    g = torch.Generator(device=dev).manual_seed(78)
    layers = [Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * 0.02,
                                  torch.randn(n, device=dev, generator=g) * 0.01)
              for n, k in [(512, 128), (512, 512), (14, 512)]]
    mlp = GaussianMLP(layers)
    x = torch.randn((MLP_POINTS, 128), device=dev, generator=g).to(torch.bfloat16)
    mlp(x)
    return _graph_ms(torch, stream, lambda: mlp(x), steps, world)


def run_reference(args, rank):
    if rank != 0:
        return
    # Each step is a bounded sample (at least one pass of the capped sweep); the whole run stays within a few minutes
    # however many steps are asked for.
    seconds_per_step = min(2.0, 150.0 / max(1, args.steps))
    sample = cpu_reference_runner()
    vals = []
    for _ in range(args.warmup):
        sample(0.0)
    for _ in range(args.steps):
        v, cores, kind, text = sample(seconds_per_step)
        vals.append(v)
    v = statistics.median(vals)
    print(json.dumps({
        "metric": METRIC, "value": round(v, 4), "unit": UNIT, "impl": "reference", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded normal activations, Q8_0 of normal weights)",
        "config": {"workload": "config2_q8_0_gemm_sweep", "M": list(MS), "KN": [list(kn) for kn in KNS],
                   "sample": f"M capped at 256 rows per shape, {seconds_per_step:.2f} s (at least one pass) of CPU "
                             "work per step"},
        "cpu_baseline": {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": kind, "sample": text},
        "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-baselines", action="store_true")
    ap.add_argument("--profile-shape", default=None,
                    help="M,K,N: run only this GEMM (warmup + steps launches) for an ncu capture; 'block' or 'mlp' "
                         "runs the config-3 block or the config-4 MLP instead")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.profile_shape:
        run_profile_shape(args)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
