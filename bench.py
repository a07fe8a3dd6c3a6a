"""Benchmark of the Q8_0 linear hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (config 5): the denoiser's stack of 24 transformer blocks over a batch of 64 independent images, each
image two CFG branches of 4096 tokens (D 1024, 16 heads x 64, Q8_0 QKV/out/MLP 1024->4096->1024 with GELU tanh, fp32
residual stream, bf16 activations), seeded random weights and inputs. The 64 images are split contiguously across
the N ranks (one process per GPU, each a full replica of the Q8_0 weights, no collective on the data path), so the
total work is fixed and the scaling is strong. One step = one pass of the stack over this rank's images.

value      : block-steps/s = 24 blocks x 64 images x K steps / max-over-ranks device time of the K steps (inputs
             resident in HBM; CUDA events on the launching stream). A block-step is one image (its two CFG branches)
             through one block: 343.6 GFLOP (206.2 in the Q8_0 linears, 137.4 in attention).
e2e        : the same metric through DenoiserStack.forward_ with the images' residual streams in pinned host memory:
             each chunk of images is copied host->device, run through the 24 blocks and copied back, the copies of one
             chunk overlapping the compute of its neighbours; every copy is inside the timed region.
roofline   : the kernel with the largest share of a block's device time, timed alone on the block's own shapes
             (algorithmic FLOPs per launch / CUDA-event duration) against the measured dense bf16 peak; `kernels`
             lists every kernel of the block the same way.
gemm_sweep : (N = 1) the Q8_0 GEMM shape sweep M in {1, 16, 128, 1024, 4096, 16384} x (K, N) in {(1024, 3072),
             (1024, 4096), (4096, 1024)}: its own rooflines (tensor-bound M >= 4096, HBM-bound M <= 16), per-shape
             times and GPU baselines on the same device (the reference's unfused PackedLinear path, dense cuBLAS).
cpu_baseline, --impl reference: the reference's own CPU functions (src/kernels.cpp gemm_packed float kernel and
             attention, src/decoders.cpp norm_rows / rms_heads / gelu_tanh; OpenMP over every host thread; compiled into
             oracle/_ref) composing the same block on the same shapes. One step is one block-step, the bounded sample of
             the workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
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
SWEEP_METRIC = "Q8_0 GEMM TFLOP/s (config 2 shape sweep)"

BLOCK_IMAGES, BLOCK_TOKENS, BLOCK_D, BLOCK_HEADS, BLOCK_H = 2, 4096, 1024, 16, 4096
BLOCK_FLOPS = (2.0 * BLOCK_IMAGES * BLOCK_TOKENS * (3 * BLOCK_D * BLOCK_D + BLOCK_D * BLOCK_D + 2 * BLOCK_H * BLOCK_D)
               + 4.0 * BLOCK_TOKENS ** 2 * BLOCK_D * BLOCK_IMAGES)
STACK_BLOCKS, STACK_IMAGES, CFG = 24, 64, 2
CHUNK_IMAGES = 4  # images per pass through the blocks (8 sequences, 32768 rows)
# norm, qkv with the q/k norm fused, attention, out + residual, norm, ff1, ff2 + residual, and before each of the four
# GEMMs the launch that dequantises its weights into the dense layout (the large-M GEMM path)
LAUNCHES_PER_BLOCK = 11
METRIC = "denoiser-block steps/s (config 5: 24-block stack over 64 images x 2 CFG branches, sharded by image)"
UNIT = "block-steps/s"


def config5(world):
    """The workload description both arms print (identical for the same N)."""
    return {"workload": "config5_denoiser_stack", "blocks": STACK_BLOCKS, "images": STACK_IMAGES,
            "cfg_branches": CFG, "tokens": BLOCK_TOKENS, "dim": BLOCK_D, "heads": BLOCK_HEADS, "hidden": BLOCK_H,
            "weights": "Q8_0", "residual": "fp32", "activations": "bf16", "gelu": "tanh",
            "work": "343.6 GFLOP per block-step (206.2 linears + 137.4 attention)",
            "parallelism": f"dp{world}: images split contiguously over ranks, weights replicated, no collective",
            "l2": "inputs larger than L2: a rank's residual streams are >= 268 MB and each step rereads them all"}


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
def cpu_info():
    """Host facts for the CPU baseline: model, usable logical CPUs, physical cores, nominal clock, and the fp32 FMA
    peak of the AVX2 units (physical cores x GHz x 32 FLOP per cycle: two 8-wide FMA pipes)."""
    model, phys, cur, flags = "unknown", set(), {}, set()
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines() + [""]:
            if not line.strip():
                if cur:
                    phys.add((cur.get("physical id"), cur.get("core id", cur.get("processor"))))
                cur = {}
                continue
            key, _, val = line.partition(":")
            cur[key.strip()] = val.strip()
            if key.strip() == "model name":
                model = val.strip()
            if key.strip() == "flags":
                flags = set(val.split())
    except OSError:
        pass
    logical = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    physical = min(len(phys), logical) if phys else logical
    m = re.search(r"@\s*([\d.]+)\s*GHz", model)
    ghz, source = (float(m.group(1)), "model name") if m else (None, None)
    if ghz is None:
        try:  # the highest clock the kernel reports for a CPU
            khz = int(Path("/sys/devices/system/cpu/cpu0/cpufreq/cpuinfo_max_freq").read_text())
            ghz, source = khz / 1e6, "cpuinfo_max_freq"
        except (OSError, ValueError):
            mhz = [float(l.split(":")[1]) for l in Path("/proc/cpuinfo").read_text().splitlines()
                   if l.startswith("cpu MHz")] if Path("/proc/cpuinfo").exists() else []
            if mhz:
                ghz, source = max(mhz) / 1e3, "cpu MHz"
    return {"model": model, "logical_cpus": logical, "physical_cores": physical, "ghz": ghz, "ghz_source": source,
            "avx2_fma_peak_gflops": round(physical * ghz * 32, 1) if ghz else None, "flags": flags}


def cpu_reference_runner():
    """One block-step of the config-5 block (one image: 2 CFG branches x 4096 tokens, D 1024) on the reference's own
    CPU functions (oracle.RefBlock over oracle/_ref, every usable host thread); without oracle/_ref, the C
    restatement on 2 x 512 tokens, converted to block-steps by its FLOPs. Returns (step() -> block-steps/s, facts)."""
    from oracle import oracle as O
    info = cpu_info()
    rng = np.random.default_rng(0)
    D, H = BLOCK_D, BLOCK_H
    layers = {}
    for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "ff1": (H, D), "ff2": (D, H)}.items():
        layers[name] = (O.q8_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32)),
                        rng.normal(0, 0.01, n).astype(np.float32), n, k)
    layers["q_gamma"] = rng.normal(1, 0.1, D).astype(np.float32)
    layers["k_gamma"] = rng.normal(1, 0.1, D).astype(np.float32)
    if O.have_ref():
        kind, threads, tokens = "reference", O.ref_threads(info["logical_cpus"]), BLOCK_TOKENS
        blk = O.RefBlock(layers, BLOCK_HEADS)
        run = lambda x: blk.forward_(x, images=CFG)  # noqa: E731
    else:
        kind, threads, tokens = "port", 1, 512
        run = lambda x: O.block_forward(x, layers, BLOCK_HEADS, images=CFG)  # noqa: E731
    x0 = O.f32_to_bf16_round(rng.normal(0, 1, (CFG * tokens, D)).astype(np.float32))
    sample_flops = (2.0 * CFG * tokens * (3 * D * D + D * D + 2 * H * D) + 4.0 * tokens ** 2 * D * CFG)
    unit_flops = BLOCK_FLOPS / BLOCK_IMAGES * CFG

    def step():
        x = x0.copy()
        t0 = time.perf_counter()
        run(x)
        dt = time.perf_counter() - t0
        return sample_flops / unit_flops / dt, dt

    def vnni_step():
        """The same block with the reference's integer-activation kernel (set_quant_kernel(1), its default on CPUs
        with AVX-VNNI); None where the host lacks AVX-VNNI or the reference library is absent."""
        if kind != "reference" or "avx_vnni" not in info.get("flags", ()):
            return None
        x = x0.copy()
        t0 = time.perf_counter()
        blk.forward_(x, images=CFG, mode=1)
        return sample_flops / unit_flops / (time.perf_counter() - t0)

    step.vnni = vnni_step

    facts = dict(info, kind=kind, threads=threads,
                 sample=(f"one block-step: one image (2 CFG branches x {tokens} tokens, D 1024) through one block on "
                         + ("the reference's compiled CPU functions, OpenMP" if kind == "reference" else
                            "the C restatement (no oracle/_ref), scaled by FLOPs to a 4096-token block-step")))
    return step, facts


def cpu_baseline_entry(rates, times, facts):
    v = statistics.median(rates)
    gflops = v * BLOCK_FLOPS / BLOCK_IMAGES * CFG / 1e9
    peak = facts.get("avx2_fma_peak_gflops")
    return {"value": round(v, 4), "unit": UNIT, "cores": facts["threads"], "kind": facts["kind"],
            "sample": f"{facts['sample']}; median of {len(rates)} timed steps ({statistics.median(times):.2f} s each)",
            "cpu_model": facts["model"], "physical_cores": facts["physical_cores"],
            "omp_threads": facts["threads"], "ghz": facts["ghz"], "ghz_source": facts["ghz_source"],
            "gflops": round(gflops, 1),
            "avx2_fma_peak_gflops": peak, "frac_of_avx2_peak": round(gflops / peak, 3) if peak else None,
            "vnni_kernel_value": facts.get("vnni"),
            "vnni_kernel": "the same block with the reference's integer-activation GEMMs (set_quant_kernel(1), its "
                           "default where AVX-VNNI exists; null when the host lacks it)"}


def cpu_reference_measure(warmup, steps, budget_s=150.0):
    """Warm-up steps (at most 2), then up to `steps` timed steps within about budget_s seconds (at least 3)."""
    step, facts = cpu_reference_runner()
    t_warm = None
    for _ in range(max(1, min(warmup, 2))):
        _, t_warm = step()
    timed = max(3, min(steps, int(budget_s / max(t_warm, 1e-3))))
    rates, times = [], []
    for _ in range(timed):
        r, t = step()
        rates.append(r)
        times.append(t)
    vnni = [v for v in (step.vnni() for _ in range(min(3, timed))) if v is not None]
    facts["vnni"] = round(statistics.median(vnni), 4) if vnni else None
    return rates, times, facts


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


def reference_triton():
    """The reference's own fused GPU linear (tools/idol_triton.py fused_linear, Triton), staged into baseline/_ref/ by
    __graft_entry__.build(); None when it is not there or Triton cannot load it."""
    path = ROOT / "baseline" / "_ref" / "idol_triton.py"
    if not path.exists():
        return None
    try:
        import importlib.util
        spec = importlib.util.spec_from_file_location("reference_idol_triton", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod.fused_linear
    except Exception:
        return None


def measure_gpu_baselines(ops, stream, dev):
    """Per sweep shape, CUDA-event time of (a) the reference's unfused PackedLinear.forward on the GPU (dequantize the
    GGUF bytes to bf16, then F.linear = cuBLAS), (b) cuBLAS alone on weights dequantized beforehand, (c) the
    reference's fused Triton linear (tools/idol_triton.py:94-126) in bf16 and, where its dense branch applies
    (fp16, M >= 4096), in fp16; each over R operand copies in one CUDA graph, as the fused kernel's per-launch
    timing. Returns per-shape microseconds (None where a path does not apply or did not run)."""
    import torch
    import torch.nn.functional as F
    triton_linear = reference_triton()
    rows = []
    for o in ops:
        m, k, n = o["m"], o["k"], o["n"]
        per_copy = n * k * 2 + m * k * 2
        R = int(min(16, max(2, -(-256e6 // per_copy))))
        xs = [o["x"].clone() for _ in range(R)]
        packs = [o["packed"].clone() for _ in range(R)]
        dense = [dequantize_q8_torch(pk, n, k, torch.bfloat16) for pk in packs]
        xs16 = [x.to(torch.float16) for x in xs] if m >= 4096 else None
        b16 = o["bias"].to(torch.float16)
        variants = {"unfused": lambda r: F.linear(xs[r], dequantize_q8_torch(packs[r], n, k, torch.bfloat16),
                                                  o["bias_bf16"]),
                    "cublas": lambda r: F.linear(xs[r], dense[r], o["bias_bf16"])}
        if triton_linear is not None:
            variants["triton"] = lambda r: triton_linear(xs[r], packs[r], (n, k), 8, o["bias_bf16"])
            if xs16 is not None:
                variants["triton_fp16"] = lambda r: triton_linear(xs16[r], packs[r], (n, k), 8, b16)
        res = {"triton": None, "triton_fp16": None}
        for name, fn in variants.items():
            try:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(stream):
                    for r in range(R):
                        fn(r)
                    with torch.cuda.graph(g, stream=stream):
                        for r in range(R):
                            fn(r)
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
            except Exception as exc:  # a baseline that cannot run is reported as absent, not as a failure
                if name in ("unfused", "cublas"):
                    raise
                res[name] = None
                res.setdefault("error", f"{type(exc).__name__}: {str(exc)[:120]}")
        rows.append(res)
        del xs, packs, dense, xs16
        torch.cuda.empty_cache()
    return rows


# -------------------------------------------------------------------------------------------- the Q8_0 GEMM sweep
def measure_gemm_sweep(pkg, dev, stream, steps, no_gpu_baselines=False):
    """Config 2 on this GPU: value (whole sweep from a CUDA graph), per-launch times and rooflines, GPU baselines and
    an end-to-end pass through fused_linear with host buffers. Returns the sweep's entry of the JSON line."""
    import torch
    hbm_peak, tc_peak, peak_kind = peaks()
    g = torch.Generator(device=dev).manual_seed(1000)
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

    def launch_step():
        for o in ops:
            pkg.gemm_into(o["y"], o["x"], o["tiles"], o["bias"], o["n"], o["k"])

    with torch.cuda.stream(stream):
        for _ in range(3):
            launch_step()
    stream.synchronize()
    # The whole sweep: a CUDA graph of G steps replayed steps // G times between CUDA events.
    G = 10
    steps = max(G, steps - steps % G)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(G):
                launch_step()
        graph.replay()
    stream.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(steps // G):
            graph.replay()
        t1.record(stream)
    stream.synchronize()
    ms = t0.elapsed_time(t1)
    del graph

    # Per-launch durations: per shape, a graph of R back-to-back launches over R distinct copies of its operands
    # (R copies total > 256 MB, so each launch reads its operands from HBM), timed by events.
    mean_ms, reps = [], []
    for o in ops:
        per_copy = o["tiles"].numel() + o["x"].numel() * 2
        R = int(min(32, max(2, -(-256e6 // per_copy))))
        copies = [(o["tiles"].clone(), o["x"].clone(), torch.empty_like(o["y"])) for _ in range(R)]
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
    base_us = None if no_gpu_baselines else measure_gpu_baselines(ops, stream, dev)

    # End to end through the drop-in API with host buffers; the independent ops' copies are pipelined with their
    # compute over three streams (PCIe is full duplex).
    host_x = [o["x"].cpu().pin_memory() for o in ops]
    host_y = [torch.empty(o["y"].shape, dtype=o["y"].dtype).pin_memory() for o in ops]
    dev_x = [torch.empty_like(o["x"]) for o in ops]
    e2e_steps = 10
    fused = pkg.fused_linear
    with torch.cuda.stream(stream):
        for o in ops:  # builds the tiled copies fused_linear caches
            fused(o["x"], o["packed"], (o["n"], o["k"]), 8, o["bias_bf16"])
    stream.synchronize()
    copy_in, copy_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in ops]
    ev_comp = [torch.cuda.Event() for _ in ops]
    outs = [None] * len(ops)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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

    rows = []
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
            for key in ("triton", "triton_fp16"):
                if base_us[i].get(key) is not None:
                    row[f"us_reference_{key}"] = round(base_us[i][key], 2)
        rows.append(row)
    big = [i for i, o in enumerate(ops) if o["m"] >= 4096]
    small = [i for i, o in enumerate(ops) if o["m"] <= 16]
    ach_t = sum(flops(ops[i]["m"], ops[i]["k"], ops[i]["n"]) for i in big) / (sum(mean_ms[i] for i in big) / 1e3)
    ach_b = sum(alg_bytes(ops[i]["m"], ops[i]["k"], ops[i]["n"]) for i in small) / (
        sum(mean_ms[i] for i in small) / 1e3)
    out = {
        "metric": SWEEP_METRIC, "value": round(step_flops * steps / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
        "steps": steps, "ms_per_step": round(ms / steps, 4),
        "timing": f"CUDA graph of {G} sweeps replayed {steps // G} times between CUDA events; operands resident, each "
                  f"used once per sweep (a sweep streams "
                  f"{sum(o['x'].numel() * 2 + o['tiles'].numel() + o['y'].numel() * 2 for o in ops) / 1e9:.2f} GB "
                  "> 126 MB L2)",
        "e2e": {"value": round(step_flops * e2e_steps / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "fused_linear(value, packed, shape, 8, bias) on host-pinned inputs; per op H2D copy, compute "
                       "and D2H copy pipelined over three streams"},
        "roofline": {"bound": "tensor", "achieved": round(ach_t / 1e12, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(ach_t / 1e12 / tc_peak, 3), "peak_source": f"{peak_kind} bf16 burst",
                     "launches": "M in {4096, 16384}"},
        "roofline_small_m": {"bound": "hbm", "achieved": round(ach_b / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(ach_b / 1e9 / hbm_peak, 3), "peak_source": f"{peak_kind} copy",
                             "launches": "M in {1, 16}"},
        "shapes": rows,
        "per_launch_timing": "per shape, a CUDA graph of R launches over R operand copies (> 256 MB in total) "
                             "replayed 3 times between CUDA events",
    }
    tfile = ROOT / "profiles" / "q8_gemm_traffic.json"
    if tfile.exists():
        out["roofline"]["traffic"] = json.loads(tfile.read_text()).get("bytes_per_launch_tensor_bound")
    if base_us is not None:
        sweep_unfused = sum(r["unfused"] for r in base_us) / 1e6
        sweep_cublas = sum(r["cublas"] for r in base_us) / 1e6
        out["gpu_baselines"] = {
            "unit": "TFLOP/s", "timing": "per shape, R operand copies in one CUDA graph, CUDA events (as shapes[].us)",
            "sweep_ours": round(step_flops / (sum(mean_ms) / 1e3) / 1e12, 1),
            "packedlinear_unfused": {
                "value": round(step_flops / sweep_unfused / 1e12, 1),
                "what": "the reference's GPU path without the fused kernel (tools/idol_packed.py:71-79): dequantize "
                        "the GGUF Q8_0 bytes to bf16 with torch ops every call, then F.linear (cuBLAS)"},
            "cublas_bf16_dense": {
                "value": round(step_flops / sweep_cublas / 1e12, 1),
                "what": "F.linear (cuBLAS) on bf16 weights dequantized beforehand: 2 bytes per weight instead of "
                        "1.0625, no dequantization in the call"}}
        if all(r.get("triton") is not None for r in base_us):
            out["gpu_baselines"]["reference_triton_fused_linear"] = {
                "value": round(step_flops / (sum(r["triton"] for r in base_us) / 1e6) / 1e12, 1),
                "what": "the reference's own fused GPU linear (tools/idol_triton.py:94-126, Triton _linear_kernel, "
                        "bf16 activations) on the same shapes and operands; per shape in shapes[].us_reference_triton"}
        else:
            errs = [r.get("error") for r in base_us if r.get("error")]
            out["gpu_baselines"]["reference_triton_fused_linear"] = {
                "value": None, "why": errs[0] if errs else "baseline/_ref/idol_triton.py not staged"}
    del ops
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------- config 5, the stack
def make_stack(dev, blocks=STACK_BLOCKS, seed=4242):
    """The 24-block denoiser stack with seeded random Q8_0 weights (the same on every rank: replicas)."""
    import torch
    from idol_b200.block import DenoiserBlock, DenoiserStack, Q8Weight
    g = torch.Generator(device=dev).manual_seed(seed)
    D, H = BLOCK_D, BLOCK_H
    out = []
    for _ in range(blocks):
        w = {}
        for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "ff1": (H, D), "ff2": (D, H)}.items():
            w[name] = Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * 0.02,
                                          torch.randn(n, device=dev, generator=g) * 0.01)
        out.append(DenoiserBlock(w["qkv"], w["out"], w["ff1"], w["ff2"], 1 + 0.1 * torch.randn(D, device=dev, generator=g),
                                 1 + 0.1 * torch.randn(D, device=dev, generator=g), BLOCK_HEADS))
    return DenoiserStack(out)


def make_images(dev, first, count):
    """The residual streams of images first .. first + count - 1: [count * 2 * 4096, D] fp32, image i drawn from its
    own seed, so the union over ranks is the same 64 images for every N."""
    import torch
    x = torch.empty((count * CFG * BLOCK_TOKENS, BLOCK_D), device=dev)
    for j in range(count):
        g = torch.Generator(device=dev).manual_seed(9000 + first + j)
        x[j * CFG * BLOCK_TOKENS:(j + 1) * CFG * BLOCK_TOKENS] = torch.randn(
            (CFG * BLOCK_TOKENS, BLOCK_D), device=dev, generator=g).to(torch.bfloat16).float()
    return x


def block_kernel_times(block, dev, stream, seqs):
    """Each kernel of one DenoiserBlock.forward_ timed alone on that call's own shapes (seqs sequences of 4096 tokens):
    per kernel, a CUDA graph of R launches replayed 3 times between CUDA events. Returns rows with the launches per
    block, mean microseconds per launch and the algorithmic FLOPs (or bytes) per launch."""
    import torch
    from idol_b200 import _capi as C
    from idol_b200 import layers
    rows, D, H = seqs * BLOCK_TOKENS, BLOCK_D, BLOCK_H
    qkv_w, out_w, ff1_w, ff2_w = block.weights
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((rows, D), device=dev, generator=g)
    h = torch.randn((rows, D), device=dev, generator=g).to(torch.bfloat16)
    qkv = torch.empty((rows, 3 * D), device=dev, dtype=torch.bfloat16)
    f1 = torch.empty((rows, H), device=dev, dtype=torch.bfloat16)
    att = torch.empty((rows, D), device=dev, dtype=torch.bfloat16)
    qkv_w(h, out=qkv)
    ff1_w(h, act=C.ACT_GELU_TANH, out=f1)
    kernels = [
        ("norm_rows (fp32 -> bf16)", 2, lambda: layers.norm_rows(x, 1e-6, out=h), "hbm", rows * D * (4 + 2)),
        ("q8_gemm qkv 1024->3072 + rms_heads of q, k", 1,
         lambda: qkv_w.heads(h, 2 * D, D, block.q_gamma, block.k_gamma, out=qkv), "tensor", 2.0 * rows * 3 * D * D),
        ("attention", 1, lambda: layers.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], BLOCK_HEADS,
                                                  batch=seqs, out=att), "tensor",
         4.0 * BLOCK_TOKENS ** 2 * D * seqs),
        ("q8_gemm out 1024->1024 + residual", 1, lambda: out_w(att, residual=x, out=x), "tensor", 2.0 * rows * D * D),
        ("q8_gemm ff1 1024->4096 gelu", 1, lambda: ff1_w(h, act=C.ACT_GELU_TANH, out=f1), "tensor",
         2.0 * rows * H * D),
        ("q8_gemm ff2 4096->1024 + residual", 1, lambda: ff2_w(f1, residual=x, out=x), "tensor", 2.0 * rows * D * H),
    ]
    R = 10
    res = []
    for name, per_block, fn, bound, work in kernels:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()
            with torch.cuda.graph(gr, stream=stream):
                for _ in range(R):
                    fn()
            gr.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(3):
                gr.replay()
            e1.record(stream)
        stream.synchronize()
        res.append((name, per_block, e0.elapsed_time(e1) * 1e3 / (3 * R), bound, work))
        del gr
    return res


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from idol_b200.shard import image_shard
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, tc_peak, peak_kind = peaks()
    stream = torch.cuda.Stream(device=dev)

    first, count = image_shard(STACK_IMAGES, rank, world)
    seqs, chunk = count * CFG, args.chunk_images * CFG
    stack = make_stack(dev)
    x = make_images(dev, first, count)
    host_x = x.cpu().pin_memory()  # the same images, for the end-to-end pass
    torch.cuda.synchronize()

    def step():
        stack.forward_(x, seqs, chunk)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    status = pkg._capi.device_status(local_rank)

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
        for _ in range(args.steps):
            step()
        t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall1 = time.time()
    ms = t_begin.elapsed_time(t_end)
    clk = clocks.stop(wall0, wall1) if rank == 0 else None
    status = max(status, pkg._capi.device_status(local_rank))

    # End to end: the rank's images start and end in pinned host memory. Chunks of CHUNK_IMAGES images go through a
    # ring of four device buffers: host->device on one stream, the 24 blocks on two compute streams in turn (the two
    # lanes DenoiserStack.forward_ uses within one call), device->host on a fourth, so one chunk's copies overlap its
    # neighbours' compute.
    host_y = torch.empty(host_x.shape, dtype=host_x.dtype, pin_memory=True)
    rows_chunk = chunk * BLOCK_TOKENS
    nchunks = -(-seqs // chunk)
    ring = [torch.empty((rows_chunk, BLOCK_D), device=dev) for _ in range(min(4, nchunks))]
    computes = [stream, torch.cuda.Stream(device=dev)]
    copy_in, copy_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in ring]
    ev_done = [torch.cuda.Event() for _ in ring]
    ev_out = [torch.cuda.Event() for _ in ring]
    used = [False] * len(ring)
    e2e_steps = max(1, min(args.steps, 3))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    copy_in.wait_event(e0)
    copy_out.wait_event(e0)
    for _ in range(e2e_steps):
        for c in range(nchunks):
            b = c % len(ring)
            r0 = c * rows_chunk
            r1 = min(seqs * BLOCK_TOKENS, r0 + rows_chunk)
            buf = ring[b][:r1 - r0]
            with torch.cuda.stream(copy_in):
                if used[b]:
                    copy_in.wait_event(ev_out[b])
                buf.copy_(host_x[r0:r1], non_blocking=True)
                ev_in[b].record(copy_in)
            cs = computes[c % 2]
            with torch.cuda.stream(cs):
                cs.wait_event(ev_in[b])
                stack.forward_(buf, (r1 - r0) // BLOCK_TOKENS, chunk)
                ev_done[b].record(cs)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[b])
                host_y[r0:r1].copy_(buf, non_blocking=True)
                ev_out[b].record(copy_out)
            used[b] = True
    stream.wait_stream(copy_out)
    stream.wait_stream(computes[1])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    io_bytes = host_x.numel() * host_x.element_size()
    status = max(status, pkg._capi.device_status(local_rank))

    # Every kernel of a block on a chunk's shapes, timed alone (for the roofline of the dominant one).
    kern = block_kernel_times(stack.blocks[0], dev, stream, chunk)
    latency = measure_single_image_latency(stack, dev, stream, world)

    if world > 1:
        t = torch.tensor([ms, e2e_ms, float(status)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, status = float(t[0]), float(t[1]), int(t[2])
    if rank != 0:
        return

    units = STACK_BLOCKS * STACK_IMAGES
    kernels, block_us = [], sum(us * n for (_, n, us, _, _) in kern)
    for name, per_block, us, bound, work in kern:
        if bound == "tensor":
            ach, peak, unit = work / (us / 1e6) / 1e12, tc_peak, "TFLOP/s"
        else:
            ach, peak, unit = work / (us / 1e6) / 1e9, hbm_peak, "GB/s"
        kernels.append({"kernel": name, "launches_per_block": per_block, "us": round(us, 2),
                        "share": round(us * per_block / block_us, 3), "bound": bound, "achieved": round(ach, 1),
                        "unit": unit, "peak": peak, "frac": round(ach / peak, 3),
                        ("flops" if bound == "tensor" else "bytes"): work})
    top = max(kernels, key=lambda k: k["share"])
    line = {
        "metric": METRIC, "value": round(units * args.steps / (ms / 1e3), 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded normal residual streams, Q8_0 of seeded normal weights)",
        "config": config5(world),
        "images_per_s": round(STACK_IMAGES * args.steps / (ms / 1e3), 3),
        "tflops": round(units * BLOCK_FLOPS * args.steps / (ms / 1e3) / 1e12, 1),
        "e2e": {"value": round(units * e2e_steps / (e2e_ms / 1e3), 2), "unit": UNIT,
                "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes, "steps": e2e_steps,
                "api": f"DenoiserStack.forward_ per chunk of {args.chunk_images} images from pinned host memory; "
                       "H2D, compute (two lanes, chunks in turn) and D2H on four streams"},
        "roofline": {"bound": top["bound"], "kernel": top["kernel"], "achieved": top["achieved"],
                     "peak": top["peak"], "unit": top["unit"], "frac": top["frac"],
                     "peak_source": f"{peak_kind} {'bf16 burst' if top['bound'] == 'tensor' else 'copy'}",
                     "traffic": traffic_for(top["kernel"]),
                     "work_per_launch": f"{top.get('flops', top.get('bytes')):.4g} "
                                        f"{'FLOP' if top['bound'] == 'tensor' else 'bytes'} "
                                        f"({chunk} sequences x {BLOCK_TOKENS} tokens)"},
        "kernels": kernels,
        "single_request_latency": latency,
        "block_us_sum_of_kernels": round(block_us, 1),
        "block_us_in_stack": round(ms * 1e3 / args.steps / (STACK_BLOCKS * nchunks), 1),
        "gpu_launches": LAUNCHES_PER_BLOCK * STACK_BLOCKS * nchunks * args.steps,
        "device_status": status,
        "clocks": clk,
    }
    if world == 1 and not args.no_extras:
        line["gemm_sweep"] = measure_gemm_sweep(pkg, dev, stream, args.sweep_steps, args.no_gpu_baselines)
        line.update(measure_compositions(pkg, dev, stream, args))
    if world == 1 and not args.no_cpu_baseline:
        rates, times, facts = cpu_reference_measure(1, 10, budget_s=20.0)
        line["cpu_baseline"] = cpu_baseline_entry(rates, times, facts)
    print(json.dumps(line), flush=True)


def measure_single_image_latency(stack, dev, stream, world, passes=3):
    """Latency of one request: the 24-block stack over one image (2 CFG branches x 4096 tokens). On N > 1 ranks each
    block runs shard.column_parallel_block_forward_ (the MLP's ff1 and ff2 split by output features over the ranks,
    each slice all-gathered by NCCL; the result equals the one-GPU block bit for bit); on one GPU the stack itself.
    Device time of `passes` passes (CUDA events; max over ranks) and the all-gathers' share of it."""
    import torch
    import torch.distributed as dist
    from idol_b200.shard import column_parallel_block_forward_
    g = torch.Generator(device=dev).manual_seed(31)
    x0 = torch.randn((CFG * BLOCK_TOKENS, BLOCK_D), device=dev, generator=g)
    x = x0.clone()
    events = []

    def one_pass(record):
        if world == 1:
            stack.forward_(x, CFG, 1)  # each CFG branch a chunk: the two run on the stack's two lanes
        else:
            for b in stack.blocks:
                column_parallel_block_forward_(b, x, images=CFG, gather_events=events if record else None)

    with torch.cuda.stream(stream):
        for _ in range(2):
            one_pass(False)
    stream.synchronize()
    x.copy_(x0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(passes):
            one_pass(True)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    gather_ms = sum(a.elapsed_time(b) for a, b in events)
    if world > 1:
        t = torch.tensor([ms, gather_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, gather_ms = float(t[0]), float(t[1])
    return {"metric": "single-request latency: the 24-block stack over one image (2 CFG branches x 4096 tokens)",
            "ms_per_pass": round(ms / passes, 3), "passes": passes,
            "mode": ("one GPU, the two CFG branches on two streams" if world == 1 else
                     f"column-parallel MLP over {world} GPUs (ff1/ff2 split by output features, NCCL all-gather of "
                     "each slice; equal to the one-GPU result bit for bit)"),
            "all_gather_share": None if world == 1 else round(gather_ms / ms, 3)}


def traffic_for(kernel):
    """DRAM bytes per launch of a kernel from the committed ncu record, or None."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    return json.loads(f.read_text()).get(kernel, {}).get("bytes_per_launch")


def measure_compositions(pkg, dev, stream, args):
    """Config 3 (one block), config 4 (Gaussian MLP) and the decoders at the real model's size, on this GPU."""
    block_steps = mlp_steps = 30
    gs_steps, dec_steps, full_steps = 20, 5, 3
    block_ms = measure_block(pkg, dev, stream, block_steps, 1)
    mlp_ms = measure_mlp(pkg, dev, stream, mlp_steps, 1)
    gs_ms = measure_gs_block(pkg, dev, stream, gs_steps, 1)
    dec_ms = measure_gs_decoder(pkg, dev, stream, dec_steps, 1)
    full_ms = measure_decode(pkg, dev, stream, full_steps, 1)
    _, tc_peak, _ = peaks()
    return {
        "block": {"metric": "denoiser-block steps/s (config 3: 2 CFG branches x 4096 tokens, D 1024, 16 heads x 64, "
                            "Q8_0 QKV/out/MLP 1024->4096->1024, GELU tanh, fp32 residual)",
                  "value": round(block_steps / (block_ms / 1e3), 2), "unit": "block-steps/s",
                  "ms_per_step": round(block_ms / block_steps, 3), "steps": block_steps,
                  "tflops": round(BLOCK_FLOPS * block_steps / (block_ms / 1e3) / 1e12, 1),
                  "frac_tensor": round(BLOCK_FLOPS / (block_ms / block_steps / 1e3) / 1e12 / tc_peak, 3)},
        "gaussian_block": {"metric": "Gaussian-decoder block steps/s (src/decoders.cpp:296-313: 8192 anchors, "
                                     "self-attention, cross-attention to 8192 latent tokens x 16 conditions, MLP "
                                     "1024->4096->1024, D 1024, 16 heads, fp32 residual)",
                           "value": round(gs_steps / (gs_ms / 1e3), 2), "unit": "block-steps/s",
                           "ms_per_step": round(gs_ms / gs_steps, 3), "steps": gs_steps,
                           "tflops": round(GS_FLOPS * gs_steps / (gs_ms / 1e3) / 1e12, 1)},
        "gaussian_decoder": {"metric": "Gaussian decodes/s (Decoders::gaussian_features + to_gaussians: 8192 "
                                       "anchors -> 262,144 Gaussians, 16 blocks, 8192 latent tokens x 16, D 1024)",
                             "value": round(dec_steps / (dec_ms / 1e3), 3), "unit": "decodes/s",
                             "ms_per_step": round(dec_ms / dec_steps, 3), "steps": dec_steps,
                             "tflops": round(GS_FLOPS * GS_BLOCKS * dec_steps / (dec_ms / 1e3) / 1e12, 1)},
        "decode": {"metric": "Decoders::decode calls/s (latent 8192 x 16 -> sample_anchors to level 7 through the "
                             "octree decoder, 4 blocks -> Gaussian decoder, 16 blocks -> 262,144 activated Gaussians; "
                             "D 1024)", "value": round(full_steps / (full_ms / 1e3), 3), "unit": "decodes/s",
                   "ms_per_step": round(full_ms / full_steps, 2), "steps": full_steps,
                   "reference_published": "36.99 s on 8 threads and 0.34 s with the upstream GPU modules on an RTX "
                                          "4090, both octree + Gaussian decoders at 262,144 Gaussians "
                                          "(docs/data/decoder-cpu-vs-gpu.json); context only, other hardware"},
        "gaussian_mlp": {"metric": "Gaussian MLP points/s (config 4: 262,144 points, Q8_0 128->512->512->14, SiLU, "
                                   "heads)", "value": round(MLP_POINTS * mlp_steps / (mlp_ms / 1e3), 0),
                         "unit": "points/s", "ms_per_step": round(mlp_ms / mlp_steps, 3), "steps": mlp_steps,
                         "tflops": round(MLP_FLOPS * mlp_steps / (mlp_ms / 1e3) / 1e12, 1)},
    }


def run_profile_shape(args):
    """One GEMM shape (or the block / MLP composition), launched warmup + steps times back to back: the small case an
    ncu capture targets."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    if args.profile_shape in ("attention", "stack"):
        # The config-5 chunk (8 sequences x 4096 tokens): the attention kernel alone, or one pass of the 24-block
        # stack over the chunk, warmup + steps times.
        dev = torch.device("cuda", 0)
        seqs = CHUNK_IMAGES * CFG
        if args.profile_shape == "attention":
            from idol_b200 import layers
            g = torch.Generator(device=dev).manual_seed(3)
            D = BLOCK_D
            qkv = torch.randn((seqs * BLOCK_TOKENS, 3 * D), device=dev, generator=g).to(torch.bfloat16)
            out = torch.empty((seqs * BLOCK_TOKENS, D), device=dev, dtype=torch.bfloat16)
            fn = lambda: layers.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], BLOCK_HEADS,  # noqa: E731
                                          batch=seqs, out=out)
        else:
            stack = make_stack(dev)
            x = make_images(dev, 0, CHUNK_IMAGES)
            fn = lambda: stack.forward_(x, seqs)  # noqa: E731
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        print(json.dumps({"profile": args.profile_shape, "ms_per_step": round(e0.elapsed_time(e1) / args.steps, 3),
                          "device_status": pkg._capi.device_status(0)}))
        return
    if args.profile_shape in ("block", "mlp"):
        dev = torch.device("cuda", 0)
        stream = torch.cuda.Stream(device=dev)
        fn = measure_block if args.profile_shape == "block" else measure_mlp
        ms = fn(pkg, dev, stream, args.steps, 1)
        print(json.dumps({"profile": args.profile_shape, "ms_per_step": round(ms / args.steps, 3),
                          "device_status": pkg._capi.device_status(0)}))
        return
    fields = args.profile_shape.split(",")
    m, k, n = (int(v) for v in fields[:3])
    in_place = fields[3:] == ["res"]  # M,K,N,res: an fp32 output over its own fp32 residual (the blocks' out, ff2)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    packed = pkg.quantize(torch.randn((n, k), device=dev, generator=g) * 0.02)
    tiles = pkg.repack(packed, n, k)
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device=dev, generator=g) * 0.01
    if in_place:
        y = torch.randn((m, n), device=dev, generator=g)
        call = lambda: pkg.gemm_into(y, x, tiles, bias, n, k, residual=y)  # noqa: E731
    else:
        y = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
        call = lambda: pkg.gemm_into(y, x, tiles, bias, n, k)  # noqa: E731
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"profile_shape": [m, k, n], "us_per_launch": round(us, 2),
                      "tflops": round(flops(m, k, n) / us / 1e6, 1), "device_status": pkg._capi.device_status(0)}))


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


def run_reference(args, rank, world):
    """The reference arm: the block composed of the reference's own CPU functions on one image per step, on every
    usable host thread; rank 0 alone runs and prints (the other ranks exit without work)."""
    if rank != 0:
        return
    rates, times, facts = cpu_reference_measure(args.warmup, args.steps)
    v = statistics.median(rates)
    base = cpu_baseline_entry(rates, times, facts)
    print(json.dumps({
        "metric": METRIC, "value": round(v, 4), "unit": UNIT, "impl": "reference", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.median(times) * 1e3, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded normal residual streams, Q8_0 of seeded normal weights)",
        "config": config5(world), "cpu_baseline": base,
        "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--sweep-steps", type=int, default=200, help="timed sweeps of the config-2 GEMM sweep (N = 1)")
    ap.add_argument("--chunk-images", type=int, default=CHUNK_IMAGES,
                    help="images (of 2 CFG branches) per pass through the 24 blocks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-baselines", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the config-5 stack (no sweep or compositions)")
    ap.add_argument("--profile-shape", default=None,
                    help="M,K,N: run only this GEMM (warmup + steps launches) for an ncu capture (M,K,N,res: fp32 "
                         "output in place over its fp32 residual); 'block' or 'mlp' "
                         "runs the config-3 block or the config-4 MLP instead, 'attention' or 'stack' the attention "
                         "kernel or the 24-block stack on one config-5 chunk")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
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
