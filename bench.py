#!/usr/bin/env python
"""Benchmark of the B200 attention path (one JSON line on stdout, rank 0).

Workload (the configuration BASELINE.json's metric is quoted on): single-token
gated GQA decode at 32k context, bf16 KV cache, Qwen3.5-4B shapes (16 query
heads, 4 KV heads, head_dim 256), through the 8 full-attention layers of the
stack.  A step is one token through those 8 layers; per layer two kernels:
the split-KV walk (q/k norm + RoPE + KV append fused, TMA-staged K/V tiles,
both dot products on mma.sync) and the split merge + output gate.  Each
layer has its own 128 MiB cache, so a step streams 1 GiB, eight times the
126 MB L2: no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU.  The step is then one
sequence of N x 32768 positions split along the sequence, 32768 per GPU (the
same cache bytes per GPU as N = 1, so "scaling": "weak"): per layer every GPU
walks its range, pushes its partial (max, sum, output; 16,512 B) into every
GPU's exchange buffer over NVLink peer memory and merges the N partials.
`value` is the latency of one layer of that sequence, the max over ranks.
Config 4a proper (131072 positions split over the N GPUs, strong scaling) and
4b (64 sequences dealt over the GPUs, no collective) are sections of the line.

`--impl reference` times the reference's CPU implementation of the path (the
C++ restatement in oracle/, all host threads, f32 cache) on the same workload
and prints the same line with "impl": "reference"; under torchrun only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rust-llm_b200"))

CTX = 32768
N_LAYERS = 8
N_HEAD, N_KV, HD = 16, 4, 256
KV_BYTES_PER_LAYER = 2 * N_KV * CTX * HD * 2          # K + V, bf16: 134,217,728 B
METRIC = "decode attn µs/layer @32k ctx & HBM GB/s vs 8 TB/s; prefill attn TFLOPS"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def peaks_bf16():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return "measured", float(p["bf16_tflops"])
    except Exception:
        return "fallback", 1590.0


def ncu_traffic():
    """DRAM bytes per launch of the decode kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_bf16_32k.txt")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


class ClockSampler:
    """SM clocks, power and clock-event reasons of one GPU, read through NVML
    (read-only queries) every `period_s` on a background thread, from before
    the warm-up until after the timed region, plus one read right before and
    one right after the timed region (`mark`)."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, torch_device, period_s: float = 0.01):
        self.period = period_s
        self.samples = []  # (t, sm_mhz, reasons bitmask, power W)
        self.marks = {}
        self.handle = None
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(torch_device)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(props.uuid))
            except Exception:
                bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id,
                                             props.pci_device_id)
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.nvml = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                  pynvml.NVML_CLOCK_SM))
        except Exception:
            self.handle = None

    def _read(self):
        n = self.nvml
        sm = float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
        try:
            reasons = int(n.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
        except Exception:
            reasons = int(n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle))
        try:
            pw = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
        except Exception:
            pw = None
        return (time.perf_counter(), sm, reasons, pw)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._read())
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self.handle is not None:
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        return self

    def mark(self, name):
        if self.handle is not None:
            try:
                r = self._read()
                self.samples.append(r)
                self.marks[name] = r
            except Exception:
                pass

    def stop(self):
        self._stop.set()
        if self.handle is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if self.handle is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml unavailable"}
        t0 = self.marks.get("timed_start", self.samples[0])[0]
        t1 = self.marks.get("timed_end", self.samples[-1])[0]
        timed = [x for x in self.samples if t0 <= x[0] <= t1]
        window = timed if len(timed) >= 3 else self.samples
        sm = sorted(x[1] for x in window)
        reasons = sorted({name for x in window for name, bit in self.REASONS if x[2] & bit})
        pw = [x[3] for x in window if x[3] is not None]
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(window), "samples_timed_region": len(timed),
                "samples_total": len(self.samples),
                "window": "timed region" if window is timed else "warm-up through timed region",
                "sm_mhz_min": sm[0], "power_w_max": max(pw) if pw else None,
                "sm_mhz_at_timed_start": self.marks.get("timed_start", (0, None))[1],
                "sm_mhz_at_timed_end": self.marks.get("timed_end", (0, None))[1],
                "period_ms": self.period * 1e3, "source": "NVML, read-only queries"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(seconds=12.0, max_reps=20):
    """The oracle (C++ restatement of forward.rs) on one layer's decode at 32k,
    f32 cache, all host threads; time per layer in µs."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as orc
    threads = os.cpu_count() or 1
    cfg = orc.qwen35_config(CTX)
    r = orc.Rng(0)
    kv = np.empty((2, N_KV, CTX, HD), np.float32)
    kv[...] = r.normal(kv.shape)
    qg = r.normal((1, N_HEAD * 2 * HD))
    k = r.normal((1, N_KV * HD))
    v = r.normal((1, N_KV * HD))
    ones = np.ones(HD, np.float32)
    orc.full_attn(cfg, CTX - 1, qg, k, v, kv, ones, ones, threads)  # warm
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < max_reps and (len(times) < 3 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        orc.full_attn(cfg, CTX - 1, qg, k, v, kv, ones, ones, threads)
        times.append(time.perf_counter() - t0)
    us = sum(times) / len(times) * 1e6
    return us, threads, len(times)


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    us, threads, reps = cpu_baseline(seconds=max(10.0, min(60.0, 0.05 * args.steps)),
                                     max_reps=max(3, args.steps))
    sample = (f"{reps} single-layer decodes at position {CTX - 1} over a {CTX}-entry f32 "
              f"cache (16/4 heads, hd 256), {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": us, "unit": "us/layer",
        "n_gpus": world, "steps": reps, "warmup": 1, "ms_per_step": us * N_LAYERS / 1e3,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seed 0",
        "config": {"workload": "decode32k", "context": CTX, "layers": N_LAYERS,
                   "heads": [N_HEAD, N_KV, HD], "kv_dtype": "f32"},
        "cpu_baseline": {"value": us, "unit": "us/layer", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": us, "unit": "us/layer", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


DN_LAYERS = 72  # 3 x the stack's 24: 144 MiB of distinct state per step, more than L2
DN_BYTES_PER_LAYER = (2 * 32 * 128 * 128 * 4      # recurrent state read + write
                      + 2 * 8192 * 3 * 4          # conv history read + write
                      + 8192 * 4 * 4              # conv weights
                      + 4 * (8192 + 2 * 4096 + 2 * 32))  # qkv, z, out, alpha, beta


def dn_step_bench(args, dev, stream, rlcuda, torch):
    """Config 1 shapes: one Gated DeltaNet decode step per layer over 72 layers
    (three times the stack's 24, each with its own 2 MiB state, so a step moves
    144 MiB of distinct state and L2 cannot hold it), CUDA-graph captured;
    returns µs per layer and the HBM rate of the algorithmic bytes."""
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=DN_LAYERS, context=16, max_batch=1)
    ctx = rlcuda.Context(cfg, device=dev.index)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    import numpy as np
    r = np.random.default_rng(1)
    for layer in range(DN_LAYERS):
        ctx.set_weights_linear(layer, r.normal(0, 0.5, (8192, 4)).astype(np.float32),
                               -np.exp(r.uniform(0, np.log(16), 32)).astype(np.float32),
                               r.normal(0, 0.1, 32).astype(np.float32), np.ones(128, np.float32))
        ctx.write_conv(layer, r.normal(0, 0.5, (1, 8192, 3)).astype(np.float32))
        ctx.write_ssm(layer, r.normal(0, 0.1, (32, 1, 128, 128)).astype(np.float32))
    qkv = torch.randn((DN_LAYERS, 8192), generator=gen, device=dev)
    z = torch.randn((DN_LAYERS, 4096), generator=gen, device=dev)
    al = torch.randn((DN_LAYERS, 32), generator=gen, device=dev)
    be = torch.randn((DN_LAYERS, 32), generator=gen, device=dev)
    out = torch.empty((DN_LAYERS, 4096), device=dev)

    def step():
        for layer in range(DN_LAYERS):
            ctx.linear_attn(layer, 0, 1, qkv[layer], z[layer], al[layer], be[layer], out[layer])

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    steps = max(20, min(args.steps, 2000))
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            graph.replay()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    ctx.sync()
    us = e0.elapsed_time(e1) * 1e3 / (steps * DN_LAYERS)
    # one launch alone, events around it (sleep first so the host is ahead)
    ctx.profile_reset()
    ctx.profile(True)
    with torch.cuda.stream(stream):
        for b in range(10):
            torch.cuda._sleep(5_000_000)
            step()
    prof = ctx.profile_read()
    ctx.profile(False)
    ms, n = prof["dn_step"]
    graph.reset()
    # end to end through the host entry point (rl_linear_attn_host): every
    # layer's inputs from pinned host memory and its output back, host clock
    h_qkv = torch.empty((DN_LAYERS, 1, 8192), pin_memory=True)
    h_z = torch.empty((DN_LAYERS, 1, 4096), pin_memory=True)
    h_al = torch.empty((DN_LAYERS, 1, 32), pin_memory=True)
    h_be = torch.empty((DN_LAYERS, 1, 32), pin_memory=True)
    h_qkv.copy_(qkv.cpu().view(DN_LAYERS, 1, -1))
    h_z.copy_(z.cpu().view(DN_LAYERS, 1, -1))
    h_al.copy_(al.cpu().view(DN_LAYERS, 1, -1))
    h_be.copy_(be.cpu().view(DN_LAYERS, 1, -1))
    nq, nz, na, nb = h_qkv.numpy(), h_z.numpy(), h_al.numpy(), h_be.numpy()
    h_o = torch.empty((DN_LAYERS, 1, 4096), pin_memory=True)
    no = h_o.numpy()
    # the C ABI's host entry point itself, pointers made once
    host_call = rlcuda.lib().rl_linear_attn_host
    f32p = ctypes.POINTER(ctypes.c_float)
    host_args = [tuple(a[layer].ctypes.data_as(f32p) for a in (nq, nz, na, nb, no))
                 for layer in range(DN_LAYERS)]

    def e2e_layer(layer):
        code = host_call(ctx.handle, layer, 0, 1, *host_args[layer])
        if code:
            raise rlcuda.RlError(code, "rl_linear_attn_host")

    for layer in range(DN_LAYERS):  # warm
        e2e_layer(layer)
    e2e_steps = max(3, min(args.steps // 50, 50))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for layer in range(DN_LAYERS):
            e2e_layer(layer)
    e2e_us = (time.perf_counter() - t0) * 1e6 / (e2e_steps * DN_LAYERS)
    assert np.isfinite(no).all()
    ctx.close()
    peak, _ = peaks()
    gbs = DN_BYTES_PER_LAYER / (us * 1e-6) / 1e9
    return {"workload": "config 1 DeltaNet decode step, 72 layers per graph step",
            "us_per_layer": us, "bytes_per_layer": DN_BYTES_PER_LAYER, "gbs": gbs,
            "frac_of_measured_hbm": gbs / peak, "frac_of_8tbs": gbs / 8000.0,
            "avg_launch_us_alone": ms * 1e3 / max(n, 1),
            "l2": "72 x 2 MiB of state per step, more than the 126 MB L2",
            "e2e": {"value": e2e_us, "unit": "us/layer",
                    "h2d_bytes_per_layer": 4 * (8192 + 4096 + 64),
                    "d2h_bytes_per_layer": 4 * 4096,
                    "how": "rl_linear_attn_host (the C ABI) per layer, pinned host buffers, host clock"}}


PF_T = 4096
PF_LAYERS = 8
PF_FLOP_PER_LAYER = 4 * 16 * 256 * PF_T * (PF_T + 1) // 2   # causal Q K^T + P V: 137,472,507,904


def prefill_bench(args, dev, stream, rlcuda, torch):
    """Config 2's full-attention layers: 8 layers of a 4096-token causal
    prefill from an empty bf16 cache (norms + RoPE + append prologue, then the
    tcgen05 prefill kernel); returns TFLOPS per layer with and without the
    prologue, and the tensor-core kernel's share of the measured bf16 peak."""
    cfg = rlcuda.qwen35_config(n_full=PF_LAYERS, n_linear=0, context=PF_T,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=PF_T)
    ctx = rlcuda.Context(cfg, device=dev.index)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    qg = torch.randn((PF_LAYERS, PF_T, 16 * 512), generator=gen, device=dev)
    kk = torch.randn((PF_LAYERS, PF_T, 4 * 256), generator=gen, device=dev)
    vv = torch.randn((PF_LAYERS, PF_T, 4 * 256), generator=gen, device=dev)
    out = torch.empty((PF_LAYERS, PF_T, 16 * 256), device=dev)

    def step():
        for layer in range(PF_LAYERS):
            ctx.full_attn(layer, 0, PF_T, qg[layer], kk[layer], vv[layer], out[layer])

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup // 4)):
            step()
    stream.synchronize()
    ctx.sync()
    steps = max(10, min(args.steps // 100, 20))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
    stream.synchronize()
    ctx.sync()
    layer_us = e0.elapsed_time(e1) * 1e3 / (steps * PF_LAYERS)
    ctx.profile_reset()
    ctx.profile(True)
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    prof = ctx.profile_read()
    ctx.profile(False)
    kms, kn = prof["prefill"]
    pms, pn = prof["prologue"]
    ctx.close()
    kernel_us = kms * 1e3 / max(kn, 1)
    _, peak = peaks_bf16()
    return {"workload": "config 2 full-attention layers: 8 x 4096-token causal prefill, bf16 cache",
            "flop_per_layer": PF_FLOP_PER_LAYER, "us_per_layer": layer_us,
            "tflops_layer": PF_FLOP_PER_LAYER / (layer_us * 1e-6) / 1e12,
            "kernel_us": kernel_us, "prologue_us": pms * 1e3 / max(pn, 1),
            "tflops_kernel": PF_FLOP_PER_LAYER / (kernel_us * 1e-6) / 1e12,
            "frac_kernel_of_measured_bf16": PF_FLOP_PER_LAYER / (kernel_us * 1e-6) / 1e12 / peak,
            "peak_tflops": peak, "dtype": "bf16 x bf16 -> f32 (tcgen05 kind::f16)"}


DN_PF_LAYERS = 24
DN_PF_FLOP_PER_LAYER = 23.62e9  # per v head per 64-token chunk 5 C^2 d + 3 C d^2 MACs, x32 x64


def dn_prefill_bench(args, dev, stream, rlcuda, torch):
    """Config 2's DeltaNet layers: 24 layers of a 4096-token chunked prefill
    (chunk 64) from seeded states, one input set shared by the layers (the
    work per layer does not depend on the values); returns µs per layer and
    the algorithmic tensor rate (the survey's per-layer FLOP count)."""
    cfg = rlcuda.qwen35_config(n_full=0, n_linear=DN_PF_LAYERS, context=PF_T, slots=1,
                               max_batch=PF_T)
    ctx = rlcuda.Context(cfg, device=dev.index)
    ctx.set_stream(stream.cuda_stream)
    if args.dn_serial:
        ctx.set_option(rlcuda.RL_OPT_DN_OVERLAP, 0)
    import numpy as np
    r = np.random.default_rng(2)
    for layer in range(DN_PF_LAYERS):
        ctx.set_weights_linear(layer, r.normal(0, 0.5, (8192, 4)).astype(np.float32),
                               -np.exp(r.uniform(0, np.log(16), 32)).astype(np.float32),
                               r.normal(0, 0.1, 32).astype(np.float32), np.ones(128, np.float32))
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    qkv = torch.randn((PF_T, 8192), generator=gen, device=dev)
    z = torch.randn((PF_T, 4096), generator=gen, device=dev)
    al = torch.randn((PF_T, 32), generator=gen, device=dev)
    be = torch.randn((PF_T, 32), generator=gen, device=dev)
    out = torch.empty((PF_T, 4096), device=dev)

    def step():
        for layer in range(DN_PF_LAYERS):
            ctx.linear_attn(layer, 0, PF_T, qkv, z, al, be, out)

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    ctx.sync()
    steps = 2
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
    stream.synchronize()
    ctx.sync()
    ctx.close()
    us = e0.elapsed_time(e1) * 1e3 / (steps * DN_PF_LAYERS)
    _, peak = peaks_bf16()
    tf = DN_PF_FLOP_PER_LAYER / (us * 1e-6) / 1e12
    return {"workload": "config 2 DeltaNet layers: 24 x 4096-token chunked prefill (chunk 64), "
                        "f32 state between chunks",
            "us_per_layer": us, "flop_per_layer": DN_PF_FLOP_PER_LAYER,
            "tflops_algorithmic": tf, "frac_of_measured_bf16": tf / peak,
            "note": "operands as bf16 pairs (q, k in Q K^T as triples), most products three "
                    "bf16 terms (hi*hi + hi*lo + lo*hi), so the tensor pipes execute 2-6x the "
                    "algorithmic FLOP; the chunk-local Q K^T and K K^T on tcgen05 (the rest of "
                    "that kernel on mma.sync), the chunk scan on tcgen05 beside the chunk-local "
                    "kernel (off with --dn-serial)",
            "overlapped": not args.dn_serial}


VERIFY_POS, VERIFY_K = 16384, 8
VERIFY_ATTN_BYTES = 2 * N_KV * (VERIFY_POS + VERIFY_K) * HD * 2   # K + V, bf16: 67,141,632 B
VERIFY_DN_BYTES = 32 * 128 * 128 * 4 * (1 + VERIFY_K)             # read slot 0, write 8 slots
# Q K^T + P V over each row's causal prefix: 4 * 16 heads * 256 * sum_i (16384 + i + 1)
VERIFY_ATTN_FLOP = 4 * N_HEAD * HD * sum(VERIFY_POS + i + 1 for i in range(VERIFY_K))


def verify_bench(args, dev, stream, rlcuda, torch):
    """Config 3: a draft of k = 8 rows verified against a 16384-token context.
    8 full-attention layers run the 8 causal rows over the bf16 cache; 24
    DeltaNet layers run 8 sequential steps writing ring slots 1..8 of a
    9-slot ring, so accept(j) for any j is a pointer move.  Each timed pass
    restarts from slot 0 (the rollback)."""
    import numpy as np
    ctx_len = VERIFY_POS + VERIFY_K
    fcfg = rlcuda.qwen35_config(n_full=N_LAYERS, n_linear=0, context=ctx_len,
                                kv_dtype=rlcuda.RL_KV_BF16, max_batch=VERIFY_K)
    dcfg = rlcuda.qwen35_config(n_full=0, n_linear=24, context=16, slots=VERIFY_K + 1,
                                max_batch=VERIFY_K)
    fctx = rlcuda.Context(fcfg, device=dev.index)
    dctx = rlcuda.Context(dcfg, device=dev.index)
    fctx.set_stream(stream.cuda_stream)
    dctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    for layer in range(N_LAYERS):
        src = torch.randn((2, N_KV, VERIFY_POS, HD), generator=gen, device=dev)
        fctx.write_kv(layer, 0, src)
        del src
    r = np.random.default_rng(3)
    for layer in range(24):
        dctx.set_weights_linear(layer, r.normal(0, 0.5, (8192, 4)).astype(np.float32),
                                -np.exp(r.uniform(0, np.log(16), 32)).astype(np.float32),
                                r.normal(0, 0.1, 32).astype(np.float32), np.ones(128, np.float32))
    qg = torch.randn((VERIFY_K, N_HEAD * 2 * HD), generator=gen, device=dev)
    kk = torch.randn((VERIFY_K, N_KV * HD), generator=gen, device=dev)
    vv = torch.randn((VERIFY_K, N_KV * HD), generator=gen, device=dev)
    out = torch.empty((VERIFY_K, N_HEAD * HD), device=dev)
    qkv = torch.randn((VERIFY_K, 8192), generator=gen, device=dev)
    z = torch.randn((VERIFY_K, 4096), generator=gen, device=dev)
    al = torch.randn((VERIFY_K, 32), generator=gen, device=dev)
    be = torch.randn((VERIFY_K, 32), generator=gen, device=dev)
    dout = torch.empty((VERIFY_K, 4096), device=dev)

    def attn():
        for layer in range(N_LAYERS):
            fctx.full_attn(layer, VERIFY_POS, VERIFY_K, qg, kk, vv, out)

    def dn():
        for layer in range(24):
            dctx.linear_attn(layer, 0, VERIFY_K, qkv, z, al, be, dout)

    def timed(fn, reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        stream.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    reps = max(10, min(args.steps // 20, 200))
    a_us = timed(attn, reps) / N_LAYERS
    d_us = timed(dn, reps) / 24
    fctx.sync()
    dctx.sync()
    fctx.close()
    dctx.close()
    return {"workload": "config 3: k = 8 draft rows at position 16384; 8 full-attention "
                        "layers (bf16 cache) + 24 DeltaNet layers over a 9-slot state ring",
            "attn_us_per_layer": a_us, "attn_gbs": VERIFY_ATTN_BYTES / (a_us * 1e-6) / 1e9,
            "attn_tflops": VERIFY_ATTN_FLOP / (a_us * 1e-6) / 1e12,
            "attn_kernel": "prefill_kernel<verify> (tcgen05, 4 heads x 8 rows per tile, "
                           "split over the key sequence) + decode_combine_kernel",
            "dn_us_per_layer": d_us, "dn_gbs": VERIFY_DN_BYTES / (d_us * 1e-6) / 1e9,
            "pass_us": a_us * N_LAYERS + d_us * 24}


PROJ_FULL = ((8192, 2560), (1024, 2560), (1024, 2560), (2560, 4096))   # (rows, k): qg, k, v, o
PROJ_DN = ((8192, 2560), (4096, 2560), (32, 2560), (32, 2560), (2560, 4096))  # qkv, z, a, b, out


def proj_bench(args, dev, stream, rlcuda, torch):
    """The projections either side of the attention spans for one decode token
    through the 32-layer stack (8 full-attention layers: qg, k, v, o; 24
    DeltaNet layers: qkv, z, alpha, beta, out), Q4_K weights (GGUF blocks,
    distinct per layer: 734 MB, more than L2), int8 activations quantized per
    product group as Exec::matmul_group does.  CUDA-graph captured; returns µs
    per layer and the HBM rate of the weight bytes."""
    cfg = rlcuda.qwen35_config(n_full=1, n_linear=0, context=64, max_batch=1)
    ctx = rlcuda.Context(cfg, device=dev.index)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    row_bytes = lambda k: (k + 255) // 256 * 144

    def weight(rows, k):
        w = torch.randint(0, 256, (rows * (k // 256), 144), generator=gen, device=dev,
                          dtype=torch.uint8)
        w[:, 0:4] = torch.tensor([0x00, 0x20, 0x00, 0x1c], dtype=torch.uint8, device=dev)  # d, dmin
        return w
    layers = [("full", [weight(r, k) for r, k in PROJ_FULL]) for _ in range(N_LAYERS)] + \
             [("dn", [weight(r, k) for r, k in PROJ_DN]) for _ in range(24)]
    wbytes = sum(w.numel() for _, ws in layers for w in ws)
    x_in = torch.randn((1, 2560), generator=gen, device=dev)
    x_heads = torch.randn((1, 4096), generator=gen, device=dev)
    outs = {rows: torch.empty((1, rows), device=dev) for rows in (8192, 4096, 2560, 1024, 32)}

    def step_fused():
        # per layer Exec::matmul_group's two groups, one launch each (the
        # activations quantized inside): the in-projections of the normed
        # input and the out-projection of the heads
        for kind, ws in layers:
            shapes = PROJ_FULL if kind == "full" else PROJ_DN
            ctx.matmul_group(x_in, 1, 2560, [(12, w, rows, outs[rows]) for (rows, _), w in
                                             zip(shapes[:-1], ws[:-1])])
            ctx.matmul_group(x_heads, 1, 4096, [(12, ws[-1], shapes[-1][0],
                                                 outs[shapes[-1][0]])])

    def step_two():
        # the same with the quantization as its own launch before each group
        for kind, ws in layers:
            shapes = PROJ_FULL if kind == "full" else PROJ_DN
            ctx.act_quantize(x_in, 1, 2560)
            ctx.matvec_group([(12, w, rows, outs[rows]) for (rows, _), w in
                              zip(shapes[:-1], ws[:-1])])
            ctx.act_quantize(x_heads, 1, 4096)
            ctx.matvec(12, ws[-1], shapes[-1][0], outs[shapes[-1][0]])

    def timed(step):
        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        ctx.sync()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        reps = max(10, min(args.steps // 10, 100))
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
        ctx.sync()
        graph.reset()
        return e0.elapsed_time(e1) * 1e3 / reps

    fused_us = timed(step_fused)
    two_us = timed(step_two)
    step_us = min(fused_us, two_us)
    ctx.close()
    peak, _ = peaks()
    gbs = wbytes / (step_us * 1e-6) / 1e9
    n_layers = len(layers)
    return {"workload": "decode projections of the 32-layer stack (8 full: qg, k, v, o; 24 "
                        "DeltaNet: qkv, z, alpha, beta, out), Q4_K weights, t = 1",
            "us_per_token": step_us, "us_per_layer": step_us / n_layers,
            "weight_bytes_per_token": wbytes, "gbs": gbs, "frac_of_measured_hbm": gbs / peak,
            "launches_per_token": n_layers * 2 if fused_us <= two_us else n_layers * 4,
            "us_per_token_one_launch_groups": fused_us, "us_per_token_two_launch_groups": two_us,
            "arith": "int8 activations per 256-value block, integer block dots (dp4a), f32 "
                     "block scales in the reference's order (bit-identical to its scalar tier)"}


SPLIT_SEQ = 131072


def split_kv_bench(args, world, rank, dev, stream, rlcuda, torch, dist):
    """Config 4a: one sequence at 131072 positions, bf16 cache, 8 layers,
    split along the sequence across the job's GPUs; per layer each GPU walks
    its range and its merge pushes the partial (16,512 B) into every GPU's
    exchange buffer over NVLink (peer stores, then a flag); every GPU merges
    with the output gate.  Returns µs per layer (max over ranks), the same
    step with the partials all-gathered by NCCL instead, the all-gather
    alone, and each GPU's HBM rate over its share of the cache."""
    import split_kv
    lo, n = split_kv.shard_range(SPLIT_SEQ, world, rank)
    cfg = rlcuda.qwen35_config(n_full=N_LAYERS, n_linear=0, context=n,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
    ctx = rlcuda.Context(cfg, device=dev.index)
    ctx.set_stream(stream.cuda_stream)
    shard = split_kv.GpuShard(ctx, lo, SPLIT_SEQ, exchange=world > 1, rank=rank, world=world)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4 + rank)
    for layer in range(N_LAYERS):
        src = torch.randn((2, N_KV, n, HD), generator=gen, device=dev, dtype=torch.float32)
        ctx.write_kv(layer, 0, src)
        del src
    torch.cuda.empty_cache()
    gen.manual_seed(4)  # the step's inputs are the same on every rank
    qg = torch.randn((N_LAYERS, N_HEAD * 2 * HD), generator=gen, device=dev)
    kk = torch.randn((N_LAYERS, N_KV * HD), generator=gen, device=dev)
    vv = torch.randn((N_LAYERS, N_KV * HD), generator=gen, device=dev)
    out = torch.empty((N_LAYERS, N_HEAD * HD), device=dev)
    dec = split_kv.SplitDecoder(shard, world, rank, N_HEAD, HD,
                                make=lambda shape: torch.empty(shape, device=dev))
    pos = SPLIT_SEQ - 1

    def step():
        for layer in range(N_LAYERS):
            dec.step(layer, pos, qg[layer], kk[layer], vv[layer], out[layer])

    def timed(fn, reps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        stream.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    reps = max(10, min(args.steps // 10, 200))
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    ms = timed(step, reps)
    def walks():
        for layer in range(N_LAYERS):
            shard.partial(layer, pos, qg[layer], kk[layer], vv[layer], dec.partial)
    walk_ms = timed(walks, reps)
    nccl_ms = None
    if world > 1:
        shard.exchange = False  # the same step with an NCCL all-gather
        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
        nccl_ms = timed(step, reps)
        shard.exchange = True

    def gathers():
        for _ in range(N_LAYERS):
            if world > 1:
                dist.all_gather_into_tensor(dec.gathered_flat, dec.partial)
    g_ms = timed(gathers, reps)
    ctx.sync()
    ctx.close()
    us = ms * 1e3 / (reps * N_LAYERS)
    local_bytes = 2 * N_KV * n * HD * 2
    return {"workload": "config 4a: 1 sequence x 131072 positions, 8 layers, bf16 cache split "
                        f"across {world} GPU(s); partials exchanged through peer memory (64-bit "
                        "value+epoch stores over NVLink, merged on every GPU)",
            "scaling": "strong", "us_per_layer": us,
            "nccl_us_per_layer": nccl_ms * 1e3 / (reps * N_LAYERS) if nccl_ms else None,
            "walk_us_per_layer": walk_ms * 1e3 / (reps * N_LAYERS),
            "gather_us_per_layer": g_ms * 1e3 / (reps * N_LAYERS),
            "kv_bytes_per_gpu_per_layer": local_bytes,
            "hbm_gbs_per_gpu": local_bytes / (us * 1e-6) / 1e9,
            "gather_bytes_per_gpu_per_layer": N_HEAD * (HD + 2) * 4}


BATCH_SEQS, BATCH_LO, BATCH_HI = 64, 4096, 32768


def batch_bench(args, world, rank, dev, stream, rlcuda, torch, dist):
    """Config 4b: 64 independent sequences, contexts U[4096, 32768] (seed 5),
    dealt to the job's GPUs longest first (no collective); one decode row per
    sequence through 8 bf16 full-attention layers, one rl_ctx per sequence as
    the reference's Runner holds one sequence, CUDA-graph captured.  Each
    layer-step is one batched walk over all of the GPU's sequences
    (rl_batch_full_attn); the same step through one rl_full_attn per
    sequence is timed beside it.  Returns µs per layer-step of the whole
    batch (max over ranks) and the aggregate HBM rate of the cache bytes."""
    import numpy as np
    import split_kv
    lens = [int(x) for x in np.random.default_rng(5).integers(BATCH_LO, BATCH_HI + 1,
                                                              BATCH_SEQS)]
    mine = split_kv.partition_sequences(lens, world)[rank]
    gen = torch.Generator(device=dev)
    gen.manual_seed(5 + rank)
    ctxs = []
    for i in mine:
        cfg = rlcuda.qwen35_config(n_full=N_LAYERS, n_linear=0, context=lens[i] + 1,
                                   kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
        c = rlcuda.Context(cfg, device=dev.index)
        c.set_stream(stream.cuda_stream)
        src = torch.randn((2, N_KV, lens[i], HD), generator=gen, device=dev)
        for layer in range(N_LAYERS):
            c.write_kv(layer, 0, src)
        del src
        ctxs.append(c)
    torch.cuda.empty_cache()
    nb = len(mine)
    qg = torch.randn((nb, N_HEAD * 2 * HD), generator=gen, device=dev)
    kk = torch.randn((nb, N_KV * HD), generator=gen, device=dev)
    vv = torch.randn((nb, N_KV * HD), generator=gen, device=dev)
    outs = torch.empty((nb, N_HEAD * HD), device=dev)
    pos_t = torch.tensor([lens[i] for i in mine], dtype=torch.int32, device=dev)
    batch = rlcuda.Batch(ctxs) if nb else None

    def step_batched():
        for layer in range(N_LAYERS):
            batch.full_attn(layer, pos_t, qg, kk, vv, outs)

    def step_each():
        for layer in range(N_LAYERS):
            for j, i in enumerate(mine):
                ctxs[j].full_attn(layer, lens[i], 1, qg[j], kk[j], vv[j], outs[j])

    def timed(step):
        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        reps = max(3, min(args.steps // 50, 20))
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (reps * N_LAYERS)], device=dev,
                         dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        graph.reset()
        return float(t.item())

    us = timed(step_batched) if nb else 0.0
    us_each = timed(step_each) if nb else 0.0
    if batch:
        batch.close()
    for c in ctxs:
        c.sync()
        c.close()
    torch.cuda.empty_cache()
    total = sum(lens) * 2 * N_KV * HD * 2  # cache bytes of one layer over the batch
    return {"workload": f"config 4b: {BATCH_SEQS} sequences, contexts U[{BATCH_LO}, {BATCH_HI}] "
                        f"(seed 5), 8 bf16 full-attention layers, longest-first over {world} "
                        "GPU(s), no collective",
            "scaling": "strong", "sequences_per_gpu": len(mine),
            "us_per_layer_step": us, "kv_bytes_per_layer": total,
            "hbm_gbs_aggregate": total / (us * 1e-6) / 1e9,
            "launch": "rl_batch_full_attn: one walk + one merge launch per layer for all of "
                      "the GPU's sequences",
            "launches_per_step": 2 * N_LAYERS,
            "per_sequence_us_per_layer_step": us_each,
            "per_sequence_hbm_gbs_aggregate": total / (us_each * 1e-6) / 1e9}


def max_over_ranks(x, world, dev, torch, dist):
    if world == 1:
        return float(x)
    t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import rlcuda
    import split_kv

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    clocks = ClockSampler(dev).start()  # through warm-up and the timed region

    # N = 1: one sequence at 32k.  N > 1: one sequence of N x 32k positions,
    # each GPU holding a contiguous 32k of it (the same cache bytes per GPU
    # as N = 1, so "weak" scaling), its partial merged over NVLink peer memory
    # every layer; `value` is still the latency of one layer of the sequence.
    seq = CTX * world
    lo, n = split_kv.shard_range(seq, world, rank)
    assert n == CTX
    cfg = rlcuda.qwen35_config(n_full=N_LAYERS, n_linear=0, context=CTX,
                               kv_dtype=rlcuda.RL_KV_BF16, max_batch=1)
    ctx = rlcuda.Context(cfg, device=local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    if world > 1:
        split_kv.GpuShard(ctx, lo, seq, exchange=True, rank=rank, world=world)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    for layer in range(N_LAYERS):
        src = torch.randn((2, N_KV, CTX, HD), generator=gen, device=dev, dtype=torch.float32)
        ctx.write_kv(layer, 0, src)
        del src
    torch.cuda.empty_cache()
    gen.manual_seed(1234)  # the row's inputs: the same on every GPU of the sequence
    qg = torch.randn((N_LAYERS, 1, N_HEAD * 2 * HD), generator=gen, device=dev)
    kk = torch.randn((N_LAYERS, 1, N_KV * HD), generator=gen, device=dev)
    vv = torch.randn((N_LAYERS, 1, N_KV * HD), generator=gen, device=dev)
    out = torch.empty((N_LAYERS, 1, N_HEAD * HD), device=dev)
    pos = seq - 1

    def step():
        for layer in range(N_LAYERS):
            if world == 1:
                ctx.full_attn(layer, pos, 1, qg[layer], kk[layer], vv[layer], out[layer])
            else:
                ctx.full_attn_split(layer, pos, qg[layer], kk[layer], vv[layer], out[layer])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def capture():
        barrier()
        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        ctx.sync()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        return g

    def replay(g, n):
        # replays run on the current stream: keep it the library's stream,
        # which the timing events are recorded on
        with torch.cuda.stream(stream):
            for _ in range(n):
                g.replay()

    graph = capture()
    replay(graph, args.warmup)
    stream.synchronize()

    # ---- timed region: K graph replays of the 8-layer decode step
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks.mark("timed_start")
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    clocks.mark("timed_end")
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev, torch, dist)
    ctx.sync()
    graph.reset()
    kernels_per_layer = 2 if world == 1 else 3  # walk + merge (+ peer merge)
    launches = args.steps * N_LAYERS * kernels_per_layer
    us_per_layer = ms * 1e3 / (args.steps * N_LAYERS)
    hbm_gbs = world * KV_BYTES_PER_LAYER / (us_per_layer * 1e-6) / 1e9

    # ---- the walk kernel inside the same graph-timed, programmatically
    # overlapped step: each launch stamps its first CTA's start and its last
    # CTA's end on the GPU's global timer (no events, so the overlap stays)
    ctx.set_option(rlcuda.RL_OPT_WALK_SPANS, 1)
    graph = capture()
    replay(graph, args.warmup)
    stream.synchronize()
    ctx.profile_reset()
    span_steps = max(args.steps, 20)
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record(stream)
        replay(graph, span_steps)
        e3.record(stream)
    stream.synchronize()
    span_ms, span_n = ctx.profile_read()["walk_span"]
    span_step_us = max_over_ranks(e2.elapsed_time(e3) * 1e3 / (span_steps * N_LAYERS), world,
                                  dev, torch, dist)
    avg_us = max_over_ranks(span_ms * 1e3 / max(span_n, 1), world, dev, torch, dist)
    graph.reset()
    ctx.set_option(rlcuda.RL_OPT_WALK_SPANS, 0)
    achieved = KV_BYTES_PER_LAYER / (avg_us * 1e-6) / 1e9
    peak, peak_kind = peaks()
    assert avg_us <= span_step_us * 1.001, (avg_us, span_step_us)

    # ---- end to end through the public API with host buffers, on a host
    # clock: per layer the row's inputs go in from pinned host memory and its
    # output comes back (a caller needs it before the layer's projection)
    h_qg = torch.empty((N_LAYERS, 1, N_HEAD * 2 * HD), pin_memory=True)
    h_k = torch.empty((N_LAYERS, 1, N_KV * HD), pin_memory=True)
    h_v = torch.empty((N_LAYERS, 1, N_KV * HD), pin_memory=True)
    h_out = torch.empty((N_LAYERS, 1, N_HEAD * HD), pin_memory=True)
    h_qg.copy_(qg.cpu())
    h_k.copy_(kk.cpu())
    h_v.copy_(vv.cpu())
    n_qg, n_k, n_v, n_out = h_qg.numpy(), h_k.numpy(), h_v.numpy(), h_out.numpy()
    # N = 1: the C ABI's host entry point itself, as the reference's Runner
    # would call it (pointers made once; no per-call Python marshalling)
    host_call = rlcuda.lib().rl_full_attn_host
    f32p = ctypes.POINTER(ctypes.c_float)
    host_args = [tuple(a[layer].ctypes.data_as(f32p) for a in (n_qg, n_k, n_v, n_out))
                 for layer in range(N_LAYERS)]

    def e2e_layer(layer):
        if world == 1:
            code = host_call(ctx.handle, layer, pos, 1, *host_args[layer])
            if code:
                raise rlcuda.RlError(code, "rl_full_attn_host")
            return n_out[layer]
        with torch.cuda.stream(stream):
            qg[layer].copy_(h_qg[layer], non_blocking=True)
            kk[layer].copy_(h_k[layer], non_blocking=True)
            vv[layer].copy_(h_v[layer], non_blocking=True)
            ctx.full_attn_split(layer, pos, qg[layer], kk[layer], vv[layer], out[layer])
            h_out[layer].copy_(out[layer], non_blocking=True)
        stream.synchronize()
        return h_out[layer].numpy()

    e2e_steps = max(3, min(args.steps // 10, 500))
    for layer in range(N_LAYERS):  # warm
        e2e_layer(layer)
    barrier()
    t0 = time.perf_counter()
    last = None
    for _ in range(e2e_steps):
        for layer in range(N_LAYERS):
            last = e2e_layer(layer)
    t1 = time.perf_counter()
    e2e_us = max_over_ranks((t1 - t0) * 1e6 / (e2e_steps * N_LAYERS), world, dev, torch, dist)
    assert last is not None and np.isfinite(last).all()
    ctx.sync()
    h2d = N_LAYERS * 4 * (N_HEAD * 2 * HD + 2 * N_KV * HD)
    d2h = N_LAYERS * 4 * N_HEAD * HD
    ctx.close()
    clocks.stop()

    split = (split_kv_bench(args, world, rank, dev, stream, rlcuda, torch, dist)
             if not args.no_split else None)
    dn = dn_step_bench(args, dev, stream, rlcuda, torch) if not args.no_dn else None
    proj = proj_bench(args, dev, stream, rlcuda, torch) if not args.no_proj else None
    pf = prefill_bench(args, dev, stream, rlcuda, torch) if not args.no_prefill else None
    dnpf = dn_prefill_bench(args, dev, stream, rlcuda, torch) if not args.no_dn_prefill else None
    ver = verify_bench(args, dev, stream, rlcuda, torch) if not args.no_verify else None
    batch = (batch_bench(args, world, rank, dev, stream, rlcuda, torch, dist)
             if not args.no_batch else None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        us, threads, reps = cpu_baseline()
        cpu = {"value": us, "unit": "us/layer", "cores": threads, "kind": "port",
               "sample": f"{reps} single-layer decodes at position {CTX - 1} over a "
                         f"{CTX}-entry f32 cache (the reference has no bf16 cache), "
                         f"C++ restatement of forward.rs, {threads} threads"}

    traffic = ncu_traffic()
    if world == 1:
        parallelism = "one GPU, one sequence"
        workload = "decode32k"
    else:
        parallelism = (f"sequence split x{world}: one sequence of {seq} positions, {CTX} per "
                       "GPU; per layer each GPU walks its range and pushes its partial "
                       "(16,512 B) to every GPU over NVLink peer memory, every GPU merges")
        workload = f"decode32k per GPU, one {seq}-position sequence"
    line = {
        "metric": METRIC, "value": us_per_layer, "unit": "us/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) KV (torch.Generator seed 1234+rank) and q/k/v/gate (seed 1234)",
        "config": {"workload": workload, "context_per_gpu": CTX, "sequence": seq,
                   "layers": N_LAYERS, "heads": [N_HEAD, N_KV, HD], "kv_dtype": "bf16",
                   "rows": 1, "parallelism": parallelism,
                   "l2": "inputs larger than L2: 8 layers x 128 MiB KV per GPU per step",
                   "launch": "CUDA graph of the 8-layer step, programmatic launch overlap"},
        "hbm_gbs": hbm_gbs,
        "hbm_frac_of_8tbs": hbm_gbs / 8000.0 / world,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "decode_mma_kernel<fused> (split-KV walk)",
                     "peak_source": peak_kind, "avg_launch_us": avg_us,
                     "avg_launch_from": "global-timer span of every walk launch (first CTA "
                                        "start to last CTA end) inside the graph-timed step",
                     "span_step_us_per_layer": span_step_us,
                     "walk_share_of_layer": avg_us / span_step_us},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_us, "unit": "us/layer", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "how": "host clock around every layer's call of rl_full_attn_host (the C ABI: "
                       "pinned host inputs copied in, the kernels, the output copied back)"
                       if world == 1 else
                       "host clock around every layer's pinned copies in, the split call and "
                       "the copy of its output back"},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "prefill_tflops": pf["tflops_layer"] if pf else None,
        "prefill": pf,
        "dn_prefill": dnpf,
        "verify": ver,
        "config2_attention_ms": ((pf["us_per_layer"] * PF_LAYERS + dnpf["us_per_layer"] *
                                  DN_PF_LAYERS) / 1e3 if pf and dnpf else None),
        "dn_step": dn,
        "projections": proj,
        "batch_4b": batch,
        "split_kv": split,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dn", action="store_true", help="skip the DeltaNet step section")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the full-attention prefill section")
    ap.add_argument("--no-dn-prefill", action="store_true",
                    help="skip the DeltaNet chunked-prefill section")
    ap.add_argument("--dn-serial", action="store_true",
                    help="run the chunk scan after the chunk-local kernel rather than beside it "
                         "(for profilers that serialise kernels, under which the overlapped "
                         "scan waits for chunks that cannot arrive and gives up)")
    ap.add_argument("--no-verify", action="store_true", help="skip the speculative-verify section")
    ap.add_argument("--no-batch", action="store_true",
                    help="skip the config-4b batched multi-sequence section")
    ap.add_argument("--no-split", action="store_true",
                    help="skip the long-context split-sequence section")
    ap.add_argument("--no-proj", action="store_true",
                    help="skip the projections (k-quant matvec) section")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="full-attention layers per step (8 in the model; fewer only to "
                         "keep a profiler capture small)")
    args = ap.parse_args()
    globals()["N_LAYERS"] = args.layers
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
