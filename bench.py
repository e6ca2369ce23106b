#!/usr/bin/env python3
"""Benchmark of the W4A6 GEMM (MXFP6 activations x NVFP4 weights transcoded on chip).

Workload (the decode sweep): N=14336, K=4096, M in {1,4,16,32,64}.
One step = for each M, one GEMM against each of L=8 distinct weight matrices (a decode pass
over 8 layers), i.e. 40 GEMMs reading 8 x 33.0 MB of NVFP4 weights per M. The 8 matrices
(264 MB) exceed the 126 MB L2, so every GEMM streams its weights from HBM.

Metric: decode weight GB/s = weight bytes (N*K/2 codes + N*K/16 E4M3 scales + 4) per GEMM,
summed over the step, divided by the step time. Multi-GPU (torchrun): every rank holds its own
N-shard of a (14336*world) x 4096 weight matrix per layer and runs the same sweep with no
collective in the timed region (weak scaling); the time is the max over ranks.

--impl reference times the reference's CPU path (the oracle port of kernel/nvfp4_codec.py +
dequantise + fp32 matmul) on the host cores instead.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_W, K_W = 14336, 4096
M_SWEEP = (1, 4, 16, 32, 64)
LAYERS = 8
METRIC = "decode weight GB/s (W4A6 GEMM, NVFP4 weights transcoded on chip)"
UNIT = "GB/s"


def weight_bytes(N, K):
    return N * K // 2 + N * K // 16 + 4


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def load_traffic():
    """dram bytes per weight byte of the GEMM kernel, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "w4a6_gemm_decode.md")
    try:
        for line in open(p):
            if line.startswith("traffic_per_weight_byte:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler(threading.Thread):
    """Samples SM clock, max clock, power and clock-event reasons via NVML (read only)."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80, "gpu_idle": 0x1,
        "applications_clocks_setting": 0x2,
    }

    def __init__(self, index, period=0.01):
        super().__init__(daemon=True)
        self.index, self.period = index, period
        self.samples = []
        self.stop_evt = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report it instead of guessing
            self.err = repr(e)

    def run(self):
        while self.ok and not self.stop_evt.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((sm, rs, pw))
            except Exception:
                pass
            time.sleep(self.period)

    def summary(self):
        self.stop_evt.set()
        self.join(timeout=2)
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, rs, _ in self.samples:
            for name, bit in self.REASONS.items():
                if rs & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "power_w_max": max(p for _, _, p in self.samples), "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------
# CPU leg: the reference's CPU path (oracle port), timed on the host cores.

def cpu_reference_run(seconds=10.0, rows=512):
    """Per GEMM of the sweep: NVFP4 -> MXFP6 transcode of a `rows`-row slice of the weights
    (C restatement, all threads), dequantisation, fp32 matmul (OpenBLAS) with M tokens.
    Returns (weight GB/s, cores, sample description)."""
    import ctypes
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    lib_path = os.path.join(ROOT, "oracle", "liborc.so")
    if not os.path.exists(lib_path):
        import subprocess
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True,
                       capture_output=True)
    lib = ctypes.CDLL(lib_path)
    lib.orc_transcode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.orc_dequant.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                ctypes.c_void_p, ctypes.c_int]
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(2)
    K = K_W
    packed = rng.integers(0, 256, (rows, K // 2), dtype=np.uint8)
    scales = rng.integers(0x58, 0x7F, (rows, K // 16), dtype=np.uint8)
    nblk = rows * K // 32
    e6 = np.empty(nblk * 32, np.uint8)
    e8 = np.empty(nblk, np.uint8)
    Bf = np.empty((rows, K), np.float32)
    acts = {M: rng.standard_normal((M, K)).astype(np.float32) for M in M_SWEEP}
    done = 0
    t0 = time.perf_counter()
    while True:
        for M in M_SWEEP:
            lib.orc_transcode(packed.ctypes.data, scales.ctypes.data, nblk, 16, e6.ctypes.data,
                              e8.ctypes.data, cores)
            lib.orc_dequant(e6.ctypes.data, e8.ctypes.data, nblk, Bf.ctypes.data, cores)
            _ = acts[M] @ Bf.T
            done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = done * weight_bytes(rows, K) / el / 1e9
    sample = (f"{done} GEMMs of the M sweep on a {rows}x{K} weight slice "
              f"(transcode + dequant + fp32 matmul), {el:.1f} s")
    return gbs, cores, sample


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    t_run = time.perf_counter()
    vals = []
    for _ in range(max(1, args.warmup)):
        cpu_reference_run(seconds=0.5)
    for _ in range(args.steps):
        v, cores, sample = cpu_reference_run(seconds=max(0.25, args.cpu_seconds / max(1, args.steps)))
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes -> fp32", "data": "synthetic",
        "config": {"workload": f"decode sweep N={N_W} K={K_W} M in {list(M_SWEEP)}",
                   "path": "CPU oracle port of the reference codec + numpy fp32 matmul"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t_run,
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------------
# GPU leg

def run_ours(args, rank, world, local_rank):
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    bd.load()
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    def rand_u8(shape, lo, hi):
        return torch.randint(lo, hi, shape, dtype=torch.uint8, device=dev, generator=g)

    # weights: L layers of this rank's N-shard, NVFP4 bytes (values do not change the timing)
    weights = []
    for _ in range(LAYERS):
        codes = rand_u8((N_W, K_W // 2), 0, 256)
        sc = rand_u8((N_W, K_W // 16), 0x58, 0x7F)
        weights.append(ops.pack_weights(codes, sc, 1.0 / 2688.0))
        del codes, sc
    # activations per M (natural codes + scales, packed once for the kernel-level leg)
    nat = {M: (rand_u8((M, K_W), 0, 64), rand_u8((M, K_W // 32), 120, 135)) for M in M_SWEEP}
    acts = {M: ops.pack_activations(*nat[M]) for M in M_SWEEP}
    outs = {M: torch.empty((M, N_W), dtype=torch.bfloat16, device=dev) for M in M_SWEEP}
    splits = {M: 0 for M in M_SWEEP}   # 0 = persistent stream-K schedule
    wss = {M: ops.Workspace() for M in M_SWEEP}
    launches_per_step = len(M_SWEEP) * LAYERS

    # no-output guard (kernel/bench_sweep.py:297-326): a launch must write C
    for M in M_SWEEP:
        outs[M].zero_()
        ops.w4a6_gemm(acts[M], weights[0], out=outs[M], split_k=splits[M], workspace=wss[M])
    torch.cuda.synchronize()
    if not all(bool(outs[M].any()) for M in M_SWEEP):
        raise RuntimeError("W4A6 GEMM wrote no output; refusing to time it")
    if bd.device_error() != 0:
        raise RuntimeError("kernel error word set")

    stream = torch.cuda.Stream(device=dev)
    # consecutive GEMMs overlap: each may start streaming its (static) weights while the
    # previous one finishes; A, C and the workspace wait for the previous kernel
    ov = not args.no_overlap

    def step_kernels():
        for M in M_SWEEP:
            for w in weights:
                ops.w4a6_gemm(acts[M], w, out=outs[M], split_k=splits[M], workspace=wss[M],
                              stream=stream, overlap_prev=ov, weights_static=ov)

    # e2e: pinned host inputs -> device, pack (public API), GEMMs, device -> pinned host outputs
    h_in = {M: (torch.empty((M, K_W), dtype=torch.uint8).pin_memory(),
                torch.empty((M, K_W // 32), dtype=torch.uint8).pin_memory()) for M in M_SWEEP}
    for M in M_SWEEP:
        h_in[M][0].copy_(nat[M][0].cpu())
        h_in[M][1].copy_(nat[M][1].cpu())
    h_out = {M: torch.empty((M, N_W), dtype=torch.bfloat16).pin_memory() for M in M_SWEEP}
    d_in = {M: (torch.empty_like(nat[M][0]), torch.empty_like(nat[M][1])) for M in M_SWEEP}
    e2e_acts = {}
    h2d = sum(M * K_W + M * K_W // 32 for M in M_SWEEP)
    d2h = sum(M * N_W * 2 for M in M_SWEEP)

    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)

    e2e_order = sorted(M_SWEEP, reverse=True)  # the largest output returns first, not last

    def step_e2e():
        # each batch's input goes over (its scales re-laid out; the codes are used in place) on
        # a side stream, and its GEMMs wait only for that batch; the GEMMs run as one
        # programmatic-launch chain, and each batch's output returns on a second side stream
        # while later GEMMs run
        cur = torch.cuda.current_stream()
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        ready = {}
        with torch.cuda.stream(s_in):
            for M in e2e_order:
                d_in[M][0].copy_(h_in[M][0], non_blocking=True)
                d_in[M][1].copy_(h_in[M][1], non_blocking=True)
                e2e_acts[M] = ops.pack_activations(d_in[M][0], d_in[M][1], stream=s_in,
                                                   inplace=True)
                ready[M] = torch.cuda.Event()
                ready[M].record(s_in)
        for M in e2e_order:
            cur.wait_event(ready[M])
            for w in weights:
                ops.w4a6_gemm(e2e_acts[M], w, out=outs[M], split_k=splits[M],
                              workspace=wss[M], stream=cur, overlap_prev=ov,
                              weights_static=ov)
            done = torch.cuda.Event()
            done.record(cur)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                h_out[M].copy_(outs[M], non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    def capture(fn):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn()  # warm the allocator outside the graph
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=stream):
                fn()
        return graph

    g_k = capture(step_kernels)
    g_e = capture(step_e2e)

    def timed(graph, steps, warmup, clocks=None):
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        if clocks is not None:
            clocks.start()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            t0.record(stream)
            for _ in range(steps):
                graph.replay()
            t1.record(stream)
        torch.cuda.synchronize()
        clk = clocks.summary() if clocks is not None else None
        if world > 1:
            torch.distributed.barrier()
        ms = t0.elapsed_time(t1)
        if world > 1:
            tt = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            ms = float(tt.item())
        return ms, clk

    clocks = ClockSampler(local_rank)
    ms_k, clk = timed(g_k, args.steps, args.warmup, clocks)
    ms_e, _ = timed(g_e, max(3, args.steps // 2), args.warmup)
    steps_e = max(3, args.steps // 2)
    # the host copies hold each batch's last-layer output: it must equal a fresh device GEMM
    for M in M_SWEEP:
        ref = ops.w4a6_gemm(acts[M], weights[-1], split_k=splits[M]).cpu()
        if not torch.equal(ref, h_out[M]):
            raise RuntimeError(f"e2e output for M={M} differs from the device GEMM")

    wb_step = len(M_SWEEP) * LAYERS * weight_bytes(N_W, K_W)
    value = world * wb_step * args.steps / (ms_k / 1e3) / 1e9
    e2e_val = world * wb_step * steps_e / (ms_e / 1e3) / 1e9
    flops_step = sum(2 * M * N_W * K_W * LAYERS for M in M_SWEEP)

    # roofline of the dominant kernel, w4a6_gemm_kernel<16> (the M = 1, 4, 16 launches): its
    # launches alone in a graph, timed with CUDA events on the launching stream
    dom_M = [M for M in M_SWEEP if M <= 16]

    def step_dom():
        for M in dom_M:
            for w in weights:
                ops.w4a6_gemm(acts[M], w, out=outs[M], split_k=splits[M], workspace=wss[M],
                              stream=stream, overlap_prev=ov, weights_static=ov)
    g_d = capture(step_dom)
    ms_d, _ = timed(g_d, args.steps, args.warmup)
    n_dom = len(dom_M) * LAYERS
    alg_dom = [weight_bytes(N_W, K_W) + M * K_W + M * K_W // 32 + 2 * M * N_W for M in dom_M]
    alg_per_launch = sum(alg_dom) / len(alg_dom)
    us_per_launch = ms_d * 1e3 / (args.steps * n_dom)
    peaks, peak_kind = load_peaks()
    achieved = alg_per_launch / (us_per_launch * 1e-6) / 1e9
    tpw = load_traffic()
    del g_d

    extra = {}
    if not args.no_prefill and world == 1:
        extra["prefill"] = prefill_bench(torch, ops, dev, g, peaks)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_k / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "mxfp6 x mxfp6 (fp32 accumulate, bf16 out)",
        "data": "synthetic (uniform random E2M1 codes and E4M3 scale bytes; timing is value-independent)",
        "config": {"workload": f"decode sweep N={N_W} K={K_W} M in {list(M_SWEEP)} x {LAYERS} layers",
                   "per_rank_N": N_W, "global_N": N_W * world, "K": K_W,
                   "schedule": "persistent stream-K (tiles split across CTAs finished in-kernel)",
                   "l2": f"{LAYERS} weight matrices per rank ({LAYERS * weight_bytes(N_W, K_W) / 1e6:.0f} MB) "
                         "rotate, larger than the 126 MB L2",
                   "parallelism": f"N-sharded x{world}, no collective in the timed region",
                   "launch": "CUDA graph of one step" + (
                       ", programmatic serialisation between GEMMs" if ov else "")},
        "tflops": flops_step * args.steps / (ms_k / 1e3) / 1e12 * world,
        "roofline": {"bound": "hbm", "kernel": "w4a6_gemm_kernel<16> (launches with M = 1, 4, 16)",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind,
                     "traffic": (tpw * weight_bytes(N_W, K_W)) if tpw else None,
                     "algorithmic_bytes_per_launch": alg_per_launch,
                     "us_per_launch": us_per_launch,
                     "note": "achieved = algorithmic bytes per launch (weights + A + C) / the "
                             "kernel's mean launch duration (CUDA events over a graph of its "
                             "launches); traffic = DRAM bytes per launch from the committed ncu "
                             "summary (profiles/w4a6_gemm_decode.md)"},
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "pinned host A -> device, bd_pack_a, bd_w4a6_gemm x layers, C -> pinned host"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
        **extra,
    }
    del g_k, g_e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_reference_run(seconds=args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def prefill_bench(torch, ops, dev, g, peaks):
    """BASELINE config 3 shapes at M=8192 (gate/up 14336x4096, down 4096x14336): TFLOPS."""
    res = {}
    for name, (N, K) in {"gate_up": (14336, 4096), "down": (4096, 14336)}.items():
        M = 8192
        w = ops.pack_weights(torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev,
                                           generator=g),
                             torch.randint(0x58, 0x7F, (N, K // 16), dtype=torch.uint8, device=dev,
                                           generator=g), 1.0)
        a = ops.pack_activations(torch.randint(0, 64, (M, K), dtype=torch.uint8, device=dev,
                                               generator=g),
                                 torch.randint(120, 135, (M, K // 32), dtype=torch.uint8,
                                               device=dev, generator=g))
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        wsp = ops.Workspace()
        for _ in range(3):
            ops.w4a6_gemm(a, w, out=out, workspace=wsp)
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        it = 10
        t0.record()
        for _ in range(it):
            ops.w4a6_gemm(a, w, out=out, workspace=wsp)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / it
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        res[name] = {"M": M, "N": N, "K": K, "ms": ms, "tflops": tf,
                     "frac_of_2x_bf16_peak": tf / (2.0 * peaks["bf16_tflops"])}
    return res


def run_case(args):
    """One kernel shape, repeated: `--case gemm` (a single W4A6 GEMM), `--case transcode`
    (the standalone NVFP4 -> MXFP6 transcode of config 5), `--case quantize` (the MXFP6
    activation quantiser) or `--case quantize_b` (the NVFP4 weight quantiser; bytes count the
    two passes over the weights). Prints its own JSON line; used for Nsight Compute captures of one
    launch."""
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if args.case == "gemm":
        # weight matrices rotate so the working set exceeds the 126 MB L2; the calls are
        # captured in one CUDA graph so the time is device time, not host launch overhead
        M, N, K = args.M, args.N, args.K
        reps = max(2, -(-300_000_000 // weight_bytes(N, K)))
        ws_list = [ops.pack_weights(torch.randint(0, 256, (N, K // 2), dtype=torch.uint8,
                                                  device=dev, generator=g),
                                    torch.randint(0x58, 0x7F, (N, K // 16), dtype=torch.uint8,
                                                  device=dev, generator=g), 1.0)
                   for _ in range(reps)]
        a = ops.pack_activations(torch.randint(0, 64, (M, K), dtype=torch.uint8, device=dev,
                                               generator=g),
                                 torch.randint(120, 135, (M, K // 32), dtype=torch.uint8,
                                               device=dev, generator=g))
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        split = args.split
        wsp = ops.Workspace()
        stream = torch.cuda.Stream(device=dev)
        ov = bool(args.overlap)

        def body():
            for i in range(args.steps):
                ops.w4a6_gemm(a, ws_list[i % reps], out=out, split_k=split, workspace=wsp,
                              stream=stream, overlap_prev=ov, weights_static=ov)
        with torch.cuda.stream(stream):
            body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        fn = graph.replay  # noqa: E731
        calls = args.steps
        work = {"M": M, "N": N, "K": K, "split_k": split, "overlap": ov, "rotating_weights": reps,
                "weight_bytes": weight_bytes(N, K), "flops": 2 * M * N * K}
    elif args.case == "linear":
        # raw bf16 activations -> on-device quantiser -> GEMM (w4a6_linear), over rotating
        # weight matrices, captured in one CUDA graph
        M, N, K = args.M, args.N, args.K
        reps = max(2, -(-300_000_000 // weight_bytes(N, K)))
        ws_list = [ops.pack_weights(torch.randint(0, 256, (N, K // 2), dtype=torch.uint8,
                                                  device=dev, generator=g),
                                    torch.randint(0x58, 0x7F, (N, K // 16), dtype=torch.uint8,
                                                  device=dev, generator=g), 1.0)
                   for _ in range(reps)]
        x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        wsp = ops.Workspace()
        stream = torch.cuda.Stream(device=dev)

        def body():
            for i in range(args.steps):
                ops.w4a6_linear(x, ws_list[i % reps], out=out, workspace=wsp, stream=stream)
        with torch.cuda.stream(stream):
            body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        fn = graph.replay  # noqa: E731
        calls = args.steps
        work = {"M": M, "N": N, "K": K, "rotating_weights": reps,
                "weight_bytes": weight_bytes(N, K), "flops": 2 * M * N * K}
    elif args.case == "quantize":
        # fp32/bf16 activations -> GEMM-ready MXFP6 (codes + tiled scales) in one launch per
        # call; the calls are captured in one CUDA graph (device time)
        M, K = args.M, args.K
        xdt = torch.bfloat16 if args.xdtype == "bf16" else torch.float32
        x = torch.randn((M, K), device=dev, generator=g).to(xdt)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            ops.quantize_activations(x, stream=stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(args.steps):
                ops.quantize_activations(x, stream=stream)
        fn = graph.replay  # noqa: E731
        calls = args.steps
        work = {"M": M, "K": K, "x_dtype": args.xdtype,
                "bytes": M * K * (x.element_size() + 1) + M * K // 32}
    elif args.case == "quantize_b":
        # fp32/bf16 weights (N, K) -> NVFP4 codes + E4M3 scales + tensor scale (amax pass and
        # quantise pass), captured in one CUDA graph
        N, K = args.N, args.K
        wdt = torch.bfloat16 if args.xdtype == "bf16" else torch.float32
        w = (torch.randn((N, K), device=dev, generator=g) * 0.02).to(wdt)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            ops.quantize_nvfp4(w, stream=stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(args.steps):
                ops.quantize_nvfp4(w, stream=stream)
        fn = graph.replay  # noqa: E731
        calls = args.steps
        work = {"N": N, "K": K, "w_dtype": args.xdtype,
                "bytes": N * K * (2 * w.element_size() + 0.5) + N * K // 16}
    else:
        nblk = args.nblk
        codes = torch.randint(0, 256, (nblk * 16,), dtype=torch.uint8, device=dev, generator=g)
        sc = torch.randint(0x01, 0x7F, (nblk * 2,), dtype=torch.uint8, device=dev, generator=g)
        e6 = torch.empty(nblk * 32, dtype=torch.uint8, device=dev)
        e8 = torch.empty(nblk, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream()
        fn = lambda: ops.transcode(codes, sc, 16, e2m3=e6, e8m0=e8)  # noqa: E731
        calls = 1
        work = {"nblk32": nblk, "bytes": nblk * (16 + 2 + 32 + 1)}
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup if args.case not in ("gemm", "linear", "quantize",
                                                               "quantize_b") else 3)):
            fn()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    reps_t = 3 if args.case in ("gemm", "linear", "quantize", "quantize_b") else args.steps
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(reps_t):
            fn()
        t1.record(stream)
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / (reps_t * calls)
    res = {"case": args.case, "us_per_call": us, **work}
    if args.case in ("gemm", "linear"):
        res["weight_gbs"] = work["weight_bytes"] / us / 1e3
        res["tflops"] = work["flops"] / us / 1e6
    else:
        res["gbs"] = work["bytes"] / us / 1e3
    if bd.device_error() != 0:
        raise RuntimeError("kernel error word set")
    print(json.dumps(res), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=["gemm", "linear", "transcode", "quantize", "quantize_b"],
                    default=None,
                    help="time one kernel shape instead of the benchmark step")
    ap.add_argument("--M", type=int, default=16)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--split", type=int, default=0)
    ap.add_argument("--overlap", type=int, default=1,
                    help="--case gemm: launch with programmatic serialisation (weights static)")
    ap.add_argument("--nblk", type=int, default=1 << 26)
    ap.add_argument("--xdtype", choices=["bf16", "f32"], default="bf16",
                    help="input dtype of --case quantize / quantize_b")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch every GEMM only after the previous kernel completed")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        return run_case(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group(
            "nccl", timeout=datetime.timedelta(seconds=120),
            device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            return run_reference(args, rank, world)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
