#!/usr/bin/env python3
"""Benchmark of the W4A6 GEMM (MXFP6 activations x NVFP4 weights transcoded on chip).

Headline workload (the decode sweep): N=14336, K=4096, M in {1,4,16,32,64}.
One step = for each M, one GEMM against each of L=8 distinct weight matrices (a decode pass
over 8 layers), i.e. 40 GEMMs reading 8 x 33.0 MB of NVFP4 weights per M. The 8 matrices
(264 MB) exceed the 126 MB L2, so every GEMM streams its weights from HBM. Weights: Student-t
(df 5) scaled to std 0.02, NVFP4-quantised on the GPU; activations: N(0,1) with 0.1% of the K
channels times 20, MXFP6-quantised on the GPU (seeds in the line's `data`).

Metric: decode weight GB/s = weight bytes (N*K/2 codes + N*K/16 E4M3 scales + 4) per GEMM,
summed over the step, divided by the step time. Multi-GPU (torchrun): every rank holds its own
14336-row N-shard of a (14336*world) x 4096 weight matrix per layer and runs the same sweep
with no collective in the timed region (weak scaling); the time is the max over ranks.

Also in the line:
* `configs`: BASELINE configs 1, 3 and 4 on one GPU (time, TFLOP/s, weight GB/s, roofline
  against the measured tensor peak of the MMA probe or the measured HBM copy rate);
* `sharded_70b` (every N): config 4 (N=28672, K=8192, M in {16, 4096}) column-sharded across
  the ranks (strong scaling): the sharded GEMM's time (max over ranks), the one-GPU time of the
  whole matrix on rank 0, efficiency t1 / (N t_N), the NCCL all-gather of C timed on its own,
  and a bit-for-bit check of the gathered C against per-shard GEMMs on rank 0;
* `cpu_baseline`: the reference's CPU path (the oracle port of its codec + dequantise + fp32
  matmul) on the host cores, transcode and GEMM timed separately.

--impl reference times that CPU path instead (rank 0 only).

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
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
SEED_W, SEED_A = 2, 3            # decode sweep: weights layer l use SEED_W * 100 + l
N70, K70 = 28672, 8192
L2_BYTES = 126 * 2 ** 20


def weight_bytes(N, K):
    return N * K // 2 + N * K // 16 + 4


def alg_bytes(M, N, K):
    """Algorithmic bytes of one GEMM: weights + A (one code byte + 1/32 scale byte per
    element) + C (bf16)."""
    return weight_bytes(N, K) + M * K + M * K // 32 + 2 * M * N


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
    """Samples SM clock, power and clock-event reasons via NVML (read only) while the timed
    regions run (started before the first, stopped after the last)."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80, "gpu_idle": 0x1,
        "applications_clocks_setting": 0x2,
    }

    def __init__(self, index, period=0.002):
        super().__init__(daemon=True)
        self.index, self.period = index, period
        self.samples = []
        self.stop_evt = threading.Event()
        self.active = threading.Event()
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
            if self.active.is_set():
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

def _orc():
    import ctypes
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
    return lib


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        if info:
            return {"library": info[0].get("internal_api"), "version": info[0].get("version"),
                    "threads": info[0].get("num_threads")}
    except Exception:
        pass
    return None


def all_blas_threads(cores):
    """OpenBLAS limited to `cores` threads for the duration of a with block (torchrun sets
    OMP_NUM_THREADS=1 for its workers; the CPU path gets every host core)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=cores, user_api="blas")
    except Exception:  # noqa: BLE001 - no threadpoolctl: the library default applies
        import contextlib
        return contextlib.nullcontext()


def cpu_reference_run(seconds=10.0, rows=N_W):
    """The decode sweep on the CPU: per GEMM, the NVFP4 -> MXFP6 transcode of the whole
    `rows` x 4096 weight matrix (C restatement, all host threads), then the GEMM: dequantisation
    and an fp32 matmul (OpenBLAS, all host threads) with M tokens; the two parts are timed
    separately, whole sweeps (M = 1, 4, 16, 32, 64) until `seconds` have passed. Returns a dict
    with the weight GB/s of the whole path and of each part, the seconds per GEMM of each part,
    the thread counts and the sample description."""
    import numpy as np
    lib = _orc()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(SEED_W)
    K = K_W
    packed = rng.integers(0, 256, (rows, K // 2), dtype=np.uint8)
    scales = rng.integers(0x28, 0x50, (rows, K // 16), dtype=np.uint8)
    nblk = rows * K // 32
    e6 = np.empty(nblk * 32, np.uint8)
    e8 = np.empty(nblk, np.uint8)
    Bf = np.empty((rows, K), np.float32)
    acts = {M: rng.standard_normal((M, K)).astype(np.float32) for M in M_SWEEP}
    done = 0
    t_tx = t_mm = 0.0
    with all_blas_threads(cores):
        blas = blas_threads()
        t0 = time.perf_counter()
        while True:
            for M in M_SWEEP:
                a = time.perf_counter()
                lib.orc_transcode(packed.ctypes.data, scales.ctypes.data, nblk, 16,
                                  e6.ctypes.data, e8.ctypes.data, cores)
                b = time.perf_counter()
                lib.orc_dequant(e6.ctypes.data, e8.ctypes.data, nblk, Bf.ctypes.data, cores)
                _ = acts[M] @ Bf.T
                c = time.perf_counter()
                t_tx += b - a
                t_mm += c - b
                done += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
    wb = weight_bytes(rows, K)
    return {
        "value": done * wb / (t_tx + t_mm) / 1e9,
        "transcode_gbs": done * wb / t_tx / 1e9,
        "gemm_gbs": done * wb / t_mm / 1e9,
        "transcode_s_per_gemm": t_tx / done,
        "gemm_s_per_gemm": t_mm / done,
        "cores": cores,
        "blas": blas,
        "sample": (f"{done // len(M_SWEEP)} decode sweeps ({done} GEMMs) on the whole {rows}x{K} "
                   f"weight matrix (transcode {t_tx:.1f} s + dequant and fp32 matmul "
                   f"{t_mm:.1f} s), {el:.1f} s"),
    }


def cpu_config_rates(seconds=4.0):
    """Throughputs of the CPU path's two parts on representative shapes, for the per-config
    table: transcode (weight bytes/s, C restatement, all threads) and dequant + fp32 matmul
    (GEMM flop/s at M=128, K=4096, OpenBLAS). Per-config CPU seconds are these rates applied
    to each config's bytes and flops (extrapolated; the full prefill matmul would take minutes)."""
    import numpy as np
    lib = _orc()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(9)
    rows, K, M = 1024, 4096, 128
    packed = rng.integers(0, 256, (rows, K // 2), dtype=np.uint8)
    scales = rng.integers(0x28, 0x50, (rows, K // 16), dtype=np.uint8)
    nblk = rows * K // 32
    e6 = np.empty(nblk * 32, np.uint8)
    e8 = np.empty(nblk, np.uint8)
    Bf = np.empty((rows, K), np.float32)
    A = rng.standard_normal((M, K)).astype(np.float32)
    t_tx = t_mm = 0.0
    n = 0
    limits = all_blas_threads(cores)
    limits.__enter__()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        a = time.perf_counter()
        lib.orc_transcode(packed.ctypes.data, scales.ctypes.data, nblk, 16, e6.ctypes.data,
                          e8.ctypes.data, cores)
        b = time.perf_counter()
        lib.orc_dequant(e6.ctypes.data, e8.ctypes.data, nblk, Bf.ctypes.data, cores)
        _ = A @ Bf.T
        c = time.perf_counter()
        t_tx += b - a
        t_mm += c - b
        n += 1
    limits.__exit__(None, None, None)
    return {"transcode_bytes_per_s": n * weight_bytes(rows, K) / t_tx,
            "gemm_flops_per_s": n * 2.0 * M * rows * K / t_mm,
            "dequant_matmul_shape": f"M={M} x {rows}x{K}", "iterations": n}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    t_run = time.perf_counter()
    vals = []
    last = None
    for _ in range(max(1, args.warmup)):
        cpu_reference_run(seconds=0.5)
    for _ in range(args.steps):
        last = cpu_reference_run(seconds=max(0.25, args.cpu_seconds / max(1, args.steps)))
        vals.append(last["value"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes -> fp32", "data": "synthetic",
        "config": {"workload": f"decode sweep N={N_W} K={K_W} M in {list(M_SWEEP)}",
                   "path": "CPU oracle port of the reference codec + numpy fp32 matmul"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": last["cores"], "kind": "port",
                         "sample": last["sample"], "blas": last["blas"],
                         "transcode_gbs": last["transcode_gbs"], "gemm_gbs": last["gemm_gbs"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t_run,
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------------
# GPU leg: synthetic operands with the BASELINE configs' distributions

def gen_student_t(torch, shape, std, g):
    """Student-t (df 5) scaled to standard deviation `std`: z / sqrt(chi2_5 / 5)."""
    z = torch.randn(shape, device=g.device, generator=g)
    chi = torch.zeros(shape, device=g.device)
    for _ in range(5):
        chi += torch.randn(shape, device=g.device, generator=g).square()
    return z / torch.sqrt(chi / 5.0) * (std / math.sqrt(5.0 / 3.0))


def gen_outlier_acts(torch, shape, g):
    """N(0,1) with 0.1% of the K channels multiplied by 20."""
    x = torch.randn(shape, device=g.device, generator=g)
    ch = torch.rand(shape[-1], device=g.device, generator=g) < 0.001
    return torch.where(ch[None, :], x * 20.0, x)


def generator(torch, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g


def graph_of(torch, body, stream):
    """CUDA graph of one call of `body` (warmed outside the graph first). Everything enqueued
    before (on any stream) completes first: the operands were made on the default stream, and
    buffers freed there may be reused by tensors the side stream writes."""
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        body()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            body()
    return graph


def time_graph(torch, graph, stream, iters, warmup=3):
    """Mean ms per replay, CUDA events on the launching stream, synchronised on both sides."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(iters):
            graph.replay()
        t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / iters


def rotating_copies(bytes_each, min_total=3 * L2_BYTES):
    """How many distinct copies of an operand make the rotating working set exceed L2."""
    return max(2, -(-min_total // max(1, bytes_each)))


def clone_weights(ops, w):
    return ops.PackedWeights(w.codes.clone(), w.scales.clone(), w.tensor_scale, w.N, w.K,
                             w.sideband)


def gemm_roofline(M, N, K, ms, tensor_peak, tensor_kind, hbm_peak, hbm_kind):
    """One GEMM's figures and its roofline: the bound is the one whose time is longer at the
    peaks (flops / tensor peak vs algorithmic bytes / HBM copy rate)."""
    flops = 2.0 * M * N * K
    ab = alg_bytes(M, N, K)
    tflops = flops / (ms / 1e3) / 1e12
    gbs = ab / (ms / 1e3) / 1e9
    tensor_bound = flops / (tensor_peak * 1e12) >= ab / (hbm_peak * 1e9)
    roof = ({"bound": "tensor", "achieved": tflops, "peak": tensor_peak, "unit": "TFLOP/s",
             "frac": tflops / tensor_peak, "peak_kind": tensor_kind} if tensor_bound else
            {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
             "frac": gbs / hbm_peak, "peak_kind": hbm_kind})
    return {"M": M, "N": N, "K": K, "ms": ms, "us": ms * 1e3, "tflops": tflops,
            "weight_gbs": weight_bytes(N, K) / (ms / 1e3) / 1e9, "alg_gbs": gbs,
            "frac_of_tensor_peak": tflops / tensor_peak, "frac_of_hbm": gbs / hbm_peak,
            "roofline": roof}


def time_gemm_config(torch, ops, dev, M, N, K, w_kind, w_std, a_kind, seed, stream,
                     launches=None):
    """One BASELINE config on one GPU: weights quantised on the GPU from the config's
    distribution, rotated over enough copies that the working set exceeds L2, the GEMMs of one
    pass captured in a CUDA graph (back to back, programmatic serialisation with static
    weights), replayed for about 20 ms per timing; the median of three timings. Returns ms per
    GEMM."""
    g = generator(torch, dev, seed)
    w = (gen_student_t(torch, (N, K), w_std, g) if w_kind == "t"
         else torch.randn((N, K), device=dev, generator=g) * w_std)
    pw = ops.quantize_weights(w)
    del w
    x = gen_outlier_acts(torch, (M, K), g) if a_kind == "outlier" else \
        torch.randn((M, K), device=dev, generator=g)
    acts = ops.quantize_activations(x)
    del x
    reps = rotating_copies(weight_bytes(N, K))
    ws = [pw] + [clone_weights(ops, pw) for _ in range(reps - 1)]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    wsp = ops.Workspace()
    n = launches or max(reps, 8)

    def body():
        for i in range(n):
            ops.w4a6_gemm(acts, ws[i % reps], out=out, workspace=wsp, stream=stream,
                          overlap_prev=True, weights_static=True)
    graph = graph_of(torch, body, stream)
    per_replay = time_graph(torch, graph, stream, iters=1)
    iters = max(3, int(20.0 / max(per_replay, 1e-3)))
    ms = sorted(time_graph(torch, graph, stream, iters=iters, warmup=1) for _ in range(3))[1] / n
    del graph
    return ms


def sharded_70b(torch, ops, dev, rank, world, stream, steps):
    """Config 4 column-sharded across the ranks (strong scaling) -- see the module doc."""
    import torch.distributed as dist
    from bitdance_b200 import shard
    res = {"N": N70, "K": K70, "world": world, "shard_rows": N70 // world}
    # every rank draws the whole matrix from the same seed, so the tensor scale is global, and
    # quantises it on its own GPU; it keeps only its shard (rank 0 also keeps all, for the check)
    g = generator(torch, dev, 4000)
    w = torch.randn((N70, K70), device=dev, generator=g) * 0.015
    codes, sc, tstat = ops.quantize_nvfp4(w)
    del w
    s_t = ops.tensor_scale_of(tstat)
    lo, hi = shard.shard_rows(N70, world, rank)
    mine = ops.pack_weights(codes[lo:hi].contiguous(), sc[lo:hi].contiguous(), s_t)
    full = ops.pack_weights(codes, sc, s_t) if rank == 0 else None
    per = {}
    for M in (16, 4096):
        ga = generator(torch, dev, 4100 + M)
        acts = ops.quantize_activations(torch.randn((M, K70), device=dev, generator=ga))
        n = hi - lo
        reps = rotating_copies(weight_bytes(n, K70))
        ws = [mine] + [clone_weights(ops, mine) for _ in range(reps - 1)]
        out = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
        wsp = ops.Workspace()
        launches = max(reps, 8)

        def body():
            for i in range(launches):
                ops.w4a6_gemm(acts, ws[i % reps], out=out, workspace=wsp, stream=stream,
                              overlap_prev=True, weights_static=True)
        graph = graph_of(torch, body, stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = time_graph(torch, graph, stream, iters=max(3, steps // 20)) / launches
        del graph, ws
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        entry = {"t_N_ms": ms, "weight_gbs_total": weight_bytes(N70, K70) / (ms / 1e3) / 1e9,
                 "tflops_total": 2.0 * M * N70 * K70 / (ms / 1e3) / 1e12}
        # the whole matrix on one GPU (rank 0), same method
        if rank == 0:
            entry["t_1_ms"] = time_gemm_full(torch, ops, acts, full, stream)
            entry["efficiency"] = entry["t_1_ms"] / (world * ms)
        if world > 1:
            dist.barrier()
            # all-gather of the bf16 shards over NCCL, timed on its own (not in t_N)
            C = ops.w4a6_gemm(acts, mine, stream=torch.cuda.current_stream())
            buf = torch.empty((world * M, n), dtype=C.dtype, device=dev)
            for _ in range(3):
                dist.all_gather_into_tensor(buf, C)
            torch.cuda.synchronize()
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            it = 10
            e0.record()
            for _ in range(it):
                dist.all_gather_into_tensor(buf, C)
            e1.record()
            torch.cuda.synchronize()
            ag = e0.elapsed_time(e1) / it
            t = torch.tensor([ag], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ag = float(t.item())
            recv = (world - 1) * M * n * 2
            entry["allgather_ms"] = ag
            entry["allgather_gbs_per_gpu"] = recv / (ag / 1e3) / 1e9
            gathered = shard.assemble(buf.view(world, M, n))
            if rank == 0:
                # bit for bit against the per-shard GEMMs of rank 0 (same schedule per shard)
                ref = torch.cat([ops.w4a6_gemm(acts, ops.pack_weights(
                    codes[r * n:(r + 1) * n].contiguous(), sc[r * n:(r + 1) * n].contiguous(),
                    s_t)) for r in range(world)], dim=1)
                entry["gather_bit_exact"] = bool(torch.equal(gathered, ref))
            dist.barrier()
        per[f"M{M}"] = entry
    res["per_M"] = per
    return res


def time_gemm_full(torch, ops, acts, full, stream):
    reps = rotating_copies(weight_bytes(full.N, full.K))
    ws = [full] + [clone_weights(ops, full) for _ in range(reps - 1)]
    out = torch.empty((acts.M, full.N), dtype=torch.bfloat16, device=acts.codes.device)
    wsp = ops.Workspace()
    launches = max(reps, 8)

    def body():
        for i in range(launches):
            ops.w4a6_gemm(acts, ws[i % reps], out=out, workspace=wsp, stream=stream,
                          overlap_prev=True, weights_static=True)
    graph = graph_of(torch, body, stream)
    ms = time_graph(torch, graph, stream, iters=3) / launches
    del graph, ws
    return ms


def run_ours(args, rank, world, local_rank):
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    bd.load()
    peaks, peak_kind = load_peaks()

    # weights: L layers of this rank's N-shard, Student-t, NVFP4-quantised on the GPU
    weights = []
    for layer in range(LAYERS):
        g = generator(torch, dev, SEED_W * 100 + layer + 1000 * rank)
        w = gen_student_t(torch, (N_W, K_W), 0.02, g)
        weights.append(ops.quantize_weights(w))
        del w
    # activations per M: outlier channels, MXFP6-quantised on the GPU (natural codes + scales)
    nat = {}
    for M in M_SWEEP:
        g = generator(torch, dev, SEED_A * 100 + M)
        nat[M] = ops.quantize_mxfp6(gen_outlier_acts(torch, (M, K_W), g))
    acts = {M: ops.pack_activations(*nat[M]) for M in M_SWEEP}
    outs = {M: torch.empty((M, N_W), dtype=torch.bfloat16, device=dev) for M in M_SWEEP}
    wss = {M: ops.Workspace() for M in M_SWEEP}
    launches_per_step = len(M_SWEEP) * LAYERS

    # no-output guard (kernel/bench_sweep.py:297-326): a launch must write C
    for M in M_SWEEP:
        outs[M].zero_()
        ops.w4a6_gemm(acts[M], weights[0], out=outs[M], workspace=wss[M])
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
                ops.w4a6_gemm(acts[M], w, out=outs[M], workspace=wss[M],
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
                ops.w4a6_gemm(e2e_acts[M], w, out=outs[M], workspace=wss[M], stream=cur,
                              overlap_prev=ov, weights_static=ov)
            done = torch.cuda.Event()
            done.record(cur)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                h_out[M].copy_(outs[M], non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    g_k = graph_of(torch, step_kernels, stream)
    g_e = graph_of(torch, step_e2e, stream)

    clocks = ClockSampler(local_rank)
    clocks.start()

    def timed(graph, steps, warmup):
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        clocks.active.set()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")  # launch lists filter on it (ncu --nvtx-include)
        with torch.cuda.stream(stream):
            t0.record(stream)
            for _ in range(steps):
                graph.replay()
            t1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clocks.active.clear()
        if world > 1:
            torch.distributed.barrier()
        ms = t0.elapsed_time(t1)
        if world > 1:
            tt = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    ms_k = timed(g_k, args.steps, args.warmup)
    steps_e = max(3, args.steps // 2)
    ms_e = timed(g_e, steps_e, args.warmup)
    # the host copies hold each batch's last-layer output: it must equal a fresh device GEMM
    for M in M_SWEEP:
        ref = ops.w4a6_gemm(acts[M], weights[-1]).cpu()
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
                ops.w4a6_gemm(acts[M], w, out=outs[M], workspace=wss[M],
                              stream=stream, overlap_prev=ov, weights_static=ov)
    g_d = graph_of(torch, step_dom, stream)
    ms_d = timed(g_d, args.steps, args.warmup)
    n_dom = len(dom_M) * LAYERS
    alg_per_launch = sum(alg_bytes(M, N_W, K_W) for M in dom_M) / len(dom_M)
    us_per_launch = ms_d * 1e3 / (args.steps * n_dom)
    achieved = alg_per_launch / (us_per_launch * 1e-6) / 1e9
    tpw = load_traffic()
    # per-M GEMM time of the sweep (one graph per M, the same launches as the step)
    per_m = {}
    for M in M_SWEEP:
        def step_m(M=M):
            for w in weights:
                ops.w4a6_gemm(acts[M], w, out=outs[M], workspace=wss[M],
                              stream=stream, overlap_prev=ov, weights_static=ov)
        gm = graph_of(torch, step_m, stream)
        clocks.active.set()
        us = time_graph(torch, gm, stream, iters=max(3, args.steps // 4)) * 1e3 / LAYERS
        clocks.active.clear()
        per_m[str(M)] = {"us": us, "weight_gbs": weight_bytes(N_W, K_W) / us / 1e3,
                         "frac_of_hbm": weight_bytes(N_W, K_W) / us / 1e3 / peaks["hbm_gbs"]}
        del gm
    del g_d, g_k, g_e

    def no_device_error(stage):
        w = bd.device_error()
        if w != 0:
            raise RuntimeError(f"kernel error word 0x{w:x} set after {stage}")

    no_device_error("the decode sweep")
    # tensor peak of the block-scaled MMA, measured now (SS and TS operand forms, and the
    # CTA-pair MMA of the large GEMMs' tiles); the roofline takes the fastest
    probe = None
    tensor_peak, tensor_kind = 2.0 * peaks["bf16_tflops"], "2x measured cuBLAS bf16 burst"
    if not args.no_configs:
        try:
            ss = ops.mma_peak_tflops(n_cols=256, a_from_tmem=False)
            ts = ops.mma_peak_tflops(n_cols=256, a_from_tmem=True)
            pair = ops.mma_peak_tflops(pair=True)
            probe = {"ss_tflops": ss, "ts_tflops": ts, "pair_tflops": pair,
                     "what": "tcgen05.mma.kind::mxf8f6f4.block_scale N=256 K=32 back to back, "
                             "pseudo-random operands: cta_group::1 M=128 one CTA per SM (A in "
                             "shared or tensor memory), cta_group::2 M=256 one cluster per two "
                             "SMs (bd_probe_mma_peak)"}
            tensor_peak, tensor_kind = max(ss, ts, pair), "measured by the MMA probe (this run)"
        except Exception as e:  # noqa: BLE001 - report, keep the fallback
            probe = {"error": repr(e)}

    extra = {}
    if world == 1 and not args.no_configs:
        cfgs = {}
        clocks.active.set()
        cases = {
            "1": (128, 4096, 4096, "normal", 0.02, "normal", 10),
            "3_gate_up": (8192, 14336, 4096, "t", 0.02, "outlier", 30),
            "3_down": (8192, 4096, 14336, "t", 0.02, "outlier", 31),
            "4_M16": (16, N70, K70, "normal", 0.015, "normal", 40),
            "4_M4096": (4096, N70, K70, "normal", 0.015, "normal", 41),
        }
        times = {}
        for name, (M, N, K, wk, ws_, ak, seed) in cases.items():
            times[name] = time_gemm_config(torch, ops, dev, M, N, K, wk, ws_, ak, seed, stream)
            no_device_error(f"config {name}")
        clocks.active.clear()
        # the configs are timed over ~20 ms replays each, long enough for the 1 kW power cap to
        # pull the clock down: their tensor roofline takes the pair MMA sustained the same way,
        # measured right after them (launches of ~17 ms back to back, the last one timed)
        if probe is not None and "pair_tflops" in probe:
            sustained = None
            for _ in range(3):
                sustained = ops.mma_peak_tflops(pair=True, mmas_per_cta=1 << 18, reps=1)
            probe["pair_sustained_tflops"] = sustained
            probe["sustained_what"] = ("the pair MMA in launches of 2^18 MMAs per CTA (~17 ms "
                                       "at 1965 MHz), six back to back after the configs, the "
                                       "last one timed")
            tensor_peak = sustained
            tensor_kind = ("measured by the pair-MMA probe sustained over ~100 ms right after "
                           "the configs (this run; the burst figures are in tensor_peak_probe)")
        for name, (M, N, K, wk, ws_, ak, seed) in cases.items():
            cfgs[name] = gemm_roofline(M, N, K, times[name], tensor_peak, tensor_kind,
                                       peaks["hbm_gbs"], peak_kind)
        extra["configs"] = cfgs
    if not args.no_sharded:
        clocks.active.set()
        extra["sharded_70b"] = sharded_70b(torch, ops, dev, rank, world, stream, args.steps)
        clocks.active.clear()
        no_device_error("the sharded config-4 GEMMs")
    clk = clocks.summary()

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_k / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp6 x mxfp6 (fp32 accumulate, bf16 out)",
        "data": (f"synthetic: weights Student-t(df 5) std 0.02 -> NVFP4 on the GPU (torch "
                 f"generator seeds {SEED_W * 100}+layer), activations N(0,1) with 0.1% of "
                 f"channels x20 -> MXFP6 on the GPU (seeds {SEED_A * 100}+M)"),
        "config": {"workload": f"decode sweep N={N_W} K={K_W} M in {list(M_SWEEP)} x {LAYERS} layers",
                   "per_rank_N": N_W, "global_N": N_W * world, "K": K_W,
                   "schedule": "persistent stream-K (tiles split across CTAs finished in-kernel)",
                   "l2": f"{LAYERS} weight matrices per rank ({LAYERS * weight_bytes(N_W, K_W) / 1e6:.0f} MB) "
                         "rotate, larger than the 126 MB L2",
                   "parallelism": f"N-sharded x{world}, no collective in the timed region",
                   "launch": "CUDA graph of one step" + (
                       ", programmatic serialisation between GEMMs" if ov else "")},
        "tflops": flops_step * args.steps / (ms_k / 1e3) / 1e12 * world,
        "per_M": per_m,
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
        "tensor_peak_probe": probe,
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "pinned host A -> device, bd_pack_a, bd_w4a6_gemm x layers, C -> pinned host"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
        **extra,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_run(seconds=args.cpu_seconds)
        line["cpu_baseline"] = {"value": cpu["value"], "unit": UNIT, "cores": cpu["cores"],
                                "kind": "port", "sample": cpu["sample"], "blas": cpu["blas"],
                                "transcode_gbs": cpu["transcode_gbs"], "gemm_gbs": cpu["gemm_gbs"],
                                "transcode_s_per_gemm": cpu["transcode_s_per_gemm"],
                                "gemm_s_per_gemm": cpu["gemm_s_per_gemm"]}
        if "configs" in line:
            rates = cpu_config_rates()
            line["cpu_baseline"]["config_rates"] = rates
            for c in line["configs"].values():
                c["cpu_transcode_s"] = weight_bytes(c["N"], c["K"]) / rates["transcode_bytes_per_s"]
                c["cpu_gemm_s"] = 2.0 * c["M"] * c["N"] * c["K"] / rates["gemm_flops_per_s"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_case(args):
    """One kernel shape, repeated: `--case gemm` (a single W4A6 GEMM), `--case transcode`
    (the standalone NVFP4 -> MXFP6 transcode of config 5), `--case quantize` (the MXFP6
    activation quantiser), `--case quantize_b` (the NVFP4 weight quantiser; bytes count the
    two passes over the weights) or `--case probe` (the tensor-core MMA probe). Prints its own
    JSON line; used for Nsight Compute captures of one launch."""
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if args.case == "probe":
        res = {"case": "probe"}
        for n in (16, 32, 64, 128, 256):
            for tm in (False, True):
                res[f"N{n}_{'ts' if tm else 'ss'}_tflops"] = ops.mma_peak_tflops(
                    n_cols=n, a_from_tmem=tm, mmas_per_cta=args.steps * 64)
        res["N256_pair_tflops"] = ops.mma_peak_tflops(pair=True, mmas_per_cta=args.steps * 64)
        print(json.dumps(res), flush=True)
        return 0
    if args.case == "gemm":
        # weight matrices rotate so the working set exceeds the 126 MB L2; the calls are
        # captured in one CUDA graph so the time is device time, not host launch overhead
        M, N, K = args.M, args.N, args.K
        reps = max(2, -(-300_000_000 // weight_bytes(N, K)))
        if args.dist == "t":
            base = ops.quantize_weights(gen_student_t(torch, (N, K), 0.02, g))
            ws_list = [base] + [clone_weights(ops, base) for _ in range(reps - 1)]
            a = ops.quantize_activations(gen_outlier_acts(torch, (M, K), g))
        else:
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
                "dist": args.dist, "weight_bytes": weight_bytes(N, K), "flops": 2 * M * N * K}
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
    graphed = args.case in ("gemm", "linear", "quantize", "quantize_b")
    with torch.cuda.stream(stream):
        for _ in range(3 if graphed else max(3, args.warmup)):
            fn()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    reps_t = 3 if graphed else args.steps
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
    ap.add_argument("--case", choices=["gemm", "linear", "transcode", "quantize", "quantize_b",
                                       "probe"],
                    default=None,
                    help="time one kernel shape instead of the benchmark step")
    ap.add_argument("--M", type=int, default=16)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--split", type=int, default=0)
    ap.add_argument("--dist", choices=["bytes", "t"], default="bytes",
                    help="--case gemm operands: uniform random bytes, or config-2 distributions "
                         "(Student-t weights, outlier activations) quantised on the GPU")
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
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config figures (configs 1, 3, 4) and the MMA probe")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the config-4 sharded (strong scaling) figures")
    ap.add_argument("--no-prefill", action="store_true", help="alias of --no-configs")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch every GEMM only after the previous kernel completed")
    args = ap.parse_args()
    if args.no_prefill:
        args.no_configs = True
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
