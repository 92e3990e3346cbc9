"""Benchmark of the DS hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemm|fused_add_mul|reduce|recurrence|
                                gemm_large|batched_dot]

Default workload (the headline metric): DS dot_general C = A @ B with
M = N = K = 4096, A and B float64 ~ U[-1, 1] drawn from default_rng(2) (A
first), split to (hi, lo), multiplied in DS arithmetic and recombined to f64.
One step = one ds_dot_general_f64 call on device-resident inputs.  Inputs
(2 x 128 MiB) and output (128 MiB) exceed the 126 MB L2.  value = whole-job
DS-GEMM GFLOP/s (2*M*N*K per GEMM); with N GPUs every rank multiplies its
own 4096-row block of A by the replicated B (weak scaling, no collective in
the step).  e2e repeats the step through the public API with pinned host
buffers: A and B copied in and C copied out every step.

--impl reference times the reference's CPU path for the same workload on the
host cores (rank 0 only): the DS pass restated in NumPy (split, four float32
matmuls with f32 accumulation, two_sum, recombine; oracle/ds_pass_ref.py).
The reference itself needs JAX/XLA, which this image does not have.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ds-experiment_b200"))
sys.path.insert(0, ROOT)

METRIC = "DS-GEMM GFLOP/s at 4096³ (1–8 B200); DS elementwise HBM GB/s; err vs f64"
GEMM_DIM = 4096


# ---------------------------------------------------------------------------
# helpers

def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class all_host_threads:
    """BLAS on every host core for the CPU arms (torchrun sets
    OMP_NUM_THREADS=1 in every rank, which would leave numpy's BLAS on one
    thread); `.threads` is the count the BLAS libraries report inside."""

    def __enter__(self):
        try:
            from threadpoolctl import threadpool_info, threadpool_limits
        except ImportError:
            self._ctl, self.threads = None, host_cores()
            return self
        self._ctl = threadpool_limits(limits=host_cores(), user_api="blas")
        self._ctl.__enter__()
        counts = [i["num_threads"] for i in threadpool_info() if i["user_api"] == "blas"]
        self.threads = max(counts) if counts else host_cores()
        return self

    def __exit__(self, *exc):
        if self._ctl is not None:
            self._ctl.__exit__(*exc)
        return False


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(kernel_family, workload):
    """Per-launch DRAM bytes of a kernel family from profiles/ncu_traffic.txt
    (lines: family workload bytes_per_launch), or None."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == kernel_family \
                and parts[1] == workload:
            return float(parts[2])
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        """Start sampling and return once the first sample is in, so that
        nvidia-smi's start-up (NVML initialisation) lands before the timed
        region instead of inside it."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        import select
        ready, _, _ = select.select([self.proc.stdout], [], [], 10.0)
        self.first = self.proc.stdout.readline() if ready else ""

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        # the first sample was taken before the timed region: not counted
        rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        if not sm:
            return None
        mx = max(float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) < 9:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# workloads

def gemm_config(world, algo):
    """The headline workload's config: the same dict in both arms."""
    return {"workload": "ds_dot_general_f64 4096x4096x4096 (A, B f64 U[-1,1] seed 2; "
                        "per-rank 4096-row A block, B replicated)",
            "M": GEMM_DIM * world, "N": GEMM_DIM, "K": GEMM_DIM,
            "algorithm": algo, "parallelism": f"rows{world}",
            "l2": "inputs 256 MiB + output 128 MiB per step exceed the 126 MB L2"}


def gemm_inputs(rank):
    """Rank 0: exactly the 4096^3 config (default_rng(2), A then B).  Rank r > 0
    multiplies its own A block (default_rng((2, r))) by the same B."""
    rng = np.random.default_rng(2)
    A = rng.uniform(-1, 1, (GEMM_DIM, GEMM_DIM))
    B = rng.uniform(-1, 1, (GEMM_DIM, GEMM_DIM))
    if rank > 0:
        A = np.random.default_rng((2, rank)).uniform(-1, 1, (GEMM_DIM, GEMM_DIM))
    return A, B


def gemm_error(C, A, B, samples=256):
    from oracle import exact
    rows, cols = exact.sample_indices(A.shape[0], B.shape[1], samples, seed=77)
    truth = exact.exact_gemm_entries(A, B, rows, cols)
    err = np.abs(C[rows, cols] - truth)
    return float(err.max()), float(np.median(err)), rows, cols, truth


def reference_gemm_error(A, B, rows, cols, truth):
    """Error of the reference DS path (4 x f32 dots, DsTransformPass.cpp:359-365)
    on the sampled entries."""
    from oracle import ds_pass_ref
    ah, al = ds_pass_ref.from_float(A[rows])
    # only the sampled rows and columns are needed
    uniq_c, inv_c = np.unique(cols, return_inverse=True)
    bh, bl = ds_pass_ref.from_float(B[:, uniq_c])
    p = np.einsum("ik,ki->i", ah, bh[:, inv_c])
    e1 = np.einsum("ik,ki->i", ah, bl[:, inv_c])
    e2 = np.einsum("ik,ki->i", al, bh[:, inv_c])
    e3 = np.einsum("ik,ki->i", al, bl[:, inv_c])
    h, l = ds_pass_ref.two_sum(p, (e1 + e2) + e3)
    ref = ds_pass_ref.to_float(h, l)
    return float(np.abs(ref - truth).max())


# ---------------------------------------------------------------------------

def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)
    from ds_b200 import _lib, ops

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream()
    result = {}
    if args.workload != "gemm":
        raise SystemExit("only --workload gemm is the driver's contract; see --help")

    A, B = gemm_inputs(rank)
    dA = torch.from_numpy(A).to(dev)
    dB = torch.from_numpy(B).to(dev)
    algo = args.algorithm

    def step():
        return ops.ds_matmul_f64(dA, dB, algorithm=algo)

    for _ in range(args.warmup):
        C = step()
    torch.cuda.synchronize()
    C_host = C.cpu().numpy() if rank == 0 else None

    clocks = ClockSampler(local)
    # inside the timed region only the dominant kernel is bracketed with
    # events (two per step); the other families' times come from a second,
    # separately profiled pass below (a --kernels-only run brackets them all
    # in the timed steps and has no second pass)
    fam = "ozaki_gemm"
    _lib.profile_reset()
    _lib.profile_select(None if args.kernels_only else [fam])
    _lib.profile_enable(True)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        C = step()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    _lib.profile_enable(False)
    ms = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms)
    flops_step = 2.0 * GEMM_DIM ** 3
    value = world * flops_step / (ms * 1e-3) / 1e9

    # dominant kernel and its roofline (timed region)
    k_ms, k_n = _lib.profile_read(fam)
    if not args.kernels_only:
        # every family, from the same number of steps run again with all
        # brackets
        _lib.profile_reset()
        _lib.profile_select(None)
        _lib.profile_enable(True)
        for _ in range(args.steps):
            C = step()
        torch.cuda.synchronize()
        _lib.profile_enable(False)
    _lib.profile_select(None)
    launches = {}
    for f in ("ozaki_split", "ozaki_split_rows", "ozaki_colmax", "ozaki_split_rows_colmax",
              "ozaki_split_cols", "ozaki_gemm", "ozaki_crt", "ozaki_fix",
              "dot_simt", "dot_vec", "elementwise",
              "reduce", "recurrence"):
        t, n = _lib.profile_read(f)
        if n:
            launches[f] = {"launches": n, "ms_total": round(t, 4)}
    peaks, peak_src = measured_peaks()
    if k_n:
        # the product's int8 GEMMs may run as several launches (bands of A's
        # rows): achieved = the step's tensor ops over the GEMM device time
        # per step
        info = _lib.gemm_info(GEMM_DIM, GEMM_DIM, GEMM_DIM)
        per_step_ms = k_ms / args.steps
        achieved = info["tensor_ops_per_launch"] / (per_step_ms * 1e-3) / 1e12
        peak = 2.0 * peaks["bf16_tflops"]
        roofline = {"bound": "tensor", "kernel": fam, "achieved": round(achieved, 1),
                    "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                    "traffic": ncu_traffic(fam, "gemm4096"),
                    "peak_source": f"2 x {peak_src} bf16_tflops (B200 dense int8 rate = "
                                   "2x bf16); int8 ops counted as 2 per MAC",
                    "kernel_ms_per_step": round(per_step_ms, 4),
                    "launches_per_step": round(k_n / args.steps, 2),
                    # the measured bf16 proxy sits below the int8 pipe's own
                    # rate; the nominal dense int8 rate is 4.5 POPS
                    "frac_of_nominal_int8": round(achieved / 4500.0, 4)}
    else:
        fam = "dot_simt"
        k_ms, k_n = _lib.profile_read(fam)
        per_launch_ms = k_ms / max(k_n, 1)
        roofline = {"bound": "tensor", "kernel": fam, "achieved": None, "peak": None,
                    "unit": "TFLOP/s", "frac": None, "traffic": None,
                    "note": "CUDA-core path (tensor-core kernel unavailable)",
                    "kernel_ms_per_launch": round(per_launch_ms, 4)}
    # "ozaki_split" brackets the split kernels (it is not a kernel itself)
    gpu_launches = sum(v["launches"] for f, v in launches.items() if f != "ozaki_split")
    if args.kernels_only:
        # Profiling case: the timed steps alone (no e2e, accuracy or CPU legs).
        if world > 1:
            dist.destroy_process_group()
        if rank != 0:
            return None
        return {"metric": METRIC, "value": round(value, 1), "unit": "GFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms, 4), "roofline": roofline,
                "kernel_launches": launches, "note": "--kernels-only profiling run"}

    # e2e through the public API with pinned host buffers: every step copies
    # its A and B in and its C out.  Steps are pipelined over three streams
    # (copy in, compute, copy out) with two device buffer sets, as a caller
    # streaming products would run them: step k's copies overlap step k-1's
    # product and step k-2's read-back.  The GEMM stream runs only the
    # product's kernels, one after another.
    hA = torch.from_numpy(A).pin_memory()
    hB = torch.from_numpy(B).pin_memory()
    hC = [torch.empty((GEMM_DIM, GEMM_DIM), dtype=torch.float64).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    dA2 = [torch.empty_like(dA) for _ in range(2)]
    dB2 = [torch.empty_like(dB) for _ in range(2)]
    dC2 = [None, None]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(k):
        j = k % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_comp[j])          # buffers j free: product k-2 done
            dA2[j].copy_(hA, non_blocking=True)
            dB2[j].copy_(hB, non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])             # C buffer j read back (step k-2)
        dC2[j] = ops.ds_matmul_f64(dA2[j], dB2[j], algorithm=algo)
        ev_comp[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[j])
            hC[j].copy_(dC2[j], non_blocking=True)
            ev_out[j].record(s_out)

    for k in range(2):
        e2e_step(k)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for k in range(args.steps):
        e2e_step(k)
    stream.wait_event(ev_out[(args.steps - 1) % 2])
    stream.wait_event(ev_out[args.steps % 2])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_ok = bool(np.array_equal(hC[(args.steps - 1) % 2].numpy().view(np.uint64),
                                 C_host.view(np.uint64))) if rank == 0 else None
    e2e = {"value": round(world * flops_step / (e_ms * 1e-3) / 1e9, 1), "unit": "GFLOP/s",
           "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": int(A.nbytes + B.nbytes),
           "d2h_bytes_per_step": int(A.nbytes),
           "pipeline": "copy-in, compute and copy-out streams, two buffer sets",
           "result_matches_device_run": e2e_ok}

    # The same steps' copies alone (A and B in, C out, on the copy streams,
    # no product): when the e2e step takes about as long, the host copies
    # bound it, not the GPU.
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    c0, c1 = _events()
    c0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for k in range(args.steps):
        j = k % 2
        with torch.cuda.stream(s_in):
            dA2[j].copy_(hA, non_blocking=True)
            dB2[j].copy_(hB, non_blocking=True)
        with torch.cuda.stream(s_out):
            hC[j].copy_(dC2[j], non_blocking=True)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    c1.record(stream)
    torch.cuda.synchronize()
    barrier()
    copy_ms = max_over_ranks(c0.elapsed_time(c1) / args.steps)
    e2e["copies_alone_ms_per_step"] = round(copy_ms, 4)
    e2e["host_copy_GB/s_whole_job"] = round(
        world * (A.nbytes + B.nbytes + A.nbytes) / (copy_ms * 1e-3) / 1e9, 1)
    e2e["limiter"] = ("host copies: the step takes no longer than its copies alone"
                      if e_ms <= 1.1 * copy_ms else
                      "the product: the step outlasts its copies alone")

    if rank == 0:
        err_max, err_med, rows, cols, truth = gemm_error(C_host, A, B)
        ref_err = reference_gemm_error(A, B, rows, cols, truth)
        result["accuracy"] = {"max_abs_err_vs_exact": err_max, "median_abs_err": err_med,
                              "reference_ds_path_max_abs_err": ref_err,
                              "sampled_entries": int(len(rows)),
                              "truth": "exact products summed with math.fsum"}
        # the config's float32 variant: A and B rounded to f32, split as (v, 0)
        A32 = A.astype(np.float32).astype(np.float64)
        B32 = B.astype(np.float32).astype(np.float64)
        C32 = ops.ds_matmul_f64(torch.from_numpy(A32).to(dev), torch.from_numpy(B32).to(dev),
                                algorithm=algo).cpu().numpy()
        e32, _, r32, c32, t32 = gemm_error(C32, A32, B32)
        result["accuracy"]["f32_inputs"] = {
            "max_abs_err_vs_exact": e32,
            "reference_ds_path_max_abs_err": reference_gemm_error(A32, B32, r32, c32, t32)}
        if world == 1:
            result["cpu_baseline"] = cpu_baseline_gemm(A, B)
            if not args.no_secondary:
                result["configs"] = every_config(dev, clk, roofline.get("kernel_ms_per_step"))
    if world > 1 and not args.no_secondary:
        sc = config5_strong(dev, rank, world, barrier, max_over_ranks)
        if rank == 0:
            result["config5_strong_scaling"] = sc

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (numpy default_rng(2) U[-1,1] f64, as the config)",
        "config": gemm_config(world, algo),
        "e2e": e2e, "roofline": roofline, "gpu_launches": gpu_launches,
        "kernel_launches": launches,
        "kernel_launches_pass": "the same steps run again with every kernel family bracketed "
                                "by events; the timed steps bracket the GEMM alone",
        "clocks": clk,
    }
    line.update(result)
    return line


def cpu_baseline_gemm(A, B, reps=1):
    """The reference DS path on the host (NumPy restatement, BLAS on all cores)."""
    from oracle import ds_pass_ref
    with all_host_threads() as pool:
        t = time.perf_counter()
        for _ in range(reps):
            ds_pass_ref.dot_general_f64(A, B)
        dt = (time.perf_counter() - t) / reps
    return {"value": round(2.0 * A.shape[0] * A.shape[1] * B.shape[1] / dt / 1e9, 2),
            "unit": "GFLOP/s", "cores": pool.threads, "kind": "port",
            "sample": f"one full {A.shape[0]}x{A.shape[1]}x{B.shape[1]} DS GEMM: split, four "
                      "float32 numpy matmuls (f32 accumulation), two_sum, recombine"}


# ---------------------------------------------------------------------------
# every configuration in the default line (N = 1)

# f32 operations per iteration of x <- x*a + b: ds_mul 14 (the product and
# its FMA error term 2, cross 3, two_sum 6, low word 3) + ds_add 20 + the
# range test that keeps Dekker's bits (about 2 per element: one min, one
# max and a compare for four chains, one vote).
REC_F32_OPS = 36
FP32_LANES_PER_SM = 128
SMS = 148


def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _time_calls(fn, steps, warmup=3, families=()):
    """Device time per call of fn (CUDA events on the current stream, ms),
    and the named kernel families' device time per call (ms): the family
    events are taken in a second pass, so they do not disturb the first."""
    import torch
    from ds_b200 import _lib
    stream = torch.cuda.current_stream()
    out = None
    for _ in range(warmup):
        out = fn()
    torch.cuda.synchronize()
    e0, e1 = _events()
    e0.record(stream)
    for _ in range(steps):
        out = fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    fam = {}
    if families:
        _lib.profile_reset()
        _lib.profile_enable(True)
        for _ in range(steps):
            fn()
        torch.cuda.synchronize()
        _lib.profile_enable(False)
        for f in families:
            t, n = _lib.profile_read(f)
            fam[f] = t / steps if n else None
    return ms, fam, out


def _graph_replay_us(fn, calls, want):
    """Device time per call (us) of `calls` calls of fn captured in one CUDA
    graph and replayed, and whether the last captured result has the bits
    of `want` (an eager result of the same call)."""
    import torch
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()  # warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            outs = [fn() for _ in range(calls)]
    torch.cuda.current_stream().wait_stream(stream)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    e0, e1 = _events()
    e0.record(cur)
    g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / calls * 1e3
    ok = bool(torch.equal(outs[-1].view(torch.int64), want.view(torch.int64)))
    del g
    return us, ok


def _hbm_roofline(bytes_per_call, kernel_ms, family, peaks, peak_src, workload):
    ach = bytes_per_call / (kernel_ms * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": family, "achieved": round(ach, 1),
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4),
            "traffic": ncu_traffic(family, workload), "peak_source": f"{peak_src} hbm_gbs",
            "kernel_ms": round(kernel_ms, 4)}


def _cpu_rate(fn, work, reps=1):
    fn()
    t = time.perf_counter()
    for _ in range(reps):
        fn()
    return work * reps / (time.perf_counter() - t) / 1e9


def config1_lines(dev, peaks, peak_src):
    """Config 1: y = (a + b) * c on f64 inputs (U[-1,1], seed 0) through the
    DS chain, recombined to f64; at the config's 2^20 (32 MiB, L2-resident:
    no flush) and at 2^26 (2 GiB per call, above L2)."""
    import torch
    from ds_b200 import ops
    from oracle import dso
    out = {}
    for lg in (20, 26):
        n = 1 << lg
        rng = np.random.default_rng(0)
        a, b, c = (rng.uniform(-1, 1, n) for _ in range(3))
        da, db, dc = (torch.from_numpy(v).to(dev) for v in (a, b, c))
        fn = lambda: ops.ds_fused_add_mul3_to_f64(da, db, dc)  # noqa: E731
        ms, fam, y = _time_calls(fn, 50 if lg == 20 else 20, families=("elementwise",))
        got = y.cpu().numpy()
        m = min(n, 1 << 22)
        want = dso.ds_fused_add_mul3_to_f64(a[:m], b[:m], c[:m], dso.max_threads())
        line = {"n": n, "ms": round(ms, 4), "GB/s": round(32.0 * n / (ms * 1e-3) / 1e9, 1),
                "bytes_per_elem": 32,
                "l2": "fits in L2 (no flush: the config's size)" if lg == 20
                      else "inputs and output exceed the 126 MB L2",
                "roofline": _hbm_roofline(32.0 * n, fam["elementwise"], "elementwise", peaks,
                                          peak_src, f"fused_add_mul{n}"),
                "bit_exact_vs_oracle": bool(np.array_equal(got[:m].view(np.uint64),
                                                           want.view(np.uint64))),
                "bit_exact_checked": m,
                "max_abs_err_vs_numpy_f64": float(np.max(np.abs(got - (a + b) * c)))}
        if lg == 20:
            # Back-to-back calls from Python leave the GPU idle between
            # launches at this size, and that idle time falls inside the
            # kernel's events.  The same calls captured in one CUDA graph
            # run with no host gaps: the device time per call, the
            # roofline's time here.
            calls = 50
            gus, gok = _graph_replay_us(fn, calls, y)
            line["graph"] = {"us_per_call": round(gus, 2),
                             "GB/s": round(32.0 * n / (gus * 1e-6) / 1e9, 1),
                             "result_bits_equal": gok,
                             "what": f"{calls} calls captured in one CUDA graph and replayed"}
            line["roofline"] = _hbm_roofline(32.0 * n, gus * 1e-3, "elementwise", peaks,
                                             peak_src, f"fused_add_mul{n}")
            line["roofline"]["kernel_ms_source"] = (
                "graph replay, device time per call (the launch gaps between the graph's "
                "kernels included); the kernel's own events, with host gaps, read "
                f"{fam['elementwise']:.4f} ms")
        # e2e through the public op: pinned inputs copied in, the result out
        ha, hb, hc = (torch.from_numpy(v).pin_memory() for v in (a, b, c))
        hy = torch.empty(n, dtype=torch.float64).pin_memory()

        def e2e():
            da.copy_(ha, non_blocking=True)
            db.copy_(hb, non_blocking=True)
            dc.copy_(hc, non_blocking=True)
            hy.copy_(ops.ds_fused_add_mul3_to_f64(da, db, dc), non_blocking=True)
        ems, _, _ = _time_calls(e2e, 5 if lg == 26 else 20)
        line["e2e"] = {"GB/s": round(32.0 * n / (ems * 1e-3) / 1e9, 1), "ms": round(ems, 4),
                       "h2d_bytes_per_step": 24 * n, "d2h_bytes_per_step": 8 * n}
        ms_ = min(n, 1 << 24)
        one = _cpu_rate(lambda: dso.ds_fused_add_mul3_to_f64(a[:ms_], b[:ms_], c[:ms_], 1),
                        32.0 * ms_)
        th = dso.max_threads()
        allc = _cpu_rate(lambda: dso.ds_fused_add_mul3_to_f64(a[:ms_], b[:ms_], c[:ms_], th),
                         32.0 * ms_, reps=3)
        line["cpu_baseline"] = {"value": round(allc, 3), "unit": "GB/s", "cores": th,
                                "kind": "port", "single_thread_GB/s": round(one, 3),
                                "sample": f"{ms_} elements of (a+b)*c through the C "
                                          "restatement of the reference ops"}
        out[f"n_2^{lg}"] = line
        del da, db, dc, y, ha, hb, hc, hy
    return out


def config2_lines(dev, peaks, peak_src):
    """Config 2: DS sum of x_i = s_i 1e8 + u_i 1e-3 (s alternating, u ~ U[0,1),
    seed 1) at N = 10^4 (launch-bound) and 2^26 (512 MiB)."""
    import torch
    from ds_b200 import ops
    from oracle import dso, exact
    out = {}
    for n in (10_000, 1 << 26):
        s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
        x = s * 1e8 + np.random.default_rng(1).uniform(0, 1, n) * 1e-3
        dx = torch.from_numpy(x).to(dev)
        fn = lambda: ops.ds_sum_f64(dx)  # noqa: E731
        steps = 200 if n == 10_000 else 20
        ms, fam, r = _time_calls(fn, steps, families=("reduce",))
        truth = exact.exact_sum(x)
        h, l = dso.ds_reduce_f64_seq(x)
        err = abs(float(r.item()) - truth)
        ref_err = abs(float(h) + float(l) - truth)
        line = {"n": n, "ms": round(ms, 5), "GB/s": round(8.0 * n / (ms * 1e-3) / 1e9, 1),
                "bytes_per_elem": 8, "abs_err_vs_fsum": err,
                "reference_ds_seq_abs_err": ref_err, "err_le_reference": err <= ref_err,
                "f32_abs_err": abs(float(np.sum(x.astype(np.float32), dtype=np.float32)) - truth)}
        if n == 10_000:
            torch.cuda.synchronize()
            t = time.perf_counter()
            for _ in range(steps):
                fn()
            host_us = (time.perf_counter() - t) / steps * 1e6
            torch.cuda.synchronize()
            kus = fam["reduce"] * 1e3
            graph_us, graph_ok = _graph_replay_us(fn, steps, r)
            line.update({"us_per_call": round(ms * 1e3, 2), "kernel_us": round(kus, 2),
                         "host_us_per_call": round(host_us, 2),
                         "graph_us_per_call": round(graph_us, 2),
                         "graph_result_bits_equal": graph_ok,
                         "bound": "launch: the two kernels (block partials, their fold) run "
                                  f"{kus:.1f} us; back-to-back calls cost "
                                  f"{ms * 1e3:.1f} us each on the device and {host_us:.1f} us "
                                  "of host time (Python op, argument checks, launches); "
                                  f"{steps} calls captured in one CUDA graph replay at "
                                  f"{graph_us:.1f} us per call, the host's share gone"})
        else:
            line["roofline"] = _hbm_roofline(8.0 * n, fam["reduce"], "reduce", peaks, peak_src,
                                             f"reduce{n}")
        m = min(n, 1 << 24)
        rate = _cpu_rate(lambda: dso.ds_reduce_f64_seq(x[:m]), 8.0 * m)
        line["cpu_baseline"] = {"value": round(rate, 3), "unit": "GB/s", "cores": 1,
                                "kind": "port",
                                "sample": f"sequential DS fold of {m} elements (the reference "
                                          "reduce body in index order; one thread, as the "
                                          "order is sequential)"}
        out["n_10^4" if n == 10_000 else "n_2^26"] = line
        del dx
    return out


def config4_lines(dev, peaks, clock_mhz):
    """Config 4: x <- x*a + b, k = 1 .. 1024 times, 2^24 elements (seed 3)."""
    import torch
    from ds_b200 import ops
    from oracle import dso
    n = 1 << 24
    rng = np.random.default_rng(3)
    x0 = rng.uniform(-1, 1, n)
    a = rng.uniform(0.999, 1.001, n)
    b = rng.uniform(-1e-3, 1e-3, n)
    dx, da, db = (torch.from_numpy(v).to(dev) for v in (x0, a, b))
    pipe = SMS * FP32_LANES_PER_SM * clock_mhz * 1e6  # f32 ops/s of the FP32 pipe
    sweep = []
    y = None
    for k in REC_KS:
        fn = lambda k=k: ops.ds_recurrence_mul_add_to_f64(dx, da, db, k)  # noqa: E731
        steps = max(2, min(20, int(2000 / k)))
        ms, fam, y = _time_calls(fn, steps, families=("recurrence",))
        kms = fam["recurrence"]
        ops_s = REC_F32_OPS * n * k / (kms * 1e-3)
        sweep.append({"k": k, "ms": round(ms, 4), "GB/s": round(32.0 * n / (ms * 1e-3) / 1e9, 1),
                      "Gelem_iter_per_s": round(n * k / (ms * 1e-3) / 1e9, 2),
                      "fp32_pipe_frac": round(ops_s / pipe, 4),
                      "hbm_frac": round(32.0 * n / (kms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)})
    m = 1 << 16
    got = y[:m].cpu().numpy()
    want = dso.ds_recurrence_mul_add_to_f64(x0[:m], a[:m], b[:m], REC_KS[-1], dso.max_threads())
    # the reference's own form, z <- (z + y) * y (x0 as z, a as y)
    ref_ms, _, _ = _time_calls(lambda: ops.ds_recurrence_add_mul_to_f64_cuda(dx, da, 1024), 2)
    th = dso.max_threads()
    mm = 1 << 18
    rate = _cpu_rate(lambda: dso.ds_recurrence_mul_add_to_f64(x0[:mm], a[:mm], b[:mm], 1024, th),
                     float(mm) * 1024)
    out = {"n": n, "sweep": sweep, "f32_ops_per_iteration": REC_F32_OPS,
           "fp32_pipe_peak": f"{SMS} SMs x {FP32_LANES_PER_SM} lanes x {clock_mhz:.0f} MHz",
           "bit_exact_vs_oracle_k1024": bool(np.array_equal(got.view(np.uint64),
                                                            want.view(np.uint64))),
           "bit_exact_checked": m,
           "reference_form_(z+y)*y_k1024": {
               "ms": round(ref_ms, 4),
               "Gelem_iter_per_s": round(n * 1024 / (ref_ms * 1e-3) / 1e9, 2)},
           "cpu_baseline": {"value": round(rate, 3), "unit": "Gelem-iter/s", "cores": th,
                            "kind": "port", "sample": f"{mm} elements, k=1024, C restatement"}}
    del dx, da, db, y
    return out


def config5_lines(dev, peaks, peak_src):
    """Config 5 on one GPU: the 65536 x 8192 x 8192 product and the batched
    dot (4096 x 65536), entries 1 + 1e-7 u (seed 4, drawn A, B, X, Y)."""
    import torch
    from ds_b200 import _lib, ops
    from oracle import ds_pass_ref, exact
    out = {}
    A, B, _ = large_inputs("gemm_large", 0, 1)
    dA, dB = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    # two warm-up calls: the allocator then holds both output buffers (the
    # previous result is alive while the next is made), so no cudaMalloc of a
    # 4 GiB result lands in the timed calls
    ms, fam, C = _time_calls(lambda: ops.ds_matmul_f64(dA, dB), 3, warmup=2,
                             families=("ozaki_gemm",))
    info = _lib.gemm_info(LARGE_M, LARGE_N, LARGE_K)
    ach = info["tensor_ops_per_launch"] / (fam["ozaki_gemm"] * 1e-3) / 1e12
    peak = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    rows, cols = exact.sample_indices(LARGE_M, LARGE_N, 64, seed=5)
    Ch = C.cpu().numpy()
    truth = exact.exact_gemm_entries(A, B, rows, cols)
    err = np.abs(Ch[rows, cols] - truth)
    ref_err = reference_gemm_error(A, B, rows, cols, truth)
    sub = A[:256]
    with all_host_threads() as pool:
        rate = _cpu_rate(lambda: ds_pass_ref.dot_general_f64(sub, B),
                         2.0 * 256 * LARGE_N * LARGE_K)
    out["gemm"] = {
        "M": LARGE_M, "N": LARGE_N, "K": LARGE_K, "ms": round(ms, 3),
        "GFLOP/s": round(2.0 * LARGE_M * LARGE_N * LARGE_K / (ms * 1e-3) / 1e9, 1),
        "roofline": {"bound": "tensor", "kernel": "ozaki_gemm", "achieved": round(ach, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(ach / peak, 4),
                     "traffic": None, "kernel_ms": round(fam["ozaki_gemm"], 3),
                     "peak_source": f"2 x {peak_src} bf16_tflops_sustained (a ~45 ms kernel "
                                    "run back to back)"},
        "accuracy": {"max_abs_err_vs_exact": float(err.max()),
                     "reference_ds_path_max_abs_err": ref_err,
                     "err_le_reference": bool(np.all(err <= ref_err)),
                     "sampled_entries": int(len(rows))},
        "cpu_baseline": {"value": round(rate, 2), "unit": "GFLOP/s", "cores": pool.threads,
                         "kind": "port", "sample": "256 rows of A times B: the DS pass in NumPy"}}
    del dA, dB, C, Ch, A, B
    torch.cuda.empty_cache()
    X, Y, _ = large_inputs("batched_dot", 0, 1)
    dX, dY = torch.from_numpy(X).to(dev), torch.from_numpy(Y).to(dev)
    fn = lambda: ops.ds_dot_general_f64(dX, dY, lhs_contracting=1, rhs_contracting=1,  # noqa
                                        lhs_batch=(0,), rhs_batch=(0,))
    ms, fam, d = _time_calls(fn, 10, families=("dot_vec",))
    nbytes = 2.0 * BATCH_DOTS * DOT_LEN * 8
    got = d.cpu().numpy()
    idx = np.arange(0, BATCH_DOTS, BATCH_DOTS // 16)
    truth = np.array([exact.exact_dot(X[i], Y[i]) for i in idx])
    ah, al = ds_pass_ref.from_float(X[idx])
    bh, bl = ds_pass_ref.from_float(Y[idx])
    p = np.einsum("ik,ik->i", ah, bh)
    e = (np.einsum("ik,ik->i", ah, bl) + np.einsum("ik,ik->i", al, bh)) + \
        np.einsum("ik,ik->i", al, bl)
    ref = ds_pass_ref.to_float(*ds_pass_ref.two_sum(p, e))
    derr = np.abs(got[idx] - truth)
    rerr = np.abs(ref - truth)

    def host_dots():
        h1, l1 = ds_pass_ref.from_float(X[:256])
        h2, l2 = ds_pass_ref.from_float(Y[:256])
        return ds_pass_ref.two_sum(np.einsum("ik,ik->i", h1, h2),
                                   (np.einsum("ik,ik->i", h1, l2) +
                                    np.einsum("ik,ik->i", l1, h2)) + np.einsum("ik,ik->i", l1, l2))
    with all_host_threads() as pool:
        rate = _cpu_rate(host_dots, 2.0 * 256 * DOT_LEN * 8)
    out["batched_dot"] = {
        "batch": BATCH_DOTS, "length": DOT_LEN, "ms": round(ms, 3),
        "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1), "bytes_per_mac": 16,
        "roofline": _hbm_roofline(nbytes, fam["dot_vec"], "dot_vec", peaks, peak_src,
                                  "batched_dot"),
        "accuracy": {"max_abs_err_vs_exact": float(derr.max()),
                     "reference_ds_path_max_abs_err": float(rerr.max()),
                     "err_le_reference": bool(np.all(derr <= rerr)), "sampled_dots": len(idx)},
        "cpu_baseline": {"value": round(rate, 2), "unit": "GB/s", "cores": pool.threads,
                         "kind": "port", "sample": "256 of the dot products: the DS pass in NumPy"}}
    del dX, dY, d, X, Y
    torch.cuda.empty_cache()
    return out


def config5_strong(dev, rank, world, barrier, max_over_ranks):
    """Config 5's product strong-scaled over the N ranks: the 65536 rows of A
    split across them, B drawn on rank 0 and broadcast before timing.  T1,
    the whole product on rank 0 alone, is measured in the same run while the
    other ranks wait, so the efficiency T1 / (N T_N) needs no other run.  e2e
    adds each rank's pinned A block copied in and C block copied out."""
    import torch
    from ds_b200 import ops
    from ds_b200 import dist as dsd
    if rank == 0:
        B = torch.from_numpy(large_draw(LARGE_M * LARGE_K, (LARGE_K, LARGE_N))).to(dev)
    else:
        B = torch.empty((LARGE_K, LARGE_N), dtype=torch.float64, device=dev)
    dsd.replicate(B, src=0)
    r0, r1 = shard_rows(LARGE_M, rank, world)
    hA = torch.from_numpy(large_draw(r0 * LARGE_K, (r1 - r0, LARGE_K))).pin_memory()
    dA = hA.to(dev)
    t1 = None
    if rank == 0:
        full = torch.from_numpy(large_draw(0, (LARGE_M, LARGE_K))).to(dev)
        t1, _, c = _time_calls(lambda: ops.ds_matmul_f64(full, B), 3, warmup=2)
        del full, c
        torch.cuda.empty_cache()
    stream = torch.cuda.current_stream()
    C = None
    for _ in range(2):
        C = ops.ds_matmul_f64(dA, B)
    barrier()
    torch.cuda.synchronize()
    steps = 3
    e0, e1 = _events()
    e0.record(stream)
    for _ in range(steps):
        C = ops.ds_matmul_f64(dA, B)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    tn = max_over_ranks(e0.elapsed_time(e1) / steps)
    hC = torch.empty(C.shape, dtype=torch.float64).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        dA.copy_(hA, non_blocking=True)
        C = ops.ds_matmul_f64(dA, B)
        hC.copy_(C, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    te = max_over_ranks(e0.elapsed_time(e1) / steps)
    del dA, B, C
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    flops = 2.0 * LARGE_M * LARGE_N * LARGE_K
    return {"what": "65536x8192x8192 DS GEMM, rows of A split over the ranks, B replicated "
                    "(broadcast before timing); value is the whole job",
            "n_gpus": world, "rows_per_rank": int(r1 - r0),
            "ms_per_step": round(tn, 3), "GFLOP/s": round(flops / (tn * 1e-3) / 1e9, 1),
            "single_gpu_ms_same_run": round(t1, 3),
            "efficiency_vs_single_gpu": round(t1 / (world * tn), 4),
            "e2e": {"ms_per_step": round(te, 3), "GFLOP/s": round(flops / (te * 1e-3) / 1e9, 1),
                    "h2d_bytes_per_step_per_rank": int(hA.numel() * 8),
                    "d2h_bytes_per_step_per_rank": int(hC.numel() * 8),
                    "note": "each rank's copies cross its own PCIe link"}}


def int8_library_line(dev, ours_kernel_ms):
    """cuBLASLt's int8 GEMM (torch._int_mm, s8 x s8 -> s32) at 4096^3 and
    8192^3 on the same GPU, beside the product's own int8 GEMM kernel (14
    residue GEMMs of 4096^3 per launch)."""
    import torch
    out = {}
    for n in (4096, 8192):
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev)
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device=dev)
        ms, _, _ = _time_calls(lambda: torch._int_mm(a, b), 20 if n == 4096 else 10)
        out[f"cublaslt_int8_{n}^3_TOPS"] = round(2.0 * n ** 3 / (ms * 1e-3) / 1e12, 1)
        del a, b
    if ours_kernel_ms:
        ours = 14 * 2.0 * 4096 ** 3 / (ours_kernel_ms * 1e-3) / 1e12
        out["ozaki_gemm_4096^3_TOPS"] = round(ours, 1)
        out["ozaki_gemm_over_cublaslt_4096"] = round(ours / out["cublaslt_int8_4096^3_TOPS"], 3)
    return out


def published_sizes_line(dev):
    """The sizes the reference publishes for this path (one H100 PCIe; its
    handoff.md:386-389), timed its way: wall clock around the call and a
    device synchronize, median of 50 repetitions after 5 warm-up calls, so
    Python dispatch and the synchronize are included.  Inputs are f64
    U[-1,1] (seed 7); the programs are the reference benchmark's."""
    import torch
    from ds_b200 import fuse, ops
    rng = np.random.default_rng(7)

    def median_ms(fn, reps=50):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            t = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t)
        return round(statistics.median(ts) * 1e3, 4)

    n = 1 << 20
    A, B = (torch.from_numpy(rng.uniform(-1, 1, n)).to(dev) for _ in range(2))
    aab = fuse.jit(lambda a, b: a * a + b)
    out = {"method": "wall clock around the call and torch.cuda.synchronize(), median of 50",
           "elementwise_A*A+B_1M": {"ms": median_ms(lambda: aab(A, B)),
                                   "reference_h100_pcie_ms": 0.058,
                                   "program": "one fused DS program, f64 in and out"},
           "sum_1M": {"ms": median_ms(lambda: ops.ds_sum_f64(A)),
                      "reference_h100_pcie_ms": 0.043}}
    for m, ref in ((256, 0.06), (2048, 0.32)):
        X, Y = (torch.from_numpy(rng.uniform(-1, 1, (m, m))).to(dev) for _ in range(2))
        out[f"matmul_{m}^2"] = {"ms": median_ms(lambda: ops.ds_matmul_f64(X, Y)),
                                "reference_h100_pcie_ms": ref}
    out["matmul_2048^2"]["reference_note"] = (
        "the reference's four sub-GEMMs ran at default precision (TF32)")
    return out


def every_config(dev, clk, ours_kernel_ms):
    """The other configurations, each with its roofline, CPU baseline and
    exactness flag (rank 0, N = 1)."""
    peaks, peak_src = measured_peaks()
    mhz = (clk or {}).get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    out = {}
    for name, fn in (("config1_fused_add_mul", lambda: config1_lines(dev, peaks, peak_src)),
                     ("config2_ds_sum", lambda: config2_lines(dev, peaks, peak_src)),
                     ("config4_recurrence", lambda: config4_lines(dev, peaks, mhz)),
                     ("config5", lambda: config5_lines(dev, peaks, peak_src)),
                     ("int8_library_gemm", lambda: int8_library_line(dev, ours_kernel_ms)),
                     ("reference_published_sizes", lambda: published_sizes_line(dev))):
        t = time.perf_counter()
        out[name] = fn()
        out[name]["host_seconds"] = round(time.perf_counter() - t, 1)
    return out


STREAM_METRICS = {
    "fused_add_mul": ("DS fused (a+b)*c -> f64 HBM GB/s", "GB/s"),
    "reduce": ("DS sum of f64 HBM GB/s", "GB/s"),
    "recurrence": ("DS recurrence x<-x*a+b Gelem-iter/s", "Gelem-iter/s"),
}
REC_KS = (1, 4, 16, 64, 256, 1024)


def stream_inputs(workload, n, rank):
    """Seeded inputs of the stream configs (rank r > 0 draws its own shard)."""
    if workload == "fused_add_mul":     # config 1 distribution, seed 0
        rng = np.random.default_rng(0 if rank == 0 else (0, rank))
        return [rng.uniform(-1, 1, n) for _ in range(3)]
    if workload == "reduce":            # config 2: +-1e8 alternating + U[0,1)*1e-3, seed 1
        s = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)
        rng = np.random.default_rng(1 if rank == 0 else (1, rank))
        return [s * 1e8 + rng.uniform(0, 1, n) * 1e-3]
    rng = np.random.default_rng(3 if rank == 0 else (3, rank))   # config 4, seed 3
    x0 = rng.uniform(-1, 1, n)
    a = rng.uniform(0.999, 1.001, n)
    b = rng.uniform(-1e-3, 1e-3, n)
    return [x0, a, b]


def run_stream(args):
    """--workload fused_add_mul | reduce | recurrence: the HBM-bound DS ops.

    Every rank processes its own n elements (weak scaling); the reduce adds
    the ranks' (hi, lo) partials with one all-gather.  Inputs are 2^26
    elements per rank by default (>= 512 MiB, above L2); the recurrence uses
    the config's 2^24 and sweeps k.
    """
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from ds_b200 import _lib, ops
    from ds_b200 import dist as dsd
    wl = args.workload
    n = args.n or (1 << 24 if wl == "recurrence" else 1 << 26)
    host_in = stream_inputs(wl, n, rank)
    dev_in = [torch.from_numpy(v).to(dev) for v in host_in]
    peaks, peak_src = measured_peaks()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps, profile=False):
        # warm-up keeps each result alive like the timed loop does, so that
        # the allocator already holds both output buffers when timing starts
        out = None
        for _ in range(args.warmup):
            out = fn()
        del out
        barrier()
        torch.cuda.synchronize()
        if profile:
            _lib.profile_reset()
            _lib.profile_enable(True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            out = fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps), out

    line = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32x2 (DS) from f64", "data": "synthetic (numpy default_rng, as the configs)"}
    metric, unit = STREAM_METRICS[wl]
    line["metric"], line["unit"] = metric, unit
    clocks = ClockSampler(local)
    if wl in ("fused_add_mul", "reduce"):
        if wl == "fused_add_mul":
            a, b, c = dev_in
            fn = lambda: ops.ds_fused_add_mul3_to_f64(a, b, c)  # noqa: E731
            bpe, fam = 32.0, "elementwise"
            launches_per_step = 1
        else:
            x = dev_in[0]
            if world > 1:
                # the ranks' totals cross NVLink inside the reduce's last kernel
                exchange = dsd.PeerExchange(timeout_ms=2000)
                fn = lambda: dsd.ds_sum_f64_sharded(x, exchange=exchange)  # noqa: E731
            else:
                fn = lambda: ops.ds_sum_f64(x)  # noqa: E731
            bpe, fam = 8.0, "reduce"
            launches_per_step = 2  # block partials; their fold (+ the exchange at N > 1)
        clocks.start()
        ms, out = timed(fn, args.steps, profile=True)
        clk = clocks.stop()
        _lib.profile_enable(False)
        if wl == "reduce" and world > 1:
            exchange.check()
            exchange.close()
        if wl == "fused_add_mul":
            # the same chain as a generated kernel (ds_b200.fuse): one kernel
            # per elementwise DAG, as the retargeted pass would emit it
            from ds_b200 import fuse
            chain = fuse.jit(lambda a_, b_, c_: (a_ + b_) * c_)
            fms, fout = timed(lambda: chain(a, b, c), args.steps)
            line["fused_program"] = {
                "GB/s": round(world * bpe * n / (fms * 1e-3) / 1e9, 1), "ms_per_step": round(fms, 4),
                "bit_exact_vs_hand_written": bool(torch.equal(fout.view(torch.int64),
                                                              out.view(torch.int64)))}
            # sum((a + b) * c): the chain reduced in its own kernel, no stores
            # (24 B read per element), against the chain's packed values
            # written and then read by the packed reduce (8 + 8 B more)
            red = fuse.Prepared([(0, 0, 0, 0.0), (0, 1, 0, 0.0), (2, 0, 1, 0.0), (0, 2, 0, 0.0),
                                 (4, 2, 3, 0.0)], ["f64"] * 3, "packed")
            rms, _ = timed(lambda: red.reduce([a, b, c], (n,)), args.steps)
            two = fuse.jit(lambda a_, b_, c_: (a_ + b_) * c_, out_dtype="packed")
            tms, _ = timed(lambda: ops.ds_reduce_packed(two(a, b, c)), args.steps)
            line["fused_map_reduce"] = {
                "what": "sum((a + b) * c) per rank, one kernel (ds_fused_reduce)",
                "GB/s": round(world * 24.0 * n / (rms * 1e-3) / 1e9, 1),
                "ms_per_step": round(rms, 4), "unfused_ms_per_step": round(tms, 4)}
            # the same kernel over 2^20 .. 2^28 values per rank (uniform
            # [-1, 1) drawn on the device: timing only, no data-dependent path)
            sweep = []
            for lg in (20, 22, 24, 26, 28):
                m = 1 << lg
                xs = [torch.rand(m, dtype=torch.float64, device=dev) * 2 - 1 for _ in range(3)]
                sms, _ = timed(lambda: ops.ds_fused_add_mul3_to_f64(*xs), args.steps)
                sweep.append({"n": m, "GB/s": round(world * 32.0 * m / (sms * 1e-3) / 1e9, 1),
                              "ms_per_step": round(sms, 4),
                              "l2": "fits in L2" if 32.0 * m < 126e6 else "exceeds L2"})
                del xs
            line["size_sweep"] = sweep
        k_ms, k_n = _lib.profile_read(fam)
        # device time of the family per step: at N > 1 the reduce family
        # also holds the tiny combine of the gathered pairs
        per = k_ms / max(args.steps, 1)
        achieved = bpe * n / (per * 1e-3) / 1e9
        line.update({
            "value": round(world * bpe * n / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4),
            "config": {"workload": f"{wl} n={n} per rank", "bytes_per_elem": bpe,
                       "exchange": ("DS totals over NVLink peer stores inside the reduce kernel"
                                    if wl == "reduce" and world > 1 else None),
                       "l2": "inputs exceed the 126 MB L2" if bpe * n > 126e6 else
                             "fits in L2 (no flush)"},
            "roofline": {"bound": "hbm", "kernel": fam, "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "traffic": ncu_traffic(fam, f"{wl}{n}"),
                         "peak_source": f"{peak_src} hbm_gbs",
                         "kernel_ms_per_step": round(per, 4)},
            "gpu_launches": int(launches_per_step * args.steps), "clocks": clk})
        if rank == 0:
            got = out.cpu().numpy()
            from oracle import dso, exact
            if wl == "fused_add_mul":
                m = min(n, 1 << 22)
                want = dso.ds_fused_add_mul3_to_f64(*(v[:m] for v in host_in), dso.max_threads())
                line["accuracy"] = {"bit_exact_vs_oracle_first_2^22": bool(
                    np.array_equal(got[:m].view(np.uint64), want.view(np.uint64)))}
            elif world == 1:
                truth = exact.exact_sum(host_in[0])
                h, l = dso.ds_reduce_f64_seq(host_in[0])
                line["accuracy"] = {"abs_err_vs_fsum": abs(float(got) - truth),
                                    "reference_ds_seq_abs_err": abs(float(h) + float(l) - truth)}
    else:
        x0, a, b = dev_in
        sweep = []
        for k in REC_KS:
            fn = lambda k=k: ops.ds_recurrence_mul_add_to_f64(x0, a, b, k)  # noqa: E731
            steps = max(1, min(args.steps, int(2000 / max(k, 1))))
            ms, out = timed(fn, steps)
            sweep.append({"k": k, "ms": round(ms, 4),
                          "GB/s": round(32.0 * n / (ms * 1e-3) / 1e9, 1),
                          "Gelem_iter_per_s": round(world * n * k / (ms * 1e-3) / 1e9, 2)})
        last = sweep[-1]
        line.update({"value": last["Gelem_iter_per_s"], "ms_per_step": last["ms"],
                     "config": {"workload": f"recurrence x<-x*a+b n={n} per rank, k sweep",
                                "k": list(REC_KS)},
                     "sweep": sweep,
                     "roofline": {"bound": "hbm", "kernel": "recurrence",
                                  "achieved": sweep[0]["GB/s"], "peak": peaks["hbm_gbs"],
                                  "unit": "GB/s",
                                  "frac": round(sweep[0]["GB/s"] / peaks["hbm_gbs"], 4),
                                  "traffic": None, "note": "k=1 (HBM-bound end of the sweep)"},
                     "gpu_launches": len(REC_KS)})
        if rank == 0:
            from oracle import dso
            m = 1 << 16
            got = out[:m].cpu().numpy()
            want = dso.ds_recurrence_mul_add_to_f64(x0[:m].cpu().numpy(), a[:m].cpu().numpy(),
                                                    b[:m].cpu().numpy(), REC_KS[-1],
                                                    dso.max_threads())
            line["accuracy"] = {"bit_exact_vs_oracle_first_2^16_k1024": bool(
                np.array_equal(got.view(np.uint64), want.view(np.uint64)))}
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline_stream(wl, host_in)
    if world > 1:
        dist.destroy_process_group()
    return line if rank == 0 else None


def cpu_baseline_stream(wl, host_in, threads=None):
    """The reference CPU ops (C oracle, OpenMP over the host cores) on a
    bounded sample of the same inputs."""
    from oracle import dso
    threads = threads or dso.max_threads()
    if wl == "fused_add_mul":
        m = min(host_in[0].size, 1 << 24)
        fn = lambda: dso.ds_fused_add_mul3_to_f64(*(v[:m] for v in host_in), threads)  # noqa
        bpe, unit, count = 32.0, "GB/s", m
        sample = f"{m} elements of (a+b)*c"
    elif wl == "reduce":
        m = min(host_in[0].size, 1 << 24)
        fn = lambda: dso.ds_reduce_f64_seq(host_in[0][:m])  # noqa: E731
        bpe, unit, count, threads = 8.0, "GB/s", m, 1
        sample = f"sequential DS fold of {m} elements (the reference reduce body in order)"
    else:
        m = 1 << 18
        fn = lambda: dso.ds_recurrence_mul_add_to_f64(*(v[:m] for v in host_in), 1024, threads)  # noqa
        bpe, unit, count = None, "Gelem-iter/s", m * 1024
        sample = f"{m} elements, k=1024"
    fn()
    t = time.perf_counter()
    fn()
    dt = time.perf_counter() - t
    value = bpe * count / dt / 1e9 if bpe else count / dt / 1e9
    return {"value": round(value, 3), "unit": unit, "cores": threads, "kind": "port",
            "sample": sample}


def run_reference(args):
    """Each step is one full 4096^3 product (one rank's block of the weak-scaled
    job; at N > 1 rank 0 runs it for the whole job, value being a rate)
    through the NumPy restatement of the reference DS pass on all host cores:
    split, four float32 matmuls with f32 accumulation, two_sum, recombine.
    The reference itself needs JAX/XLA, absent in this image."""
    rank, world, _ = env_rank()
    if rank != 0:
        return None
    A, B = gemm_inputs(0)
    from oracle import ds_pass_ref
    with all_host_threads() as pool:
        for _ in range(args.warmup):
            ds_pass_ref.dot_general_f64(A, B)
        t = time.perf_counter()
        for _ in range(args.steps):
            ds_pass_ref.dot_general_f64(A, B)
        dt = (time.perf_counter() - t) / args.steps
    value = 2.0 * GEMM_DIM ** 3 / dt / 1e9
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "GFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32x2 (DS)", "data": "synthetic (default_rng(2))",
        "config": gemm_config(world, args.algorithm),
        "cpu_baseline": {"value": round(value, 2), "unit": "GFLOP/s", "cores": pool.threads,
                         "kind": "port",
                         "sample": "one full 4096^3 DS GEMM per step: the DS pass restated in "
                                   "NumPy (split, 4 float32 matmuls, two_sum, recombine) with "
                                   "BLAS on all host cores"},
        "e2e": {"value": round(value, 2), "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_stream(args):
    """Reference arm of the stream workloads: the reference CPU ops (C oracle)
    on the host cores, one bounded sample per step (rank 0 only)."""
    rank, world, _ = env_rank()
    if rank != 0:
        return None
    wl = args.workload
    n = args.n or (1 << 24 if wl == "recurrence" else 1 << 26)
    host_in = stream_inputs(wl, min(n, 1 << 24), 0)
    vals = [cpu_baseline_stream(wl, host_in) for _ in range(max(1, min(args.steps, 5)))]
    value = statistics.median(v["value"] for v in vals)
    metric, unit = STREAM_METRICS[wl]
    cb = dict(vals[0], value=value)
    return {"impl": "reference", "metric": metric, "value": value, "unit": unit,
            "n_gpus": world, "steps": len(vals), "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "config": {"workload": f"{wl} (bounded host sample)"}, "cpu_baseline": cb,
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the large configuration: 65536 x 8192 x 8192 GEMM and the batched dot

LARGE_M, LARGE_N, LARGE_K = 65536, 8192, 8192
BATCH_DOTS, DOT_LEN = 4096, 65536
LARGE_METRICS = {
    "gemm_large": ("DS-GEMM GFLOP/s 65536x8192x8192 near-cancellation (rows of A sharded)",
                   "GFLOP/s"),
    "batched_dot": ("DS batched dot 4096 x 65536 HBM GB/s", "GB/s"),
}


def large_draw(offset, shape):
    """Values 1 + 1e-7 u, u = default_rng(4).uniform(-1, 1) at stream position
    `offset` onwards (one 64-bit draw per value, so any block of the A, B, X,
    Y sequence is generated without the values before it)."""
    bg = np.random.PCG64(4)
    bg.advance(int(offset))
    return 1.0 + 1e-7 * np.random.Generator(bg).uniform(-1.0, 1.0, shape)


def large_inputs(workload, rank, world):
    """This rank's share of the configuration drawn in the order A, B, X, Y:
    gemm_large -> (A rows, B, first row); batched_dot -> (X rows, Y rows, first row)."""
    if workload == "gemm_large":
        r0, r1 = shard_rows(LARGE_M, rank, world)
        A = large_draw(r0 * LARGE_K, (r1 - r0, LARGE_K))
        B = large_draw(LARGE_M * LARGE_K, (LARGE_K, LARGE_N))
        return A, B, r0
    r0, r1 = shard_rows(BATCH_DOTS, rank, world)
    base = LARGE_M * LARGE_K + LARGE_K * LARGE_N
    X = large_draw(base + r0 * DOT_LEN, (r1 - r0, DOT_LEN))
    Y = large_draw(base + BATCH_DOTS * DOT_LEN + r0 * DOT_LEN, (r1 - r0, DOT_LEN))
    return X, Y, r0


def shard_rows(n, rank, world):
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def run_large(args):
    """--workload gemm_large | batched_dot (strong scaling: the rows of A, or
    the batch of dot products, are split across the ranks; B is replicated)."""
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from ds_b200 import _lib, ops
    from oracle import exact
    wl = args.workload
    L, R, r0 = large_inputs(wl, rank, world)
    dL = torch.from_numpy(L).to(dev)
    dR = torch.from_numpy(R).to(dev)
    stream = torch.cuda.current_stream()
    if wl == "gemm_large":
        step = lambda: ops.ds_matmul_f64(dL, dR)  # noqa: E731
        fam = "ozaki_gemm"
    else:
        step = lambda: ops.ds_dot_general_f64(dL, dR, lhs_contracting=1,  # noqa: E731
                                              rhs_contracting=1, lhs_batch=(0,),
                                              rhs_batch=(0,))
        fam = "dot_vec"
    out = None
    for _ in range(args.warmup):
        out = step()
    del out
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    _lib.profile_reset()
    _lib.profile_enable(True)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        out = step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    _lib.profile_enable(False)
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    k_ms, k_n = _lib.profile_read(fam)
    per = k_ms / args.steps  # device time of the family per step (all its launches)
    launches = {}
    for f in ("ozaki_split_rows", "ozaki_colmax", "ozaki_split_rows_colmax", "ozaki_split_cols",
              "ozaki_gemm",
              "ozaki_crt", "dot_vec"):
        t_, n_ = _lib.profile_read(f)
        if n_:
            launches[f] = {"launches": n_, "ms_total": round(t_, 4)}
    peaks, peak_src = measured_peaks()
    metric, unit = LARGE_METRICS[wl]
    line = {"metric": metric, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic: 1 + 1e-7 u, u = default_rng(4) U[-1,1] in the order A, B, X, Y",
            "clocks": clk, "kernel_launches": launches,
            "gpu_launches": int(sum(v["launches"] for v in launches.values()))}
    if wl == "gemm_large":
        flops = 2.0 * LARGE_M * LARGE_N * LARGE_K
        line["value"] = round(flops / (ms * 1e-3) / 1e9, 1)
        info = _lib.gemm_info(L.shape[0], LARGE_N, LARGE_K)
        ach = info["tensor_ops_per_launch"] / (per * 1e-3) / 1e12
        # a ~50 ms kernel back to back for seconds: the sustained figure
        # (power cap) is its ceiling
        peak = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        line["roofline"] = {"bound": "tensor", "kernel": fam, "achieved": round(ach, 1),
                            "peak": peak, "unit": "TFLOP/s", "frac": round(ach / peak, 4),
                            "traffic": None, "kernel_ms_per_step": round(per, 4),
                            "peak_source": f"2 x {peak_src} bf16_tflops_sustained"}
        line["config"] = {"workload": "ds_dot_general_f64 65536x8192x8192, A rows sharded, "
                                      "B replicated", "M": LARGE_M, "N": LARGE_N, "K": LARGE_K,
                          "rows_per_rank": int(L.shape[0]), "parallelism": f"rows{world}",
                          "l2": "inputs and output exceed the 126 MB L2"}
        if rank == 0:
            C = out.cpu().numpy()
            rows, cols = exact.sample_indices(L.shape[0], LARGE_N, 64, seed=5)
            truth = exact.exact_gemm_entries(L, R, rows, cols)
            err = np.abs(C[rows, cols] - truth)
            ref_err = reference_gemm_error(L, R, rows, cols, truth)
            line["accuracy"] = {"max_abs_err_vs_exact": float(err.max()),
                                "median_abs_err": float(np.median(err)),
                                "reference_ds_path_max_abs_err": ref_err,
                                "sampled_entries": int(len(rows)),
                                "truth": "exact products summed with math.fsum"}
    else:
        nbytes = 2.0 * BATCH_DOTS * DOT_LEN * 8
        line["value"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
        local_bytes = 2.0 * L.shape[0] * DOT_LEN * 8
        ach = local_bytes / (per * 1e-3) / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": fam, "achieved": round(ach, 1),
                            "peak": peaks["hbm_gbs"], "unit": "GB/s",
                            "frac": round(ach / peaks["hbm_gbs"], 4),
                            "traffic": ncu_traffic(fam, "batched_dot") if world == 1 else None,
                            "kernel_ms_per_step": round(per, 4),
                            "peak_source": f"{peak_src} hbm_gbs"}
        line["config"] = {"workload": "ds_dot_general_f64 batched dot, batch 4096 x length "
                                      "65536 (batch sharded)", "bytes_per_mac": 16,
                          "dots_per_rank": int(L.shape[0]), "parallelism": f"batch{world}",
                          "l2": "4 GiB of operands per step exceed the 126 MB L2"}
        if rank == 0:
            got = out.cpu().numpy()
            idx = np.arange(0, L.shape[0], max(1, L.shape[0] // 16))
            truth = np.array([exact.exact_dot(L[i], R[i]) for i in idx])
            from oracle import ds_pass_ref
            ah, al = ds_pass_ref.from_float(L[idx])
            bh, bl = ds_pass_ref.from_float(R[idx])
            p = np.einsum("ik,ik->i", ah, bh)
            e = (np.einsum("ik,ik->i", ah, bl) + np.einsum("ik,ik->i", al, bh)) + \
                np.einsum("ik,ik->i", al, bl)
            h, l_ = ds_pass_ref.two_sum(p, e)
            ref = ds_pass_ref.to_float(h, l_)
            line["accuracy"] = {"max_abs_err_vs_exact": float(np.abs(got[idx] - truth).max()),
                                "reference_ds_path_max_abs_err": float(np.abs(ref - truth).max()),
                                "sampled_dots": int(len(idx))}
    if world > 1:
        dist.destroy_process_group()
    return line if rank == 0 else None


def run_reference_large(args):
    """Reference arm of the large configuration on the host (rank 0 only):
    the DS pass restated in NumPy on a bounded block per step (256 rows of A
    times B, or 256 of the dot products)."""
    rank, world, _ = env_rank()
    if rank != 0:
        return None
    from oracle import ds_pass_ref
    wl = args.workload
    m = 256
    if wl == "gemm_large":
        A = large_draw(0, (m, LARGE_K))
        B = large_draw(LARGE_M * LARGE_K, (LARGE_K, LARGE_N))
        fn = lambda: ds_pass_ref.dot_general_f64(A, B)  # noqa: E731
        work, unit = 2.0 * m * LARGE_N * LARGE_K, "GFLOP/s"
        sample = f"{m} rows of A times B (8192^2) per step"
    else:
        base = LARGE_M * LARGE_K + LARGE_K * LARGE_N
        X = large_draw(base, (m, DOT_LEN))
        Y = large_draw(base + BATCH_DOTS * DOT_LEN, (m, DOT_LEN))

        def fn():
            ah, al = ds_pass_ref.from_float(X)
            bh, bl = ds_pass_ref.from_float(Y)
            p = np.einsum("ik,ik->i", ah, bh)
            e = (np.einsum("ik,ik->i", ah, bl) + np.einsum("ik,ik->i", al, bh)) + \
                np.einsum("ik,ik->i", al, bl)
            return ds_pass_ref.to_float(*ds_pass_ref.two_sum(p, e))
        work, unit = 2.0 * m * DOT_LEN * 8, "GB/s"
        sample = f"{m} of the 4096 dot products per step"
    steps = max(1, min(args.steps, 5))
    with all_host_threads() as pool:
        for _ in range(min(args.warmup, 1)):
            fn()
        t = time.perf_counter()
        for _ in range(steps):
            fn()
        dt = (time.perf_counter() - t) / steps
    value = round(work / dt / 1e9, 2)
    metric, _ = LARGE_METRICS[wl]
    cb = {"value": value, "unit": unit, "cores": pool.threads, "kind": "port",
          "sample": sample + ": the DS pass restated in NumPy (split, four float32 products "
                             "with f32 accumulation, two_sum, recombine)"}
    return {"impl": "reference", "metric": metric, "value": value, "unit": unit,
            "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "config": {"workload": f"{wl} (bounded host sample)"},
            "cpu_baseline": cb, "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gemm")
    ap.add_argument("--algorithm", default="tensor", choices=["tensor", "cuda_core"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--kernels-only", action="store_true",
                    help="time the device steps only (the case used for ncu captures)")
    ap.add_argument("--n", type=int, default=0,
                    help="elements per rank for the stream workloads")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload not in ("gemm",) + tuple(STREAM_METRICS) + tuple(LARGE_METRICS):
        raise SystemExit(f"unknown workload {args.workload!r}")
    if args.impl == "reference":
        if args.workload == "gemm":
            line = run_reference(args)
        elif args.workload in LARGE_METRICS:
            line = run_reference_large(args)
        else:
            line = run_reference_stream(args)
    elif args.workload == "gemm":
        line = run_ours(args)
    elif args.workload in LARGE_METRICS:
        line = run_large(args)
    else:
        line = run_stream(args)
    if line is not None:
        print(json.dumps(line))


if __name__ == "__main__":
    main()
