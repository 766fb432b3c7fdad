"""Benchmark: Cl(6,0) full-cycle training at batch 2^22 per GPU, float64.

One step = one pass of the fused full cycle over the GPU's minibatch:
forward x*W -> residual -> 0.5|r|^2 -> parameter VJP -> (NCCL all-gather of the
per-rank gradient record when N > 1) -> Adam (lr 1e-3, betas 0.9/0.999,
eps 1e-8, V8 semantics). Data is synthetic: X ~ U[-1,1], targets
Y = W* X-products + N(0, 1e-3) noise with W* ~ N(0, 1), W0 ~ N(0, std 1/8).
X and T are 2 GiB each per GPU, far larger than the 126 MB L2, so no flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 launch one process per GPU with torch.distributed.run; rank 0 prints
one JSON line. `value` is device-timed (CUDA events, max over ranks);
`e2e` runs the same step through the public host-buffer call
(geo_b200_trainer_step_host) from pinned host memory, timed on the host around
that synchronous call (max over ranks). `--impl reference` times the
reference's own CPU code (oracle/_ref, compiled from its sources) on the host
cores for the same metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import shutil
import statistics
import subprocess
import sys
import time

import numpy as np

METRIC = "multivector products/s and training samples/s at Cl(6,0), % of HBM/FP64 roofline"
UNIT = "training samples/s"
BYTES_PER_SAMPLE = 2 * 64 * 8     # read x and t once per step (float64, 64 blades)
FLOPS_PER_SAMPLE = 4 * 64 * 64    # forward 2*4^n + parameter VJP 2*4^n
FORWARD_BYTES_PER_SAMPLE = 2 * 64 * 8  # forward: read x, write y


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--batch-log2", type=int, default=22, help="per-GPU batch = 2^k (22 is the headline shape)")
    p.add_argument("--negative", type=int, default=0, help="q of Cl(6-q, q); 0 = Cl(6,0)")
    p.add_argument("--no-extras", action="store_true", help="skip e2e, Cl(3,3) and cpu_baseline legs")
    p.add_argument("--leg", choices=["train", "pairwise-f32", "v8-graph", "forward", "operators", "reference-gpu"],
                   default="train",
                   help="pairwise-f32: run only the float32 pairwise sweep (for profiling)")
    p.add_argument("--pairwise-log2", type=int, default=26, help="batch 2^k of the float32 pairwise sweep")
    p.add_argument("--algorithm", choices=["auto", "cayley", "representation"], default="auto",
                   help="kernel family of the headline step (auto picks the representation for n = 6)")
    return p.parse_args()


# --------------------------------------------------------------------------- helpers
def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s (profiling recipe)"


# --------------------------------------------------------------------------- data
def make_data(lib, sig, batch, seed, left=0):
    """X ~ U[-1,1]; T = x*W* (+ noise 1e-3) via the library's own forward kernel."""
    import torch

    from geometricelementaryoperators_b200 import abi

    gen = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.rand((batch, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    w_star = torch.randn(64, dtype=torch.float64, device="cuda", generator=gen)
    T = torch.empty_like(X)
    plan = abi.BatchGpPlan()
    assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), 6, abi.sig_array(sig)) == 0
    cplan = abi.CudaPlan()
    assert lib.geo_batch_gp_cuda_plan_upload(ctypes.byref(cplan), ctypes.byref(plan)) == 0
    st = lib.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(cplan), ctypes.c_void_p(X.data_ptr()), batch,
                                                   ctypes.c_void_p(w_star.data_ptr()), left,
                                                   ctypes.c_void_p(T.data_ptr()),
                                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    lib.geo_batch_gp_cuda_plan_destroy(ctypes.byref(cplan))
    T.add_(torch.randn(T.shape, dtype=torch.float64, device="cuda", generator=gen), alpha=1e-3)
    w0 = torch.randn(64, dtype=torch.float64, generator=torch.Generator().manual_seed(seed + 1)) * 0.125
    return X, T, w0.numpy()


ALGORITHM_NAMES = {1: "cayley", 2: "representation"}
KERNEL_NAMES = {1: "tiled_kernel<64, cycle> (Cayley matrix, FP64 FMA)",
                2: "rep_ws_kernel<16, 4> (warp-specialised D x D representation, FP64 tensor cores)"}
# DRAM bytes (read + write) per sample of each kernel family, from one ncu
# capture of the same step on 2^20 samples (dram__bytes_read.sum +
# dram__bytes_write.sum of one launch); traffic grows with the samples processed.
NCU_TRAFFIC_PER_SAMPLE = {1: (1.073777e9 + 6.1568e6) / 2**20, 2: (1.073927e9 + 4.560896e6) / 2**20}


class Trainer:
    def __init__(self, lib, sig, w0, left=0, algorithm=0):
        from geometricelementaryoperators_b200 import abi

        self.lib = lib
        self.h = ctypes.c_void_p()
        cfg = abi.OptimizerConfig(2, 1e-3, 0.9, 0.999, 1e-8)
        import numpy as np

        self.w0 = np.ascontiguousarray(w0, dtype=np.float64)
        st = lib.geo_b200_trainer_create(ctypes.byref(self.h), 6, abi.sig_array(sig), left,
                                         self.w0.ctypes.data_as(ctypes.c_void_p), ctypes.byref(cfg))
        if st != 0:
            raise RuntimeError(f"trainer_create failed: {st}")
        if algorithm:
            assert lib.geo_b200_trainer_set_algorithm(self.h, algorithm) == 0
        self.algorithm = lib.geo_b200_trainer_algorithm(self.h)

    def destroy(self):
        self.lib.geo_b200_trainer_destroy(self.h)


# --------------------------------------------------------------------------- reference arm
REFERENCE_CHUNKS = (16, 32, 64, 128, 256, 1024)  # samples per call tried by the calibration


def _reference_worker(args):
    """Run the reference's batched training step (compiled from its sources)
    `calls` times on `chunk` samples: geo_batch_gp_right_mse_sgd_step_f64 =
    forward, residual, 0.5|r|^2, parameter VJP and the SGD update in one call.
    Returns samples processed."""
    calls, seed, signature, chunk = args
    import numpy as np

    from oracle.oracle import Reference

    ref = Reference()
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (chunk, 64))
    t = rng.uniform(-1, 1, (chunk, 64))
    w = rng.normal(0, 0.125, 64)
    done = 0
    for _ in range(calls):
        st, w, _ = ref.sgd_step(signature, x, t, 1e-9, w, False)
        assert st == 0
        done += x.shape[0]
    return done


def reference_chunk(signature) -> int:
    """The call size at which the reference's step runs fastest on this host
    (its term-major loops favour short calls that stay in cache)."""
    best, best_rate = REFERENCE_CHUNKS[0], 0.0
    for chunk in REFERENCE_CHUNKS:
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 0.25:
            done += _reference_worker((max(1, 256 // chunk), 5, signature, chunk))
        rate = done / (time.perf_counter() - t0)
        if rate > best_rate:
            best, best_rate = chunk, rate
    return best


REFERENCE_STEP_NOTE = ("the reference's batch path has no Adam (its Adam lives in the per-sample V8 runtime); "
                       "the O(64) optimizer update per step is negligible beside the O(B) pass")


def reference_step(pool, workers, chunks, signature, chunk):
    t0 = time.perf_counter()
    done = sum(pool.map(_reference_worker, [(chunks, 17 + i, signature, chunk) for i in range(workers)]))
    return done, time.perf_counter() - t0


def headline_config(args, world) -> dict:
    """The workload both arms report (the reference arm times bounded samples of it)."""
    q = args.negative
    batch = 1 << args.batch_log2
    return {"workload": f"Cl({6 - q},{q}) full-cycle training step (forward + parameter VJP + MSE + Adam), "
                        f"parameter on the right, float64, batch 2^{args.batch_log2} per GPU",
            "batch_per_gpu": batch, "global_batch": batch * world, "blades": 64,
            "signature": [1] * (6 - q) + [-1] * q, "optimizer": "adam lr=1e-3 b=(0.9,0.999) eps=1e-8",
            "l2": "inputs 4 GiB per GPU per step > 126 MB L2; no flush needed", "parallelism": f"dp{world}"}


def run_reference_arm(args, world, rank):
    """The reference's own CPU implementation on all host threads (rank 0 only)."""
    if rank != 0:
        return
    from oracle import oracle as orc

    sig = [1] * (6 - args.negative) + [-1] * args.negative
    if not orc.REF_SO.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libgeo_ref.so was not built "
                          "(the reference sources were not present at build time)"}))
        return
    import multiprocessing as mp

    workers = os.cpu_count() or 1
    chunk = reference_chunk(sig)
    ctx = mp.get_context("spawn")
    chunks = max(1, 8192 // chunk)
    with ctx.Pool(workers) as pool:
        reference_step(pool, workers, 1, sig, chunk)  # import + warm
        # size the calls so one step is ~1 s of work on every core
        done, dt = reference_step(pool, workers, chunks, sig, chunk)
        chunks = max(1, int(chunks * 1.0 / max(dt, 1e-3)))
        for _ in range(args.warmup):
            reference_step(pool, workers, chunks, sig, chunk)
        total, elapsed = 0, 0.0
        for _ in range(args.steps):
            done, dt = reference_step(pool, workers, chunks, sig, chunk)
            total += done
            elapsed += dt
    value = total / elapsed
    per_step = workers * chunks * chunk
    sample = (f"each timed step is a bounded sample of this workload: {workers} processes x {chunks} calls of "
              f"geo_batch_gp_right_mse_sgd_step_f64 on {chunk} samples (the fastest call size of "
              f"{list(REFERENCE_CHUNKS)} on this host; {per_step} samples, not the "
              f"2^{args.batch_log2}-sample step); {REFERENCE_STEP_NOTE}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / args.steps,
        "ms_per_step_is": f"the time of one timed sample of {per_step} samples, not of a "
                          f"2^{args.batch_log2}-sample step",
        "samples_per_timed_step": per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": headline_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": workers, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_leg(negative: int) -> dict:
    """Reference CPU code, 1 core, bounded sample of ~10 s on the 2^22 workload's shape."""
    from oracle import oracle as orc

    sig = [1] * (6 - negative) + [-1] * negative
    if orc.REF_SO.exists():
        kind = "reference"
        worker = _reference_worker
    else:
        return {"value": None, "unit": UNIT, "cores": 1, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    chunk = reference_chunk(sig)
    done, t0, calls = 0, time.perf_counter(), 0
    while time.perf_counter() - t0 < 10.0 or calls < 8:
        done += worker((16, 99 + calls, sig, chunk))
        calls += 16
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": UNIT, "cores": 1, "kind": kind,
            "sample": f"{calls} calls of geo_batch_gp_right_mse_sgd_step_f64 on {chunk} samples (the fastest call "
                      f"size of {list(REFERENCE_CHUNKS)} on this host) of the Cl({6 - negative},{negative}) shape, "
                      f"{dt:.1f} s; {REFERENCE_STEP_NOTE}",
            "reference_benchmarks": reference_benchmarks()}


def reference_benchmarks() -> dict:
    """The reference's own CPU benchmarks, unmodified (oracle/_ref), pinned to one core:
    samples/s at n = 6 for each batch size of their built-in matrix."""
    import tempfile

    out = {}
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle", "_ref")
    with tempfile.TemporaryDirectory() as tmp:
        for name, backend in (("bench_v8_batch_gp", "geo_v8_batch"), ("bench_v8_full_cycle", "geo_v8")):
            exe = os.path.join(ref, name)
            csv_path = os.path.join(tmp, name + ".csv")
            if not os.path.exists(exe):
                out[name] = "unavailable: not built"
                continue
            cmd = ([] if shutil.which("taskset") is None else ["taskset", "-c", "0"]) + [exe, csv_path]
            res = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
            if res.returncode != 0 or not os.path.exists(csv_path):
                out[name] = f"failed with exit code {res.returncode}"
                continue
            rows = {}
            with open(csv_path) as f:
                for line in f.read().splitlines()[1:]:
                    b, mode, n, batch, rate, _ = line.split(",")
                    if b == backend and n == "6":
                        rows[f"n6_{mode}_batch{batch}"] = float(rate)
            out[name] = {"unit": "samples/s", "cores": 1, **rows}
    return out


V8_GRAPH_LOG2 = 16
# Explicitly rounded FP64 operations per sample of the all-node-kinds graph at
# n = 6: the GP node costs 3 x 4096 forward (two multiplies and an add per
# term) and 2 x 3 x 4096 backward; the other 12 nodes add < 2% and are ignored.
V8_GRAPH_FP64_OPS = 9 * 4096


def v8_graph_leg(args, world) -> dict:
    """geo_b200_v8_batch_train_step on the all-node-kinds graph (general path), Cl(6,0), Adam."""
    import torch

    from geometricelementaryoperators_b200 import v8
    from geometricelementaryoperators_b200.synthetic import normal

    batch = 1 << V8_GRAPH_LOG2
    sig = [1] * 6
    prog, ids = v8.all_node_kinds_graph(sig, normal(501, (64,), 0.25), normal(502, (64,), 0.25))
    gen = torch.Generator(device="cuda").manual_seed(503)
    X = torch.rand((batch, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    T = torch.rand((batch, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)

    def step():
        return prog.batch_train_step(ids["x"], ids["y"], X.data_ptr(), T.data_ptr(), batch, v8.ADAM, 1e-3)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier(world)
    steps = max(3, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    sec = max_over_ranks((time.perf_counter() - t0) / steps, world)
    prog.free()
    rate = batch / sec
    return {"workload": "all-node-kinds V8 graph (GP, tanh, sigmoid, Hadamard, reverse, involution, conjugate, "
                        f"grade projection, normalisation, squared norm), Cl(6,0), batch 2^{V8_GRAPH_LOG2} per GPU, "
                        "Adam, general batched path",
            "value": rate * world, "unit": "training samples/s", "ms_per_step": sec * 1e3,
            "timing": "host wall clock around the synchronous call, max over ranks",
            "fp64_ops_per_s": rate * V8_GRAPH_FP64_OPS,
            "fp64_pipe_frac": rate * V8_GRAPH_FP64_OPS / 16.8e12,
            "fp64_pipe_peak": "16.8e12 non-fused FP64 operations/s (measured DFMA instruction rate, 33.6 TFLOP/s / 2)"}


def v8_graph_reference_leg() -> dict:
    """The reference's per-sample V8 loop (oracle/_ref) on the same graph, 1 core, bounded sample."""
    from oracle import oracle as orc

    if not orc.REF_SO.exists():
        return {"value": None, "unit": "training samples/s", "cores": 1, "kind": "reference",
                "sample": "unavailable: oracle/_ref not built"}
    from geometricelementaryoperators_b200.synthetic import normal, splitmix_uniform

    ref = orc.Reference()
    values = {"input": np.zeros(64), "target": np.zeros(64), "w1": normal(501, (64,), 0.25),
              "w2": normal(502, (64,), 0.25)}
    B = 2048
    xs = splitmix_uniform(504, (B, 64))
    ts = splitmix_uniform(505, (B, 64))
    t0 = time.perf_counter()
    ref.v8_composed_train([1] * 6, values, xs, ts, 2, 1e-3, steps=1)
    dt = time.perf_counter() - t0
    return {"value": B / dt, "unit": "training samples/s", "cores": 1, "kind": "reference",
            "sample": f"one Adam step over {B} samples of the same graph through the reference's per-sample "
                      f"geo_v8_* loop, {dt:.2f} s"}


def pairwise_f32_leg(lib, args, world) -> dict:
    """y = a * b per element, float32, Cl(6,0); a even-grade stored compact."""
    import torch

    from geometricelementaryoperators_b200 import abi

    batch = 1 << args.pairwise_log2
    gen = torch.Generator(device="cuda").manual_seed(77)
    a = torch.randn((batch, 32), dtype=torch.float32, device="cuda", generator=gen)
    b = torch.rand((batch, 64), dtype=torch.float32, device="cuda", generator=gen).mul_(2).sub_(1)
    y = torch.empty((batch, 64), dtype=torch.float32, device="cuda")
    sig = abi.sig_array([1] * 6)
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ap, bp, yp = (ctypes.c_void_p(t.data_ptr()) for t in (a, b, y))
    for _ in range(2):
        assert lib.geo_b200_pairwise_gp_f32(6, sig, ap, 1, bp, yp, batch, sp) == 0
    torch.cuda.synchronize()
    reps = 5
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        assert lib.geo_b200_pairwise_gp_f32(6, sig, ap, 1, bp, yp, batch, sp) == 0
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / reps, world)
    bytes_per = (32 + 64 + 64) * 4
    gbs = batch * bytes_per / (ms / 1e3) / 1e9
    hbm_peak, _ = peaks()
    del a, b, y
    torch.cuda.empty_cache()
    return {"workload": "Cl(6,0) float32 pairwise products, even-grade left (compact 32) x dense right, "
                        f"batch 2^{args.pairwise_log2} per GPU", "value": batch * world / (ms / 1e3), "unit": "products/s",
            "ms_per_launch": ms, "bytes_per_product": bytes_per, "achieved_gbs": gbs,
            "hbm_frac": gbs / hbm_peak, "flops_per_product": 2 * 32 * 64}


# Measured FP64 peaks on this pool's B200 (148 x 8 warps of independent FMA /
# MMA chains, CUDA events; the FMA and tensor paths share the FP64 units).
FP64_DFMA_TFLOPS = 33.6
FP64_DMMA_TFLOPS = 37.1


def _time_launches(call, world, reps=10, warm=3) -> float:
    """Average device milliseconds of `call` (CUDA events on the current stream), max over ranks."""
    import torch

    stream = torch.cuda.current_stream()
    for _ in range(warm):
        assert call() == 0
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        assert call() == 0
    e.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(s.elapsed_time(e) / reps, world)


def operator_legs(lib, X, world) -> dict:
    """The per-element operator paths at Cl(6,0), float64, on 2^22 elements (x resident,
    2 GiB per operand, far above L2): sparse fixed-multivector plans (reference
    geo_operator_apply_f64) and pairwise products with both operands varying
    (reference geo_operator_gp_f64)."""
    import torch

    from geometricelementaryoperators_b200 import abi

    batch = X.shape[0]
    sig = abi.sig_array([1] * 6)
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    Y = torch.empty_like(X)
    xp, yp = ctypes.c_void_p(X.data_ptr()), ctypes.c_void_p(Y.data_ptr())
    hbm_peak, _ = peaks()
    out = {}
    # Sparse plans: one fixed blade (a signed permutation, pure streaming) and the
    # 32-term even-grade multivector with coefficients 1..32 (both on the right).
    plans = {}
    p1 = abi.OperatorPlanI32()
    assert lib.geo_operator_plan_fixed_blade_i32(ctypes.byref(p1), 6, sig, 0, 0b000011, 3) == 0
    plans["fixed_blade_e12"] = (p1, 1)
    terms = (abi.OperatorTermI32 * 32)()
    evens = [b for b in range(64) if bin(b).count("1") % 2 == 0]
    for i, b in enumerate(evens):
        terms[i].blade, terms[i].coefficient = b, i + 1
    p32 = abi.OperatorPlanI32()
    assert lib.geo_operator_plan_sparse_i32(ctypes.byref(p32), 6, sig, 0, terms, 32) == 0
    plans["sparse_even_32_terms"] = (p32, 32)
    for name, (plan, nterms) in plans.items():
        ms = _time_launches(lambda: lib.geo_b200_sparse_apply_f64(ctypes.byref(plan), xp, yp, batch, sp), world)
        gbs = batch * 1024 / (ms / 1e3) / 1e9
        out["sparse_" + name] = {"value": batch * world / (ms / 1e3), "unit": "products/s", "ms_per_launch": ms,
                                 "bytes_per_product": 1024, "flops_per_product": 2 * 64 * nterms,
                                 "achieved_gbs": gbs, "hbm_frac": gbs / hbm_peak}
    # Pairwise: y[s] = a[s] * b[s], 8192 flops and 1536 B per product.
    Bm = torch.empty_like(X).copy_(X.flip(0))
    bp = ctypes.c_void_p(Bm.data_ptr())
    ms = _time_launches(lambda: lib.geo_b200_pairwise_gp_f64(6, sig, xp, bp, yp, batch, sp), world)
    gbs = batch * 1536 / (ms / 1e3) / 1e9
    tf = batch * 8192 / (ms / 1e3) / 1e12
    # Cl(6,0) runs the representation kernel (1024 FP64 multiply-adds per product);
    # the TFLOP/s figures count the direct product's 4096 multiply-adds.
    rep_note = "Cl(6,0): representation kernel, 1024 multiply-adds per product (direct product: 4096)"
    out["pairwise_f64"] = {"value": batch * world / (ms / 1e3), "unit": "products/s", "ms_per_launch": ms,
                           "bytes_per_product": 1536, "direct_flops_per_product": 8192, "achieved_gbs": gbs,
                           "hbm_frac": gbs / hbm_peak, "direct_equivalent_tflops": tf, "kernel": rep_note}
    # Pairwise VJP: both cotangents (a_bar, b_bar) from y_bar; 16384 flops per product,
    # 2560 algorithmic bytes (a, b, y_bar read once; a_bar, b_bar written).
    Cb = torch.empty_like(X).copy_(X.roll(1, 0))
    Z = torch.empty_like(X)
    cp, zp = ctypes.c_void_p(Cb.data_ptr()), ctypes.c_void_p(Z.data_ptr())
    ms = _time_launches(lambda: lib.geo_b200_pairwise_gp_vjp_f64(6, sig, xp, bp, cp, yp, zp, batch, sp), world)
    tf = batch * 16384 / (ms / 1e3) / 1e12
    gbs = batch * 2560 / (ms / 1e3) / 1e9
    out["pairwise_f64_vjp"] = {"value": batch * world / (ms / 1e3), "unit": "products/s", "ms_per_launch": ms,
                               "bytes_per_product": 2560, "direct_flops_per_product": 16384, "achieved_gbs": gbs,
                               "hbm_frac": gbs / hbm_peak, "direct_equivalent_tflops": tf,
                               "kernel": rep_note + ", two products"}
    # Pairwise JVP: y_dot = a_dot b + a b_dot; 16384 flops, 2560 algorithmic bytes per product.
    ms = _time_launches(lambda: lib.geo_b200_pairwise_gp_jvp_f64(6, sig, xp, bp, cp, zp, yp, batch, sp), world)
    tf = batch * 16384 / (ms / 1e3) / 1e12
    gbs = batch * 2560 / (ms / 1e3) / 1e9
    out["pairwise_f64_jvp"] = {"value": batch * world / (ms / 1e3), "unit": "products/s", "ms_per_launch": ms,
                               "bytes_per_product": 2560, "direct_flops_per_product": 16384, "achieved_gbs": gbs,
                               "hbm_frac": gbs / hbm_peak, "direct_equivalent_tflops": tf,
                               "kernel": rep_note + ", two products in one pass"}
    del Y, Bm, Cb, Z
    torch.cuda.empty_cache()
    out["workload"] = ("Cl(6,0) per-element operators, float64, 2^%d elements per GPU (operands resident, "
                       "%d MiB each, %s)" % (int(math.log2(batch)), batch * 512 >> 20,
                                             "no flush needed" if batch * 512 > (256 << 20) else "small case"))
    out["fp64_peak"] = f"{FP64_DFMA_TFLOPS} TFLOP/s (measured DFMA rate on this pool's B200)"
    return out


def cl41_leg(lib, X, T, world, steps) -> dict:
    """Cl(4,1) (n = 5, 32 blades, mixed signature) full-cycle Adam steps with the
    parameter on either side, on the resident headline arrays read as 2^23 rows of
    32 blades (x and t 2 GiB each, 512 B per sample)."""
    import torch

    from geometricelementaryoperators_b200 import abi

    batch = X.numel() // 32
    sig = abi.sig_array([1, 1, 1, 1, -1])
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    xp, tp = ctypes.c_void_p(X.data_ptr()), ctypes.c_void_p(T.data_ptr())
    w0 = np.ascontiguousarray(np.random.default_rng(41).normal(0.0, 0.125, 32))
    cfg = abi.OptimizerConfig(2, 1e-3, 0.9, 0.999, 1e-8)
    hbm_peak, _ = peaks()
    out = {"workload": f"Cl(4,1) full-cycle training step (forward + parameter VJP + MSE + Adam), float64, batch "
                       f"2^{int(math.log2(batch))} per GPU, 512 B per sample"}
    for side, name in ((0, "right"), (1, "left")):
        h = ctypes.c_void_p()
        assert lib.geo_b200_trainer_create(ctypes.byref(h), 5, sig, side, w0.ctypes.data_as(ctypes.c_void_p),
                                           ctypes.byref(cfg)) == 0
        ms = _time_launches(lambda: lib.geo_b200_trainer_step_device(h, xp, tp, batch, 1.0 / batch, sp), world,
                            reps=steps)
        assert lib.geo_b200_trainer_sync(h, None) == 0
        algo = lib.geo_b200_trainer_algorithm(h)
        lib.geo_b200_trainer_destroy(h)
        gbs = batch * 512 / (ms / 1e3) / 1e9
        out[name] = {"value": batch * world / (ms / 1e3), "unit": "training samples/s", "ms_per_step": ms,
                     "achieved_gbs": gbs, "hbm_frac": gbs / hbm_peak, "algorithm": ALGORITHM_NAMES.get(algo, algo)}
    return out


def forward_leg(lib, X, q, world) -> dict:
    """Fixed-parameter forward y = x*W, Cl(6-q,q), float64, on the batch already
    resident for the training step (2 GiB of x read, 2 GiB of y written per
    launch, far above L2): geo_b200_forward_f64 on the representation kernel,
    the reference ABI's device calls a drop-in caller makes (planned forward and
    the MSE-SGD step with residuals stored: 1536 B per sample, x and t read and
    r written in one pass), and the Cayley kernel beside them."""
    import torch

    from geometricelementaryoperators_b200 import abi

    batch = X.shape[0]
    sig = [1] * (6 - q) + [-1] * q
    w = torch.randn(64, dtype=torch.float64, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9))
    Y = torch.empty_like(X)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    xp, wp, yp = (ctypes.c_void_p(t.data_ptr()) for t in (X, w, Y))
    plan = abi.BatchGpPlan()
    assert lib.geo_batch_gp_plan_init(ctypes.byref(plan), 6, abi.sig_array(sig)) == 0
    cplan = abi.CudaPlan()
    assert lib.geo_batch_gp_cuda_plan_upload(ctypes.byref(cplan), ctypes.byref(plan)) == 0
    T = torch.empty_like(X).copy_(X.roll(3, 0))
    R = torch.empty_like(X)
    w2 = w.clone()
    g = torch.empty(64, dtype=torch.float64, device="cuda")
    loss = torch.empty(1, dtype=torch.float64, device="cuda")
    tp, rp, w2p, gp, lp = (ctypes.c_void_p(t.data_ptr()) for t in (T, R, w2, g, loss))
    calls = {
        "representation": lambda: lib.geo_b200_forward_f64(6, abi.sig_array(sig), 0, 2, xp, wp, yp, batch, sp),
        "device_abi_planned_forward": lambda: lib.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(cplan), xp,
                                                                                       batch, wp, 0, yp, sp),
        "cayley": lambda: lib.geo_b200_forward_f64(6, abi.sig_array(sig), 0, 1, xp, wp, yp, batch, sp),
        # forward -> residual (stored) -> loss -> VJP -> SGD; 1536 algorithmic bytes per sample
        "device_abi_mse_sgd_step": lambda: lib.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(cplan), xp, tp, batch,
                                                                                 1e-9, 0, w2p, rp, gp, lp, sp),
    }
    bytes_per = {"device_abi_mse_sgd_step": 3 * 64 * 8}
    out = {}
    hbm_peak, _ = peaks()
    for name, call in calls.items():
        for _ in range(3):
            assert call() == 0
        torch.cuda.synchronize()
        barrier(world)
        reps = 10
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(reps):
            assert call() == 0
        e.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(s.elapsed_time(e) / reps, world)
        gbs = batch * bytes_per.get(name, FORWARD_BYTES_PER_SAMPLE) / (ms / 1e3) / 1e9
        out[name] = {"value": batch * world / (ms / 1e3), "unit": "samples/s" if name in bytes_per else "products/s",
                     "ms_per_call": ms, "achieved_gbs": gbs, "hbm_frac": gbs / hbm_peak}
    lib.geo_batch_gp_cuda_plan_destroy(ctypes.byref(cplan))
    del Y, T, R
    torch.cuda.empty_cache()
    best = out["representation"]
    return {"workload": f"Cl({6 - q},{q}) fixed-parameter forward y = x*W, float64, batch 2^{int(math.log2(batch))} "
                        f"per GPU (x resident, {batch * 512 >> 20} MiB read + {batch * 512 >> 20} MiB written "
                        "per launch)",
            "value": best["value"], "unit": "products/s", "bytes_per_product": FORWARD_BYTES_PER_SAMPLE,
            "roofline": {"bound": "hbm", "achieved": best["achieved_gbs"], "peak": hbm_peak, "unit": "GB/s",
                         "frac": best["hbm_frac"],
                         "kernel": "rep_fwd_kernel<" + ("16, 4" if q in (0, 1, 5, 6) else "8, 8") +
                                   "> (representation forward, FP64 tensor cores), CUDA events on the launch stream"},
            "kernels": out}


REF_CUDA_SO = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle", "_ref", "libgeo_ref_cuda.so")
REF_GPU_ROWS = {"planned_forward": 20, "mse_sgd_step": 18, "hand_forward": 16}  # log2 rows per leg


def _reference_cuda():
    """The reference's own CUDA code (src/batch_gp_cuda.cu, src/hand_cuda_comparator.cu)
    compiled unmodified for sm_100a into oracle/_ref (a comparator, never part of
    the product), or None when it was not built."""
    if not os.path.exists(REF_CUDA_SO):
        return None
    from geometricelementaryoperators_b200 import abi

    L = ctypes.CDLL(REF_CUDA_SO)  # RTLD_LOCAL, linked -Bsymbolic: its symbols stay its own
    for name, (res, argtypes) in abi.SIGNATURES.items():
        if name.startswith(("geo_batch_gp_cuda_", "geo_hand_cuda_")) and hasattr(L, name):
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, argtypes
    return L


def reference_gpu_leg(lib, world) -> dict:
    """The reference's own CUDA kernels against this library's entry points of the
    same names, on the same B200, Cl(6,0), float64, parameter on the right: the
    planned forward, the MSE-SGD step (forward, residual + loss with atomics, the
    reference's 64-thread serial parameter VJP, SGD) and the hand-written forward.
    Each pair runs on the same resident rows; rates are rows per second."""
    import torch

    from geometricelementaryoperators_b200 import abi
    from oracle.oracle import Reference

    R = _reference_cuda()
    if R is None:
        return {"unavailable": "oracle/_ref/libgeo_ref_cuda.so was not built (the reference sources were not "
                               "present at build time)"}
    sig = [1] * 6
    host_plan = Reference().plan(sig)  # the reference's own plan_init
    rplan, oplan = abi.CudaPlan(), abi.CudaPlan()
    hp = ctypes.cast(host_plan, ctypes.POINTER(abi.BatchGpPlan))
    assert R.geo_batch_gp_cuda_plan_upload(ctypes.byref(rplan), hp) == 0
    assert lib.geo_batch_gp_cuda_plan_upload(ctypes.byref(oplan), hp) == 0
    rows = 1 << max(REF_GPU_ROWS.values())
    gen = torch.Generator(device="cuda").manual_seed(11)
    X = torch.rand((rows, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    T = torch.rand((rows, 64), dtype=torch.float64, device="cuda", generator=gen).mul_(2).sub_(1)
    w = torch.randn(64, dtype=torch.float64, device="cuda", generator=gen).mul_(0.125)
    Y, Yr, Res = torch.empty_like(X), torch.empty_like(X), torch.empty_like(X)
    g, loss = torch.empty(64, dtype=torch.float64, device="cuda"), torch.empty(1, dtype=torch.float64, device="cuda")
    w_r, w_o = w.clone(), w.clone()
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    out = {"workload": "Cl(6,0), float64, parameter on the right; rows per leg: " +
                       ", ".join(f"{k} 2^{v}" for k, v in REF_GPU_ROWS.items()),
           "reference_build": "src/batch_gp_cuda.cu + src/hand_cuda_comparator.cu, unmodified, nvcc -O3 "
                              "-gencode arch=compute_100a,code=sm_100a (oracle/Makefile)"}
    for name, log2 in REF_GPU_ROWS.items():
        n = 1 << log2
        if name == "planned_forward":
            ref = lambda: R.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(rplan), P(X), n, P(w), 0, P(Yr), sp)
            ours = lambda: lib.geo_batch_gp_cuda_planned_forward_f64(ctypes.byref(oplan), P(X), n, P(w), 0, P(Y), sp)
        elif name == "hand_forward":
            ref = lambda: R.geo_hand_cuda_forward_f64(ctypes.byref(rplan), P(X), n, P(w), 0, P(Yr), sp)
            ours = lambda: lib.geo_hand_cuda_forward_f64(ctypes.byref(oplan), P(X), n, P(w), 0, P(Y), sp)
        else:
            ref = lambda: R.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(rplan), P(X), P(T), n, 1e-9, 0, P(w_r),
                                                               P(Res), P(g), P(loss), sp)
            ours = lambda: lib.geo_batch_gp_cuda_mse_sgd_step_f64(ctypes.byref(oplan), P(X), P(T), n, 1e-9, 0,
                                                                  P(w_o), P(Res), P(g), P(loss), sp)
        ms_ref = _time_launches(ref, world, reps=2, warm=1)
        ms_ours = _time_launches(ours, world, reps=10, warm=3)
        entry = {"rows": n, "reference_ms": ms_ref, "ours_ms": ms_ours, "reference_rows_per_s": n / (ms_ref / 1e3),
                 "ours_rows_per_s": n / (ms_ours / 1e3), "speedup": ms_ref / ms_ours}
        if name != "mse_sgd_step":
            assert ref() == 0 and ours() == 0
            torch.cuda.synchronize()
            entry["max_abs_diff"] = float((Y[:n] - Yr[:n]).abs().max())
        out[name] = entry
    R.geo_batch_gp_cuda_plan_destroy(ctypes.byref(rplan))
    lib.geo_batch_gp_cuda_plan_destroy(ctypes.byref(oplan))
    del X, T, Y, Yr, Res
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------- main arm
def run_b200(args, world, rank, local):
    import numpy as np
    import torch

    from geometricelementaryoperators_b200 import abi

    lib = abi.lib()
    batch = 1 << args.batch_log2
    q = args.negative
    sig = [1] * (6 - q) + [-1] * q
    X, T, w0 = make_data(lib, sig, batch, 1234 + rank)
    tr = Trainer(lib, sig, w0, algorithm={"auto": 0, "cayley": 1, "representation": 2}[args.algorithm])
    comm = ctypes.c_void_p()
    if world > 1:
        import torch.distributed as dist

        uid = (ctypes.c_ubyte * 128)()
        if rank == 0:
            assert lib.geo_b200_comm_unique_id(uid) == 0
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        st = lib.geo_b200_comm_create(ctypes.byref(comm), rank, world, uid, 120000)
        if st != 0:
            raise RuntimeError(f"comm_create failed: {st}")
        assert lib.geo_b200_trainer_attach_comm(tr.h, comm) == 0
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    xp, tp = ctypes.c_void_p(X.data_ptr()), ctypes.c_void_p(T.data_ptr())
    scale = 1.0 / (batch * world)

    def step():
        st = lib.geo_b200_trainer_accumulate_device(tr.h, xp, tp, batch, sp)
        if st != 0:
            raise RuntimeError(f"accumulate failed: {st}")
        st = lib.geo_b200_trainer_apply(tr.h, scale, sp)
        if st != 0:
            raise RuntimeError(f"apply failed: {st}")

    for _ in range(args.warmup):
        step()
    loss0 = ctypes.c_double()
    assert lib.geo_b200_trainer_sync(tr.h, ctypes.byref(loss0)) == 0
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    time.sleep(0.4)
    k_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(args.steps):
        k_start[i].record(stream)
        st = lib.geo_b200_trainer_accumulate_device(tr.h, xp, tp, batch, sp)
        k_end[i].record(stream)
        st |= lib.geo_b200_trainer_apply(tr.h, scale, sp)
        if st != 0:
            raise RuntimeError(f"step failed: {st}")
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clock_info = clocks.stop()
    loss = ctypes.c_double()
    status = lib.geo_b200_trainer_sync(tr.h, ctypes.byref(loss))
    if status != 0:
        raise RuntimeError(f"training reported status {status}")
    step_ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    kernel_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(k_start, k_end)) / args.steps, world)
    value = batch * world / (step_ms / 1e3)

    extras = {}
    if not args.no_extras:
        # The other kernel family on the same data, for comparison.
        other = 1 if tr.algorithm == 2 else 2
        try:
            trc = Trainer(lib, sig, w0, algorithm=other)
        except AssertionError:
            trc = None
        if trc is not None:
            if world > 1:
                assert lib.geo_b200_trainer_attach_comm(trc.h, comm) == 0
            for _ in range(args.warmup):
                assert lib.geo_b200_trainer_step_device(trc.h, xp, tp, batch, scale, sp) == 0
            torch.cuda.synchronize()
            barrier(world)
            sc, ec = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            sc.record(stream)
            for _ in range(args.steps):
                assert lib.geo_b200_trainer_step_device(trc.h, xp, tp, batch, scale, sp) == 0
            ec.record(stream)
            torch.cuda.synchronize()
            assert lib.geo_b200_trainer_sync(trc.h, None) == 0
            msc = max_over_ranks(sc.elapsed_time(ec) / args.steps, world)
            extras["other_algorithm"] = {"algorithm": ALGORITHM_NAMES[other],
                                         "value": batch * world / (msc / 1e3), "ms_per_step": msc}
            trc.destroy()
        # Float32 pairwise products, Cl(6,0), batch 2^26: even-grade left operand
        # (compact, 32 floats), dense right operand; HBM-bound sweep.
        extras["pairwise_f32"] = pairwise_f32_leg(lib, args, world)
        extras["v8_graph"] = v8_graph_leg(args, world)
        # Fixed-parameter forward (multivector products/s) on the same resident batch.
        extras["forward"] = forward_leg(lib, X, q, world)
        extras["operators"] = operator_legs(lib, X, world)
        extras["cl41"] = cl41_leg(lib, X, T, world, args.steps)
        # Same step on Cl(3,3) (the second signature of the headline config).
        X2, T2, w2 = X, T, w0
        tr33 = Trainer(lib, [1, 1, 1, -1, -1, -1], w2)
        if world > 1:
            assert lib.geo_b200_trainer_attach_comm(tr33.h, comm) == 0
        for _ in range(args.warmup):
            assert lib.geo_b200_trainer_step_device(tr33.h, xp, tp, batch, scale, sp) == 0
        torch.cuda.synchronize()
        barrier(world)
        s33, e33 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s33.record(stream)
        for _ in range(args.steps):
            assert lib.geo_b200_trainer_step_device(tr33.h, xp, tp, batch, scale, sp) == 0
        e33.record(stream)
        torch.cuda.synchronize()
        assert lib.geo_b200_trainer_sync(tr33.h, None) == 0
        ms33 = max_over_ranks(s33.elapsed_time(e33) / args.steps, world)
        extras["cl33"] = {"value": batch * world / (ms33 / 1e3), "ms_per_step": ms33}
        tr33.destroy()

        # End to end through the public host-buffer call from pinned memory.
        hx = X.cpu().pin_memory()
        ht = T.cpu().pin_memory()
        e2e_steps = max(3, min(args.steps, 10))
        loss_h = ctypes.c_double()
        hxp, htp = ctypes.c_void_p(hx.data_ptr()), ctypes.c_void_p(ht.data_ptr())
        assert lib.geo_b200_trainer_step_host(tr.h, hxp, htp, batch, scale, ctypes.byref(loss_h)) == 0
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            assert lib.geo_b200_trainer_step_host(tr.h, hxp, htp, batch, scale, ctypes.byref(loss_h)) == 0
        torch.cuda.synchronize()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / e2e_steps, world)
        extras["e2e"] = {"value": batch * world / e2e_s, "unit": UNIT,
                         "h2d_bytes_per_step": 2 * batch * 64 * 8 * world, "d2h_bytes_per_step": 8 * world,
                         "timing": "host wall clock around the synchronous host-buffer call, max over ranks",
                         # the reference CUDA harness's classes (benchmarks/bench_v8_cuda.cu:124-135):
                         # `value` is its "resident" class, this one its "transfer_compute" (inputs
                         # uploaded every step; here the loss is also read back)
                         "timing_class": "transfer_compute",
                         "steps": e2e_steps}
        del hx, ht

    hbm_peak, peak_src = peaks()
    algo_bytes = batch * BYTES_PER_SAMPLE
    achieved = algo_bytes / (kernel_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak,
                "traffic": NCU_TRAFFIC_PER_SAMPLE[tr.algorithm] * batch if args.negative == 0 else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum on 2^20 samples, "
                                  "scaled to the launch's samples",
                "peak_source": peak_src,
                "kernel": KERNEL_NAMES[tr.algorithm] + " + record reduction, CUDA events on the launch stream",
                "kernel_ms": kernel_ms,
                "fp64_flops_achieved_tflops": batch * FLOPS_PER_SAMPLE / (kernel_ms / 1e3) / 1e12}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": headline_config(args, world),
            "roofline": roofline,
            "gpu_launches": args.steps * 3,
            "clocks": clock_info,
            "final_loss_sum": loss.value,
            "algorithm": ALGORITHM_NAMES[tr.algorithm],
        }
        if "other_algorithm" in extras:
            line["other_algorithm"] = extras["other_algorithm"]
        if "e2e" in extras:
            line["e2e"] = extras["e2e"]
        if "cl33" in extras:
            line["cl33"] = extras["cl33"]
        if "pairwise_f32" in extras:
            line["pairwise_f32"] = extras["pairwise_f32"]
        if "v8_graph" in extras:
            line["v8_graph"] = extras["v8_graph"]
        if "forward" in extras:
            line["forward"] = extras["forward"]
        if "operators" in extras:
            line["operators"] = extras["operators"]
        if "cl41" in extras:
            line["cl41"] = extras["cl41"]
        if world == 1 and not args.no_extras:
            line["cpu_baseline"] = cpu_baseline_leg(q)
            # Baseline on the GPU: the reference's own CUDA kernels on this B200.
            line["reference_gpu_baseline"] = reference_gpu_leg(lib, world)
            line["v8_graph"]["cpu_baseline"] = v8_graph_reference_leg()
        print(json.dumps(line), flush=True)
    tr.destroy()
    if world > 1:
        lib.geo_b200_comm_destroy(comm)


def main():
    args = parse()
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.leg == "v8-graph":
            res = v8_graph_leg(args, world)
            if rank == 0:
                if world == 1:
                    res["cpu_baseline"] = v8_graph_reference_leg()
                print(json.dumps(res), flush=True)
            return
        if args.leg in ("forward", "operators"):
            import torch

            from geometricelementaryoperators_b200 import abi

            gen = torch.Generator(device="cuda").manual_seed(5)
            X = torch.rand((1 << args.batch_log2, 64), dtype=torch.float64, device="cuda", generator=gen)
            X.mul_(2).sub_(1)
            res = (forward_leg(abi.lib(), X, args.negative, world) if args.leg == "forward"
                   else operator_legs(abi.lib(), X, world))
            if rank == 0:
                print(json.dumps(res), flush=True)
            return
        if args.leg == "reference-gpu":
            from geometricelementaryoperators_b200 import abi

            res = reference_gpu_leg(abi.lib(), world)
            if rank == 0:
                print(json.dumps(res), flush=True)
            return
        if args.leg == "pairwise-f32":
            from geometricelementaryoperators_b200 import abi

            res = pairwise_f32_leg(abi.lib(), args, world)
            if rank == 0:
                print(json.dumps(res), flush=True)
            return
        run_b200(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
