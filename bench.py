#!/usr/bin/env python
"""Benchmark: data-parallel 3-layer MLP training loop (1024->4096->4096->10,
global batch 65536, cross_entropy, SGD by rebind), TensorLang program executed
by the B200 backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

One step = one iteration of the program's training loop over the global
batch (forward, device backward, NCCL gradient all-reduce, fused SGD
update), replayed from a captured CUDA graph.  The batch is split
contiguously over the ranks (strong scaling: the global batch is fixed).
Timing: CUDA events on the backend's stream around K steps, after W warm-up
steps, with a host barrier and device sync on both sides; the reported time
is the maximum over ranks.  The working set (x: 256 MiB, activations
1 GiB each) exceeds the 126 MB L2, so no flush is needed between steps.

Rank 0 prints one JSON line.  At one GPU it also reports the fused
elementwise chain gelu(add(mult(x,s),b)) > 0 on [8192,8192] (GB/s against
HBM) under "fused_op".  ``--impl reference`` times the reference's NumPy
execution of the same step (the float32 oracle restatement of its kernels
and autograd) on the host cores instead.
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
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

B_GLOBAL, D_IN, D_H, N_CLS = 65536, 1024, 4096, 10
FLOP_PER_STEP = 7_712_686_521_792  # fwd 3 GEMMs + dW 3 + dX of layers 2,3
FUSED_N = 8192
FUSED_BYTES = 805_371_904  # read x, write y and m, plus s and b
C4_SHAPE = (8192, 4096, 4096)  # linear layer X[8192,4096] @ W[4096,4096]
C4_FLOP = 3 * 2 * 8192 * 4096 * 4096  # forward, dW, dX
METRIC = "MLP train steps/sec (3-layer 1024-4096-4096-10, batch 65536)"
# GEMM operand schemes (tl_gemm_set_scheme): code, description, and bf16
# MMA-times per fp32 product -- the scheme's ceiling is the bf16 peak / that
GEMM_SCHEMES = {
    "bf16x3": (2, "tcgen05 BF16X3: a0*b0 plus one bf16 pair MMA for a0*b1 + a1*b0", 3),
    "tf32bf16": (1, "tcgen05 split-TF32: TF32 hi*hi plus one bf16 pair MMA for the corrections", 4),
    "3xtf32": (0, "tcgen05 split-TF32: TF32 hi*hi + hi*lo + lo*hi", 6),
}
# DRAM bytes (read + written) of one hidden-layer GEMM kernel launch
# (65536 x 4096 x 4096, CTA pairs) per scheme, from a one-pass ncu capture of
# `bench.py --micro gemm --gemm-m 65536`; None where not captured
GEMM_TRAFFIC_BYTES = {"bf16x3": 5_250_906_112 + 1_057_456_640,
                      "tf32bf16": 10_070_651_136 + 1_101_682_176}


def set_gemm_scheme(tl, name):
    tl.runtime.check(tl.runtime.lib().tl_gemm_set_scheme(GEMM_SCHEMES[name][0], None), "gemm scheme")


TILE_SCHEDULES = {"static": 0, "dynamic": 1, "auto": 2}


def set_tile_schedule(tl, name):
    tl.runtime.check(tl.runtime.lib().tl_gemm_set_tile_schedule(TILE_SCHEDULES[name], None),
                     "tile schedule")


def set_store_path(tl, name):
    tl.runtime.check(tl.runtime.lib().tl_gemm_set_store_path(1 if name == "tma" else 0, None),
                     "store path")


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled through NVML (read-only queries)
    every 10 ms from a thread, plus explicit samples taken inside the timed
    region, so even a region of a few milliseconds has samples."""

    # NVML clocks-event reason bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.h = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.h = None

    def sample(self):
        if self.h is None:
            return
        try:
            sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            try:
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                r = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            self.samples.append((float(sm), int(r)))
        except Exception:
            pass

    def _loop(self):
        while not self._stop.wait(0.01):
            self.sample()

    def start(self):
        self.samples = []
        self._stop.clear()
        self.sample()
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def stop(self):
        if self.h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self.sample()
        self._stop.set()
        self.t.join(timeout=2)
        sm = [s for s, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_sm,
                "reasons": reasons, "samples": len(sm), "source": "nvml"}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------------------
# CPU baseline: the reference's NumPy execution (float32 oracle restatement)
# ---------------------------------------------------------------------------

def _oracle():
    from oracle import OracleProgram
    from __graft_entry__ import load_package
    tl = load_package()
    return tl, OracleProgram


def _env(tl, ast):
    return {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}


def cpu_mlp_step_times(steps: int, warmup: int):
    """Seconds of each full-batch (65536-row) training step of the float32
    oracle, after ``warmup`` untimed steps."""
    tl, OracleProgram = _oracle()
    pr = tl.programs
    ast = pr.mlp3_train(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, epochs=1)
    feeds = pr.mlp3_inputs(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, seed=0)
    env = _env(tl, ast)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        OracleProgram(ast, env, dtype=np.float32, feeds=feeds).run()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times


def _best(fn, reps):
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_configs():
    """The float32 oracle on the other workloads (best of 3 for the single
    ops, best of 20 for the small training step, one run of the linear layer)."""
    tl, OracleProgram = _oracle()
    pr = tl.programs
    out = {}
    ast, feeds = pr.mlp2_step(), pr.mlp2_inputs(seed=0)
    env = _env(tl, ast)
    t = _best(lambda: OracleProgram(ast, env, dtype=np.float32, feeds=feeds).run(), 20)
    out["mlp2_step_64x128"] = {"us_per_step": t * 1e6, "protocol": "best of 20"}
    ast, feeds = pr.fused_chain(FUSED_N), pr.fused_chain_inputs(FUSED_N, seed=0)
    env = _env(tl, ast)
    t = _best(lambda: OracleProgram(ast, env, dtype=np.float32, feeds=feeds).run(), 3)
    out["fused_chain_8192"] = {"s": t, "GB/s": FUSED_BYTES / t / 1e9, "protocol": "best of 3"}
    R, C_ = 16384, 4096
    feeds = pr.reductions_inputs(R, C_, seed=0)
    ops = {}
    from oracle.tl_oracle import op_forward
    for name, op, ax in pr.REDUCTION_OPS + [("sm", "softmax", 1), ("ln", "layer_norm", 1)]:
        src = {"argmax1": "xa1", "argmax0": "xa0", "argmin1": "xi1", "argmin0": "xi0"}.get(name, "x")
        expr = {"type": op, "tensor": src, "axis": ax}
        if op == "layer_norm":
            expr["eps"] = 0.00001
        t = _best(lambda: op_forward(expr, feeds, np.float32), 3)
        nbytes = 4.0 * R * C_ * (2 if op in ("softmax", "layer_norm") else 1)
        ops[f"{op}(axis={ax})" if ax is not None else f"{op}(all)"] = {
            "s": t, "GB/s": nbytes / t / 1e9}
    out["reductions_16384x4096"] = {"ops": ops, "protocol": "best of 3 per op"}
    M, K, N = C4_SHAPE
    ast, feeds = pr.linear_layer(M, K, N), pr.linear_layer_inputs(M, K, N, seed=0)
    env = _env(tl, ast)
    t = _best(lambda: OracleProgram(ast, env, dtype=np.float32, feeds=feeds).run(), 1)
    out["linear_layer_8192x4096x4096"] = {"s": t, "GFLOP/s": C4_FLOP / t / 1e9,
                                          "protocol": "one forward + backward"}
    return out


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    # full-batch steps cost ~10 s each on the host: at most 2 timed steps
    # after 1 warm-up step, whatever --steps/--warmup ask for
    steps, warmup = max(1, min(args.steps, 2)), min(args.warmup, 1)
    samples = cpu_mlp_step_times(steps, warmup)
    t = float(np.mean(samples))
    value = 1.0 / t
    line = {
        "impl": "reference", "metric": METRIC,
        "value": value, "unit": "steps/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "steps_requested": args.steps, "warmup_requested": args.warmup,
        "ms_per_step": t * 1000.0, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "mlp3_dp_train", "global_batch": B_GLOBAL, "dims": [D_IN, D_H, D_H, N_CLS],
                   "parallelism": "host numpy", "l2": "inputs larger than L2"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} full-batch ({B_GLOBAL}-row) training steps of the "
                                   f"float32 NumPy oracle after {warmup} warm-up step; "
                                   f"mean {t:.2f} s per step"},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_cpu_configs:
        line["configs"] = cpu_configs()
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def time_events(tl, stream, fn, reps):
    rt = tl.runtime
    e0, e1 = rt.Event(), rt.Event()
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    rt.lib().tl_stream_sync(stream)
    return e0.elapsed_ms(e1) / reps


def e2e_time(tl, dev, loop, stream, px, pt, pl, xs, ts, steps):
    """Milliseconds per training step with every batch uploaded from pinned host
    memory and every loss read back to the host.

    Step i+1's batch is copied host->device on a separate copy stream into
    staging buffers while step i computes; step i+1 then moves it into place
    with a device-to-device copy, re-prepares the hoisted operands of the
    (new) batch and replays the iteration graph.  The timed region holds
    exactly ``steps`` host->device batch copies and ``steps`` loss reads; the
    first upload is not overlapped with anything."""
    rt = tl.runtime
    L = rt.lib()
    hx, ht, hl = rt.PinnedHost(xs.nbytes), rt.PinnedHost(ts.nbytes), rt.PinnedHost(4)
    hx.array(xs.shape)[...] = xs
    ht.array(ts.shape)[...] = ts
    sx, st = rt.DeviceBuffer(dev, xs.shape), rt.DeviceBuffer(dev, ts.shape)
    cs = ctypes.c_void_p()
    rt.check(L.tl_stream_create(ctypes.byref(cs)), "copy stream")
    copy = cs.value
    start, end, ready, consumed = rt.Event(), rt.Event(), rt.Event(), rt.Event()

    def upload():
        rt.check(L.tl_memcpy_h2d(sx.ptr, hx.ptr, xs.nbytes, copy), "h2d x")
        rt.check(L.tl_memcpy_h2d(st.ptr, ht.ptr, ts.nbytes, copy), "h2d t")
        ready.record(copy)

    def step(prefetch):
        rt.check(L.tl_stream_wait_event(stream, ready.ptr), "wait batch")
        rt.check(L.tl_memcpy_d2d(px, sx.ptr, xs.nbytes, stream), "d2d x")
        rt.check(L.tl_memcpy_d2d(pt, st.ptr, ts.nbytes, stream), "d2d t")
        consumed.record(stream)
        if prefetch:  # the next batch streams in while this step computes
            rt.check(L.tl_stream_wait_event(copy, consumed.ptr), "wait staging")
            upload()
        loop.run_hoisted()
        loop.replay(1)
        rt.check(L.tl_memcpy_d2h(hl.ptr, pl, 4, stream), "d2h loss")

    def run(n):
        start.record(stream)
        rt.check(L.tl_stream_wait_event(copy, start.ptr), "wait start")
        upload()
        for i in range(n):
            step(i + 1 < n)
        end.record(stream)
        rt.check(L.tl_stream_sync(stream), "sync")
        return start.elapsed_ms(end) / n

    try:
        run(2)  # untimed: warms the copy path
        return run(steps)
    finally:  # cleanup: an error raised above is the one to report
        L.tl_stream_sync(copy)
        L.tl_stream_destroy(copy)
        hx.free()
        ht.free()
        hl.free()


def fused_op_bench(tl, dev, reps=20):
    """The fused elementwise chain on [8192,8192], GB/s of algorithmic traffic."""
    pr = tl.programs
    ast, feeds = pr.fused_chain(FUSED_N), pr.fused_chain_inputs(FUSED_N, seed=0)
    P = tl.Program(ast, None, feeds=feeds, fetch=["y", "m"], device=dev)
    P.prepare()
    regions = [s for s in P._all_steps() if type(s).__name__ == "RegionStep"]
    P.execute()
    P.sync()
    for _ in range(3):
        P.execute()
    ms = time_events(tl, P.stream, P.execute, reps)
    hbm, _, _, src = peaks()
    gbs = FUSED_BYTES / (ms * 1e-3) / 1e9
    res = {"metric": "fused-op HBM GB/s (gelu(add(mult(x,s),b)) > 0, [8192,8192])",
           "value": gbs, "unit": "GB/s", "ms_per_launch": ms, "kernels": len(regions),
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                        "frac": gbs / hbm, "peak_source": src,
                        "traffic": None, "algorithmic_bytes": FUSED_BYTES}}
    P.free()
    return res


def build_training(tl, comm, dev, rank, world, epochs, bucket_mb=None, fuse_head=True,
                   fuse_colsum=True):
    """The benchmark program on this rank's shard, prepared, with its first
    iteration run eagerly; returns (program, loop, feeds, kernel launches per
    iteration)."""
    from tensor_lang_b200 import dp
    rt = tl.runtime
    b = B_GLOBAL // world
    pr = tl.programs
    ast = pr.mlp3_train(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, epochs=epochs)
    feeds = pr.mlp3_inputs(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, seed=0, rows=(rank * b, (rank + 1) * b))
    D = dp.DataParallelProgram(ast, None, comm, device=dev, feeds=feeds, fetch=["loss", "W3"],
                               bucket_bytes=None if not bucket_mb else int(bucket_mb * (1 << 20)),
                               fuse_head=fuse_head, fuse_colsum=fuse_colsum)
    P = D.program
    P.prepare()
    loop = P.loops[0]
    # first iteration eagerly (counts kernel launches), then capture the graph
    rt.launch_count(reset=True)
    loop.run_eager()
    n_eager = rt.launch_count(reset=True)
    loop.run_hoisted()  # hoisted steps run outside the per-iteration graph
    launches_per_step = n_eager - rt.launch_count()
    loop.capture()
    return P, loop, feeds, launches_per_step


def hidden_gemm(tl, P, M, scheme, check: bool):
    """The hidden-layer product a1[M,4096] @ W2 + b2 of the program, timed
    alone (CUDA events, 5 calls); with ``check``, the error of its result on
    one row per 128-row block and one column per 256-column block against a
    float64 evaluation of the same rows and columns, relative to max|ref|."""
    rt = tl.runtime
    L = rt.lib()
    N = K = D_H
    stream = P.stream
    args = (M, N, K, P.ptr("a1"), K, P.ptr("W2"), N, P.ptr("a2"), N)
    gemm = lambda: rt.check(L.tl_gemm(0, 0, *args, P.ptr("b2"), 0, 0, stream), "gemm")  # noqa: E731
    gemm()
    P.sync()
    ms = time_events(tl, stream, gemm, 5)
    on_tc = L.tl_gemm_path(0, 0, *args) == 0
    path = f"{GEMM_SCHEMES[scheme][1]}, CTA-pair 256x256 tiles" if on_tc else "CUDA-core fp32"
    plan = (ctypes.c_int * 4)()
    rt.check(L.tl_gemm_tc_plan(M, N, K, plan), "gemm plan")
    tflops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    _, bf16, _, src = peaks()
    ceiling = bf16 / GEMM_SCHEMES[scheme][2]
    res = {"bound": "tensor", "kernel": f"GEMM {M}x{N}x{K} ({path})",
           "achieved": tflops, "peak": bf16, "unit": "TFLOP/s", "frac": tflops / bf16,
           "peak_source": f"{src} bf16 dense (burst)",
           # captured for the one-GPU launch (65536 rows) only
           "traffic": GEMM_TRAFFIC_BYTES.get(scheme) if M == B_GLOBAL else None,
           "scheme_ceiling": ceiling, "frac_of_scheme_ceiling": tflops / ceiling,
           "ms_per_call": ms,
           "launch": {"k_splits": plan[1], "tiles_per_cluster": plan[2], "clusters": plan[3],
                      "schedule": {0: "single CTA", 1: "static", 2: "dynamic"}[plan[0]]}}
    if check:
        a1, C = P.read("a1"), P.read("a2")
        W2, b2 = P.read("W2").astype(np.float64), P.read("b2").astype(np.float64)
        rng = np.random.default_rng(0)
        rows = np.arange(0, M, 128) + rng.integers(0, 128, (M + 127) // 128)
        rows = np.minimum(rows, M - 1)
        cols = np.minimum(np.arange(0, N, 256) + rng.integers(0, 256, (N + 255) // 256), N - 1)
        rr = a1[rows].astype(np.float64) @ W2 + b2
        rc = np.empty((M, len(cols)))
        for r in range(0, M, 8192):
            rc[r:r + 8192] = a1[r:r + 8192].astype(np.float64) @ W2[:, cols] + b2[cols]
        scale = max(np.abs(rr).max(), np.abs(rc).max())
        err = max(np.abs(C[rows] - rr).max(), np.abs(C[:, cols] - rc).max())
        res["max_err_of_max_abs"] = float(err / scale)
        res["error_check"] = (f"{len(rows)} rows x {N} and {M} x {len(cols)} columns of the "
                              f"result against float64")
    return res


def allreduce_alone(tl, P, comm, rdv, calls=10):
    """The gradient arena's all-reduce timed alone on the communication stream
    (CUDA events, max over ranks, after 3 untimed calls): bytes, ms and bus
    bandwidth (2 (n-1)/n of the bytes cross each GPU's links each way).  It
    sums into the gradients, so it runs after the timed steps."""
    rt = tl.runtime
    L = rt.lib()
    names = P.arena_names
    p0 = P.ptr(names[0])
    count = (P.ptr(names[-1]) - p0) // 4 + int(np.prod(P.shapes[names[-1]]))
    call = lambda: rt.check(L.tl_nccl_allreduce_sum(comm.handle, p0, count, comm.stream),  # noqa: E731
                            "allreduce")
    for _ in range(3):
        call()
    rt.check(L.tl_stream_sync(comm.stream), "sync")
    rdv.barrier()
    ms = time_events(tl, comm.stream, call, calls)
    every = rdv.gather(ms)
    ms = max(every) if every else 0.0
    n = comm.world
    nbytes = 4 * count
    bus = nbytes * 2 * (n - 1) / n / (ms * 1e-3) / 1e9 if ms else 0.0
    return {"bytes": nbytes, "ms": ms, "busbw_gbs": bus, "calls": calls,
            "note": "NCCL ring/tree over NVLink, NVLS off; timed alone, not overlapped"}


def time_training(tl, loop, stream, steps, clocks=None):
    def timed_step():
        loop.replay(1)
        if clocks is not None:
            clocks.sample()  # host-side sample while the step runs on the device
    return time_events(tl, stream, timed_step, steps)


def gpu_configs(tl, dev):
    """The other workloads on this GPU (CUDA events on the program's stream,
    after 3 untimed runs): the 2-layer training step, the reductions and
    normalisations of [16384,4096], one forward + backward of the linear layer."""
    rt = tl.runtime
    pr = tl.programs
    hbm, _, _, src = peaks()
    out = {}
    P = tl.Program(pr.mlp2_step(), None, feeds=pr.mlp2_inputs(seed=0),
                   fetch=["loss", "W1_new", "b1_new", "W2_new", "b2_new"], device=dev)
    P.prepare()
    for _ in range(3):
        P.execute()
    ms = time_events(tl, P.stream, P.execute, 50)
    out["mlp2_step_64x128"] = {"us_per_step": ms * 1e3, "launches": len(P._all_steps()),
                               "note": "one launch per step from the host, no graph: launch-bound"}
    P.free()
    R, C_ = 16384, 4096
    P = tl.Program(pr.reductions(R, C_), None, feeds=pr.reductions_inputs(R, C_),
                   fetch=[n for n, _, _ in pr.REDUCTION_OPS] + ["sm", "ln"], device=dev)
    P.prepare()
    ops = {}
    for s in P._all_steps():
        call = s.bind(P)
        for _ in range(3):
            call()
        P.sync()
        t = time_events(tl, P.stream, call, 20)
        two_way = s.label.split(":")[0] in ("softmax", "layer_norm_2d")
        gbs = 4.0 * R * C_ * (2 if two_way else 1) / (t * 1e-3) / 1e9
        ops[s.label] = {"GB/s": gbs, "frac": gbs / hbm}
    P.free()
    fr = [v["frac"] for v in ops.values()]
    out["reductions_16384x4096"] = {"ops": ops, "frac_min": min(fr), "frac_max": max(fr),
                                    "peak": hbm, "peak_source": src}
    M, K, N = C4_SHAPE
    P = tl.Program(pr.linear_layer(M, K, N), None, feeds=pr.linear_layer_inputs(M, K, N, seed=0),
                   fetch=["loss", "W_grad", "b_grad", "X_grad"], device=dev)
    P.prepare()
    for _ in range(3):
        P.execute()
    ms = time_events(tl, P.stream, P.execute, 5)
    out["linear_layer_8192x4096x4096"] = {"ms": ms, "TFLOP/s": C4_FLOP / (ms * 1e-3) / 1e12,
                                          "work": "forward, relu, mse, dW, db, dX"}
    P.free()
    return out


FIRST_RUN = r"""
import json, sys, time
t0 = time.perf_counter()
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import load_package
tl = load_package()
tl.load_library()
t1 = time.perf_counter()
pr = tl.programs
P = tl.Program(pr.mlp2_step(), None, feeds=pr.mlp2_inputs(seed=0), fetch=["loss"])
P.run()
t2 = time.perf_counter()
Q = tl.Program(pr.mlp2_step(), None, feeds=pr.mlp2_inputs(seed=1), fetch=["loss"])
Q.run()
t3 = time.perf_counter()
print(json.dumps({"load_s": t1 - t0, "first_program_s": t2 - t1, "second_program_s": t3 - t2}))
"""


def first_run_latency():
    """Wall time from process start to the first result of the 2-layer training
    step program, in fresh processes: cold (empty fused-region cubin cache, so
    every region is compiled by NVRTC) and warm (the cubins on disk)."""
    import tempfile
    out = {}
    with tempfile.TemporaryDirectory(prefix="tl_jit_") as jit:
        env = dict(os.environ, TL_JIT_DIR=jit)
        for kind in ("cold", "warm"):
            t0 = time.perf_counter()
            r = subprocess.run([sys.executable, "-c", FIRST_RUN, str(REPO)], env=env,
                               capture_output=True, text=True, timeout=300)
            wall = time.perf_counter() - t0
            if r.returncode != 0:
                raise RuntimeError(f"first-run probe failed: {r.stderr[-2000:]}")
            rec = json.loads(r.stdout.strip().splitlines()[-1])
            rec["process_wall_s"] = wall
            out[kind] = rec
    out["program"] = "2-layer MLP training step [64,128] (parse-free: AST built in Python)"
    return out


def contract_scheme(tl, comm, dev, args):
    """The same step with the GEMMs in the split-TF32 scheme (TF32 hi*hi plus
    one bf16 pair MMA for the corrections): steps/s and the hidden GEMM."""
    set_gemm_scheme(tl, "tf32bf16")
    try:
        P, loop, _, _ = build_training(tl, comm, dev, 0, 1, epochs=1 + 3 + 10)
        for _ in range(3):
            loop.replay(1)
        P.sync()
        ms = time_training(tl, loop, P.stream, 10)
        g = hidden_gemm(tl, P, B_GLOBAL, "tf32bf16", check=True)
        P.free()
    finally:
        set_gemm_scheme(tl, args.gemm_scheme)
    return {"gemm": GEMM_SCHEMES["tf32bf16"][1], "value": 1000.0 / ms, "unit": "steps/s",
            "ms_per_step": ms, "steps": 10, "warmup": 3, "roofline": g}


def run_ours(args, rank, world, local):
    from __graft_entry__ import load_package
    tl = load_package()
    rt = tl.runtime
    set_gemm_scheme(tl, args.gemm_scheme)
    set_tile_schedule(tl, args.tile_schedule)
    set_store_path(tl, args.store_path)
    from tensor_lang_b200 import dp

    dev = local
    rt.Device.get(dev)
    addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("TL_RDV_PORT", str(int(os.environ.get("MASTER_PORT", "29500")) + 17)))
    rdv = dp.Rendezvous(rank, world, addr, port)
    comm = dp.Communicator(rdv)

    b = B_GLOBAL // world
    P, loop, feeds, launches_per_step = build_training(tl, comm, dev, rank, world,
                                                       epochs=1 + args.warmup + args.steps,
                                                       bucket_mb=args.bucket_mb,
                                                       fuse_head=not args.no_head_fusion,
                                                       fuse_colsum=not args.no_colsum_fusion)
    stream = P.stream
    for _ in range(args.warmup):
        loop.replay(1)
    comm.wait(stream)
    P.sync()

    clocks = Clocks(dev)
    rdv.barrier()
    clocks.start()
    ms = time_training(tl, loop, stream, args.steps, clocks)
    clk = clocks.stop()
    rdv.barrier()
    all_ms = rdv.gather(ms)

    # e2e through the public API: every step's batch comes from pinned host
    # memory and every step's loss goes back to the host
    xs, ts = feeds["x"], feeds["t"]
    # as many steps as the device-timed region: the first batch's upload is
    # the one that overlaps nothing
    e2e_steps = max(1, args.steps)
    e2e_ms = e2e_time(tl, rt.Device.get(dev), loop, stream, P.ptr("x"), P.ptr("t"), P.ptr("loss"),
                      xs, ts, e2e_steps)
    rdv.barrier()
    all_e2e = rdv.gather(e2e_ms)
    loss = float(P.read("loss").reshape(-1)[0])
    graph_nodes = loop.graph_nodes
    ar = allreduce_alone(tl, P, comm, rdv) if world > 1 else None

    # dominant kernel: the hidden-layer GEMM (b x 4096 x 4096), timed alone
    roof = hidden_gemm(tl, P, b, args.gemm_scheme, check=(rank == 0 and not args.no_check))
    P.free()

    extra = {}
    if world == 1 and not args.no_configs:
        extra["contract_scheme"] = contract_scheme(tl, comm, dev, args)
        extra["fused_op"] = fused_op_bench(tl, dev)
        extra["configs"] = gpu_configs(tl, dev)
        extra["first_run"] = first_run_latency()

    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            t = cpu_mlp_step_times(1, 0)[0]
            cpu = {"value": 1.0 / t, "unit": "steps/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"one full-batch ({B_GLOBAL}-row) training step of the float32 NumPy "
                             f"oracle ({t:.2f} s)"}
        ms_max = max(all_ms)
        scheme = GEMM_SCHEMES[args.gemm_scheme]
        line = {
            "metric": METRIC,
            "value": 1000.0 / ms_max, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": f"f32 ({args.gemm_scheme} split GEMMs)", "data": "synthetic",
            "config": {"workload": "mlp3_dp_train", "global_batch": B_GLOBAL,
                       "per_gpu_batch": b, "dims": [D_IN, D_H, D_H, N_CLS],
                       "parallelism": f"dp{world}", "gemm": f"{scheme[1]}, CTA-pair 256x256 tiles",
                       "gradient_allreduce": ("none (one GPU)" if world == 1 else
                                              f"buckets of {args.bucket_mb:g} MiB as backward "
                                              "finalises them" if args.bucket_mb
                                              else "one, after backward"),
                       "l2": "inputs larger than L2 (no flush)"},
            "model_tflops": FLOP_PER_STEP / (ms_max * 1e-3) / 1e12,
            "loss_rank0": loss,
            # the GEMM call (bf16 pair pre-passes + tcgen05 kernel), fp32-equivalent
            # flops; per fp32 product BF16X3 issues three bf16 products (ceiling
            # bf16 / 3), TF32+bf16 one TF32 product at half the bf16 rate and two
            # bf16 products (bf16 / 4)
            "roofline": roof,
            "e2e": {"value": 1000.0 / max(all_e2e), "unit": "steps/s",
                    "h2d_bytes_per_step": int(xs.nbytes + ts.nbytes) * world,
                    "d2h_bytes_per_step": 4 * world},
            "gpu_launches": int(launches_per_step * args.steps),
            "graph": {"kernel_nodes": graph_nodes[0], "prioritised": graph_nodes[1],
                      "allreduce_buckets": sum(1 for s in P._all_steps()
                                               if type(s).__name__ == "AllReduceBucket")},
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if ar is not None:
            line["allreduce"] = ar
        line.update(extra)
        print(json.dumps(line), flush=True)
    comm.destroy()
    rdv.close()
    return 0


def run_micro(args):
    """One kernel alone, for profiling and per-kernel rooflines:
    gemm        M x 4096 x 4096 linear forward (--gemm-m, default 8192:
                A 128 MiB, B 64 MiB; 65536 is the training step's hidden GEMM)
    fused       the [8192,8192] fused elementwise chain
    softmax     softmax over rows of [16384,4096]
    rowsum      sum over rows of [16384,4096]
    reductions  every reduction / normalisation of the [16384,4096] workload,
                one JSON line each (the tensor is x ~ N(0,1); arg-reductions
                read copies with 1% tied extremes per line)
    """
    from __graft_entry__ import load_package
    tl = load_package()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    st = dev.stream
    set_gemm_scheme(tl, args.gemm_scheme)
    set_tile_schedule(tl, args.tile_schedule)
    set_store_path(tl, args.store_path)
    hbm, bf16, _, src = peaks()
    reps = args.steps
    if args.micro == "reductions":
        pr = tl.programs
        R, C_ = 16384, 4096
        P = tl.Program(pr.reductions(R, C_), None, feeds=pr.reductions_inputs(R, C_),
                       fetch=[n for n, _, _ in pr.REDUCTION_OPS] + ["sm", "ln"])
        P.prepare()
        for s in P._all_steps():
            call = s.bind(P)
            for _ in range(max(3, args.warmup)):
                call()
            P.sync()
            ms = time_events(tl, st, call, reps)
            two_way = s.label.split(":")[0] in ("softmax", "layer_norm_2d")
            nbytes = 4.0 * R * C_ * (2 if two_way else 1)
            ach = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({"micro": "reductions", "op": s.label, "ms_per_launch": ms,
                              "achieved": ach, "unit": "GB/s", "peak": hbm, "frac": ach / hbm,
                              "peak_source": src, "launches": reps}), flush=True)
        P.free()
        return 0
    if args.micro == "gemm":
        M, N, K = args.gemm_m, 4096, args.gemm_k
        rng = np.random.default_rng(0)
        A = rt.DeviceBuffer(dev, (M, K))
        A.upload(rng.standard_normal((M, K), dtype=np.float32))
        B = rt.DeviceBuffer(dev, (K, N))
        B.upload((rng.standard_normal((K, N), dtype=np.float32) / 64).astype(np.float32))
        C = rt.DeviceBuffer(dev, (M, N))
        bias = rt.DeviceBuffer(dev, (N,), zero=True)
        fn = lambda: rt.check(L.tl_gemm(0, 0, M, N, K, A.ptr, K, B.ptr, N, C.ptr, N, bias.ptr, 0, 0, st))  # noqa: E731
        work, unit, peak = 2.0 * M * N * K, "TFLOP/s", bf16
    elif args.micro == "fused":
        pr = tl.programs
        P = tl.Program(pr.fused_chain(FUSED_N), None, feeds=pr.fused_chain_inputs(FUSED_N), fetch=["y", "m"])
        P.prepare()
        fn = P.execute
        work, unit, peak = float(FUSED_BYTES), "GB/s", hbm
    else:
        R, C_ = 16384, 4096
        x = rt.DeviceBuffer(dev, (R, C_))
        x.upload(np.random.default_rng(1).standard_normal((R, C_), dtype=np.float32))
        y = rt.DeviceBuffer(dev, (R, C_) if args.micro == "softmax" else (R,))
        if args.micro == "softmax":
            fn = lambda: rt.check(L.tl_softmax_rows(x.ptr, y.ptr, R, C_, st))  # noqa: E731
            work = 8.0 * R * C_
        else:
            fn = lambda: rt.check(L.tl_reduce_rows(0, x.ptr, y.ptr, R, C_, st))  # noqa: E731
            work = 4.0 * R * C_ + 4.0 * R
        unit, peak = "GB/s", hbm
    for _ in range(max(3, args.warmup)):
        fn()
    dev.sync()
    ms = time_events(tl, st, fn, reps)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    ach = work / (ms * 1e-3) / scale
    print(json.dumps({"micro": args.micro, "ms_per_launch": ms, "achieved": ach, "unit": unit,
                      "peak": peak, "frac": ach / peak, "peak_source": src, "launches": reps}),
          flush=True)
    return 0


def main():
    global B_GLOBAL, METRIC
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="no CPU baseline step")
    ap.add_argument("--no-configs", action="store_true",
                    help="one GPU: skip the split-TF32 step and the other workloads")
    ap.add_argument("--no-cpu-configs", action="store_true",
                    help="--impl reference: skip the other workloads")
    ap.add_argument("--no-check", action="store_true", help="skip the GEMM error check")
    ap.add_argument("--no-colsum-fusion", action="store_true",
                    help="keep each bias gradient's column sum as its own pass over dY instead "
                         "of folding it into the pair step of dY")
    ap.add_argument("--no-head-fusion", action="store_true",
                    help="profiling aid: run the classifier head unfused")
    ap.add_argument("--bucket-mb", type=float, default=64,
                    help="data parallel: all-reduce gradients in buckets of this many MiB as "
                         "backward finalises them (0: one all-reduce after backward)")
    ap.add_argument("--gemm-m", type=int, default=8192, help="rows of the --micro gemm product")
    ap.add_argument("--gemm-k", type=int, default=4096, help="depth of the --micro gemm product")
    ap.add_argument("--global-batch", type=int, default=B_GLOBAL,
                    help="profiling aid: another global batch (8192 at one GPU is the per-rank "
                         "work of eight)")
    ap.add_argument("--gemm-scheme", choices=sorted(GEMM_SCHEMES), default="bf16x3",
                    help="tensor-core operand scheme of the fp32 GEMMs")
    ap.add_argument("--store-path", choices=("tma", "rows"), default="tma",
                    help="CTA-pair GEMM epilogue: TMA stores of staged 32x32 slabs, or each "
                         "lane storing its own row")
    ap.add_argument("--tile-schedule", choices=sorted(TILE_SCHEDULES), default="auto",
                    help="CTA-pair GEMM tile schedule: static groups, dynamic (running "
                         "clusters take pending clusters' tiles), or auto (the library's choice "
                         "per launch)")
    ap.add_argument("--micro", choices=["gemm", "fused", "softmax", "rowsum", "reductions"],
                    default=None,
                    help="time one kernel alone (profiling aid); prints its own JSON line")
    args = ap.parse_args()
    if args.global_batch != B_GLOBAL:
        B_GLOBAL = args.global_batch
        METRIC = METRIC.replace("batch 65536", f"batch {B_GLOBAL}")
    if args.micro:
        return run_micro(args)
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
