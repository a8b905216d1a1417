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

def cpu_mlp_step_time(rows: int, reps: int = 1):
    from oracle import OracleProgram
    from __graft_entry__ import load_package
    tl = load_package()
    pr = tl.programs
    ast = pr.mlp3_train(B=rows, I=D_IN, H=D_H, C=N_CLS, epochs=1)
    feeds = pr.mlp3_inputs(B=rows, I=D_IN, H=D_H, C=N_CLS, seed=0)
    env = {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        OracleProgram(ast, env, dtype=np.float32, feeds=feeds).run()
        times.append(time.perf_counter() - t0)
    return min(times)


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    rows = args.cpu_rows
    cores = os.cpu_count() or 1
    for _ in range(max(1, args.warmup)):
        cpu_mlp_step_time(rows)
    samples = [cpu_mlp_step_time(rows) for _ in range(max(1, args.steps))]
    t = float(np.mean(samples)) * (B_GLOBAL / rows)  # seconds per full-batch step
    value = 1.0 / t
    line = {
        "impl": "reference", "metric": "MLP train steps/sec (3-layer 1024-4096-4096-10, batch 65536)",
        "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1000.0, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "mlp3_dp_train", "global_batch": B_GLOBAL, "dims": [D_IN, D_H, D_H, N_CLS],
                   "parallelism": "host numpy", "l2": "inputs larger than L2"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": f"one training step on {rows} of the {B_GLOBAL} rows, "
                                   f"scaled x{B_GLOBAL // rows}; mean of {len(samples)}"},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
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


def run_ours(args, rank, world, local):
    from __graft_entry__ import load_package
    tl = load_package()
    rt = tl.runtime
    set_gemm_scheme(tl, args.gemm_scheme)
    from tensor_lang_b200 import dp

    dev = local
    rt.Device.get(dev)
    addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("TL_RDV_PORT", str(int(os.environ.get("MASTER_PORT", "29500")) + 17)))
    rdv = dp.Rendezvous(rank, world, addr, port)
    comm = dp.Communicator(rdv)

    b = B_GLOBAL // world
    r0, r1 = rank * b, (rank + 1) * b
    pr = tl.programs
    ast = pr.mlp3_train(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, epochs=1 + args.warmup + args.steps)
    feeds = pr.mlp3_inputs(B=B_GLOBAL, I=D_IN, H=D_H, C=N_CLS, seed=0, rows=(r0, r1))
    D = dp.DataParallelProgram(ast, None, comm, device=dev, feeds=feeds, fetch=["loss", "W3"])
    P = D.program
    P.prepare()
    loop = P.loops[0]
    stream = P.stream

    # first iteration eagerly (counts kernel launches), then capture the graph
    rt.launch_count(reset=True)
    loop.run_eager()
    n_eager = rt.launch_count(reset=True)
    loop.run_hoisted()  # hoisted steps run outside the per-iteration graph
    launches_per_step = n_eager - rt.launch_count()
    loop.capture()
    for _ in range(args.warmup):
        loop.replay(1)
    comm.wait(stream)
    P.sync()

    clocks = Clocks(dev)
    rdv.barrier()
    clocks.start()

    def timed_step():
        loop.replay(1)
        clocks.sample()  # host-side sample while the step runs on the device

    ms = time_events(tl, stream, timed_step, args.steps)
    clk = clocks.stop()
    rdv.barrier()
    all_ms = rdv.gather(ms)

    # e2e through the public API: every step's batch comes from pinned host
    # memory and every step's loss goes back to the host
    xs, ts = feeds["x"], feeds["t"]
    L = rt.lib()
    e2e_steps = max(1, min(args.steps, 10))
    e2e_ms = e2e_time(tl, rt.Device.get(dev), loop, stream, P.ptr("x"), P.ptr("t"), P.ptr("loss"),
                      xs, ts, e2e_steps)
    rdv.barrier()
    all_e2e = rdv.gather(e2e_ms)

    # dominant kernel: the hidden-layer GEMM (b x 4096 x 4096), timed alone
    M, N, K = b, D_H, D_H
    gemm = lambda: rt.check(L.tl_gemm(0, 0, M, N, K, P.ptr("a1"), K, P.ptr("W2"), N, P.ptr("a2"),  # noqa: E731
                                       N, P.ptr("b2"), 0, 0, stream), "gemm")
    gemm()
    P.sync()
    g_ms = time_events(tl, stream, gemm, 5)
    on_tc = L.tl_gemm_path(0, 0, M, N, K, P.ptr("a1"), K, P.ptr("W2"), N, P.ptr("a2"), N) == 0
    path = (f"{GEMM_SCHEMES[args.gemm_scheme][1]}, CTA-pair 256x256 tiles"
            if on_tc else "CUDA-core fp32")
    plan = (ctypes.c_int * 4)()
    rt.check(L.tl_gemm_tc_plan(M, N, K, plan), "gemm plan")
    gemm_plan = {"k_splits": plan[1], "tiles_per_cluster": plan[2], "clusters": plan[3]}
    loss = float(P.read("loss").reshape(-1)[0])

    fused = None
    if world == 1 and not args.no_fused:
        fused = fused_op_bench(tl, dev)

    if rank == 0:
        cpu = None
        if not args.no_cpu:
            rows = args.cpu_rows
            t = cpu_mlp_step_time(rows) * (B_GLOBAL / rows)
            cpu = {"value": 1.0 / t, "unit": "steps/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"float32 NumPy oracle: one training step on {rows} of {B_GLOBAL} rows, "
                             f"scaled x{B_GLOBAL // rows}"}
        ms_max = max(all_ms)
        hbm, bf16, bf16s, src = peaks()
        ceiling = bf16 / GEMM_SCHEMES[args.gemm_scheme][2]
        tflops = 2.0 * M * N * K / (g_ms * 1e-3) / 1e12
        line = {
            "metric": "MLP train steps/sec (3-layer 1024-4096-4096-10, batch 65536)",
            "value": 1000.0 / ms_max, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "mlp3_dp_train", "global_batch": B_GLOBAL,
                       "per_gpu_batch": b, "dims": [D_IN, D_H, D_H, N_CLS],
                       "parallelism": f"dp{world}", "gemm": path,
                       "l2": "inputs larger than L2 (no flush)"},
            "model_tflops": FLOP_PER_STEP / (ms_max * 1e-3) / 1e12,
            "loss_rank0": loss,
            # the GEMM call (bf16 pair pre-passes + tcgen05 kernel), fp32-equivalent
            # flops; per fp32 product BF16X3 issues three bf16 products (ceiling
            # bf16 / 3), TF32+bf16 one TF32 product at half the bf16 rate and two
            # bf16 products (bf16 / 4)
            "roofline": {"bound": "tensor", "kernel": f"GEMM {M}x{N}x{K} ({path})",
                         "achieved": tflops, "peak": bf16, "unit": "TFLOP/s",
                         "frac": tflops / bf16, "peak_source": f"{src} bf16 dense (burst)",
                         # captured for the one-GPU launch (65536 rows) only
                         "traffic": GEMM_TRAFFIC_BYTES.get(args.gemm_scheme) if M == B_GLOBAL else None,
                         "scheme_ceiling": ceiling,
                         "frac_of_scheme_ceiling": tflops / ceiling,
                         "launch": gemm_plan},
            "e2e": {"value": 1000.0 / max(all_e2e), "unit": "steps/s",
                    "h2d_bytes_per_step": int(xs.nbytes + ts.nbytes) * world,
                    "d2h_bytes_per_step": 4 * world},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if fused is not None:
            line["fused_op"] = fused
        print(json.dumps(line), flush=True)
    P.free()
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
        M, N, K = args.gemm_m, 4096, 4096
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
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=4096)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-fused", action="store_true")
    ap.add_argument("--gemm-m", type=int, default=8192, help="rows of the --micro gemm product")
    ap.add_argument("--gemm-scheme", choices=sorted(GEMM_SCHEMES), default="bf16x3",
                    help="tensor-core operand scheme of the fp32 GEMMs")
    ap.add_argument("--micro", choices=["gemm", "fused", "softmax", "rowsum", "reductions"],
                    default=None,
                    help="time one kernel alone (profiling aid); prints its own JSON line")
    args = ap.parse_args()
    if args.micro:
        return run_micro(args)
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
