"""Generate the golden fixtures that pin the oracle and the GPU backend.

Run here (where the TensorLang reference checkout is readable), never on the
GPU host:

    python tests/golden/make_golden.py --reference <checkout of the reference>

What it produces (all small JSON, committed):

* ``ref_programs.json`` -- for every ``tests/*.tl`` program of the reference:
  the AST emitted by the reference frontend (``ast_builder.build_ast``), the
  type environment from ``type_checker.type_checker``, the ``// @EXPECTED``
  block, and every tensor the reference's own executor
  (``TensorCompiler.compile_and_execute``, ``tensorlang/compiler.py:858``)
  wrote to its ``--cache-layers`` directory.

  The reference executes through PyCUDA on a GPU.  Neither exists here, so the
  reference's compiler, autograd and ``for``-loop executor run UNMODIFIED
  with two stand-ins installed underneath them:
    - a ``pycuda`` module whose ``mem_alloc``/``memcpy_htod``/``memcpy_dtoh``
      are byte buffers in host memory;
    - a ``ctypes.cdll.LoadLibrary`` that returns an emulator of the generated
      ``launch_<op>_<name>`` entry points.  Each launcher is emulated in
      float32 NumPy from the CUDA that ``tensorlang/kernel_generator.py``
      emits for it (cited per family below), using the ``kernel_info``
      tuple the reference's generator returned for that tensor.
  nvcc is not invoked (the generated ``kernel.cu`` is still written).
  Launchers whose generated CUDA has undefined behaviour (the full
  ``argmax`` kernel with aliased shared arrays, kernel_generator.py:1464-1467;
  ``equal`` with a broadcast operand, whose launcher receives one fewer
  argument than it declares, compiler.py:450-457) are recorded as such.

* ``kinfo_cases.json`` -- ``(method, args) -> kernel_info`` pairs returned by
  the reference ``KernelGenerator`` for a spread of shapes, to check the
  drop-in generator returns identical dispatch tuples.

* ``autograd_cases.json`` -- gradients computed by the reference's own
  ``autograd.ComputationGraph`` on seeded inputs, per VJP rule, to pin the
  oracle's restatement of ``tensorlang/autograd.py``.
"""
from __future__ import annotations

import argparse
import contextlib
import ctypes
import glob
import io
import json
import os
import re
import subprocess
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
# working directory of one run (a fresh temporary directory, set by
# run_reference_programs): the reference writes its kernel.cu and cache there
SCRATCH: Path = Path()


# ---------------------------------------------------------------------------
# JSON helpers
# ---------------------------------------------------------------------------

def strip_ast(obj):
    """Drop lark parse trees and turn tuples into lists so the AST is JSON."""
    if isinstance(obj, dict):
        return {k: strip_ast(v) for k, v in obj.items() if k != "tree"}
    if isinstance(obj, (list, tuple)):
        return [strip_ast(v) for v in obj]
    if isinstance(obj, (np.integer,)):
        return int(obj)
    if isinstance(obj, (np.floating,)):
        return float(obj)
    return obj


def arr_to_json(a):
    a = np.asarray(a)
    return {"shape": list(a.shape), "data": [float(v) for v in a.reshape(-1).tolist()]}


# ---------------------------------------------------------------------------
# Host-memory stand-in for pycuda.driver
# ---------------------------------------------------------------------------

class _Mem:
    """Flat byte store addressed by fake device pointers."""

    def __init__(self):
        self.bufs = {}
        self.next = 1 << 20

    def alloc(self, nbytes):
        addr = self.next
        self.next += max(256, (int(nbytes) + 255) // 256 * 256)
        self.bufs[addr] = bytearray(max(int(nbytes), 4))
        return addr

    def view(self, addr, count=None):
        buf = self.bufs[int(addr)]
        arr = np.frombuffer(buf, dtype=np.float32)
        return arr if count is None else arr[:count]


MEM = _Mem()


class _DeviceAllocation:
    def __init__(self, nbytes):
        self.addr = MEM.alloc(nbytes)

    def __int__(self):
        return self.addr

    def free(self):
        MEM.bufs.pop(self.addr, None)


def _memcpy_htod(dst, src):
    src = np.ascontiguousarray(src)
    raw = src.tobytes()
    buf = MEM.bufs[int(dst)]
    n = min(len(raw), len(buf))
    buf[:n] = raw[:n]


def _memcpy_dtoh(dst, src):
    buf = MEM.bufs[int(src)]
    raw = np.frombuffer(buf, dtype=np.uint8)
    flat = dst.reshape(-1).view(np.uint8)
    n = min(flat.size, raw.size)
    flat[:n] = raw[:n]


def install_fake_pycuda():
    pycuda = types.ModuleType("pycuda")
    driver = types.ModuleType("pycuda.driver")
    driver.mem_alloc = lambda n: _DeviceAllocation(n)
    driver.memcpy_htod = _memcpy_htod
    driver.memcpy_dtoh = _memcpy_dtoh
    autoinit = types.ModuleType("pycuda.autoinit")
    pycuda.driver = driver
    pycuda.autoinit = autoinit
    sys.modules["pycuda"] = pycuda
    sys.modules["pycuda.driver"] = driver
    sys.modules["pycuda.autoinit"] = autoinit


# ---------------------------------------------------------------------------
# float32 emulation of the generated launchers
# ---------------------------------------------------------------------------

class UndefinedBehaviour(Exception):
    pass


F32 = np.float32
_OPS = {"add": np.add, "minus": np.subtract, "mult": np.multiply, "div": np.divide}


def _seq_sum(v):
    """Sequential float32 accumulation, as the one-thread-per-row loops do."""
    acc = F32(0.0)
    for x in np.asarray(v, dtype=F32).reshape(-1):
        acc = F32(acc + x)
    return acc


class KernelEmulator:
    """Replaces the ctypes handle of the generated kernel.so."""

    def __init__(self, kinfos):
        self.kinfos = kinfos  # tensor name -> kernel_info

    def _lookup(self, symbol):
        best = None
        for name in self.kinfos:
            if symbol.endswith("_" + name) and symbol.startswith("launch_"):
                if best is None or len(name) > len(best):
                    best = name
        if best is None:
            raise KeyError(symbol)
        return best

    def __getattr__(self, symbol):
        if not symbol.startswith("launch_"):
            raise AttributeError(symbol)
        name = self._lookup(symbol)
        kinfo = self.kinfos[name]

        def launcher(*args):
            vals = [a.value if hasattr(a, "value") else a for a in args]
            emulate(kinfo, vals)

        return launcher


def _p(v):
    return int(v)


def emulate(k, a):
    """Run one launcher.  ``k`` is its kernel_info, ``a`` the ctypes values."""
    kind = k[0]
    if kind == "general_broadcast":
        # kernel_generator.py:383-463 (compute_broadcast_index :408-428)
        op = k[1]
        s1, s2, out = [int(d) for d in k[5]], [int(d) for d in k[6]], [int(d) for d in k[7]]
        total = int(k[8])
        A = MEM.view(a[0], int(np.prod(s1))).reshape(s1)
        B = MEM.view(a[1], int(np.prod(s2))).reshape(s2)
        C = MEM.view(a[2], total)
        C[:] = _OPS[op](np.broadcast_to(A, out), np.broadcast_to(B, out)).astype(F32).reshape(-1)
        return
    if kind in ("add", "minus", "mult", "div"):  # :246-275
        n = a[3]
        MEM.view(a[2], n)[:] = _OPS[kind](MEM.view(a[0], n), MEM.view(a[1], n))
        return
    if kind.endswith("_scalar"):  # :354-377
        n = a[3]
        MEM.view(a[2], n)[:] = _OPS[kind.split("_")[0]](MEM.view(a[0], n), MEM.view(a[1], 1)[0])
        return
    if kind.endswith("_broadcast_rows") or kind in (
            "add_broadcast", "minus_broadcast", "mult_broadcast", "div_broadcast"):
        # :281-348 -- B[i] when shape1[0]==shape2[0] (rows variant) else B[j]
        rows, cols = a[3], a[4]
        A = MEM.view(a[0], rows * cols).reshape(rows, cols)
        if kind.endswith("_rows"):
            B = MEM.view(a[1], rows).reshape(rows, 1)
        else:
            B = MEM.view(a[1], cols).reshape(1, cols)
        MEM.view(a[2], rows * cols)[:] = _OPS[kind.split("_")[0]](A, B).reshape(-1)
        return
    if kind == "fill":  # :469-488
        MEM.view(a[0], a[2])[:] = F32(a[1])
        return
    if kind == "matmul":  # :501-525, one thread per output, sequential K loop
        m, n, p = a[3], a[4], a[5]
        A = MEM.view(a[0], m * n).reshape(m, n).astype(F32)
        Bv = MEM.view(a[1])
        if Bv.size < n * p:
            raise UndefinedBehaviour("matmul reads B past its allocation")
        B = Bv[: n * p].reshape(n, p)
        C = np.zeros((m, p), dtype=F32)
        for kk in range(n):
            C = (C + np.outer(A[:, kk], B[kk, :]).astype(F32)).astype(F32)
        out = MEM.view(a[2])
        if out.size < m * p:
            raise UndefinedBehaviour("matmul writes C past its allocation")
        out[: m * p] = C.reshape(-1)
        return
    if kind in ("relu", "sigmoid", "tanh"):  # :209-240, :531-558
        n = a[2]
        x = MEM.view(a[0], n)
        if kind == "relu":
            y = np.maximum(F32(0.0), x)
        elif kind == "sigmoid":
            y = F32(1.0) / (F32(1.0) + np.exp(-x))
        else:
            y = np.tanh(x)
        MEM.view(a[1], n)[:] = y.astype(F32)
        return
    if kind in ("softmax", "softmax_1d"):  # :564-640, three sequential passes per row
        if kind == "softmax":
            rows, cols = a[2], a[3]
        else:
            rows, cols = 1, a[2]
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        Y = np.empty_like(X)
        for r in range(rows):
            mx = X[r].max()
            e = np.exp((X[r] - mx).astype(F32)).astype(F32)
            s = _seq_sum(e)
            Y[r] = (e / s).astype(F32)
        MEM.view(a[1], rows * cols)[:] = Y.reshape(-1)
        return
    if kind in ("greater", "less", "equal"):
        if len(k) == 6 and kind == "equal":
            # equal with a broadcast operand: compiler.py:450-457 passes one int
            # to a launcher declared with (rows, cols) -> undefined cols.
            raise UndefinedBehaviour("equal broadcast launcher argument mismatch")
        n = a[3]
        A, B = MEM.view(a[0], n), MEM.view(a[1], n)
        if kind == "greater":
            c = A > B
        elif kind == "less":
            c = A < B
        else:
            c = np.abs((A - B).astype(F32)) < F32(1e-6)
        MEM.view(a[2], n)[:] = c.astype(F32)
        return
    if kind in ("greater_broadcast", "less_broadcast"):  # :646-732, always B[j]
        rows, cols = a[3], a[4]
        A = MEM.view(a[0], rows * cols).reshape(rows, cols)
        B = MEM.view(a[1])[:cols].reshape(1, cols)
        c = A > B if kind.startswith("greater") else A < B
        MEM.view(a[2], rows * cols)[:] = c.astype(F32).reshape(-1)
        return
    if kind in ("sum_full", "mean_full"):  # :784-826, :888-936
        n = a[2]
        s = F32(np.sum(MEM.view(a[0], n), dtype=F32))
        if kind == "mean_full":
            s = F32(s / F32(n))
        MEM.view(a[1], 1)[0] = s
        return
    if kind in ("sum_axis", "sum_axis0", "mean_axis", "mean_axis0",
                "max_axis", "max_axis0", "min_axis", "min_axis0"):
        rows, cols = a[2], a[3]
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        op = kind.split("_")[0]
        ax = 0 if kind.endswith("axis0") else 1
        if op in ("sum", "mean"):
            lines = X.T if ax == 0 else X
            r = np.array([_seq_sum(v) for v in lines], dtype=F32)
            if op == "mean":
                r = (r / F32(X.shape[ax])).astype(F32)
        elif op == "max":
            r = X.max(axis=ax)
        else:
            r = X.min(axis=ax)
        MEM.view(a[1], r.size)[:] = r
        return
    if kind in ("max_full", "min_full"):  # :1246-1294 (atomicCAS fmaxf), :1352-1401
        n = a[2]
        X = MEM.view(a[0], n)
        MEM.view(a[1], 1)[0] = X.max() if kind == "max_full" else X.min()
        return
    if kind in ("argmax_axis", "argmax_full", "argmin_axis"):
        if len(k) == 5:
            # full argmax: grid(1) kernel whose float and int shared arrays
            # alias (kernel_generator.py:1464-1501)
            raise UndefinedBehaviour("full argmax kernel aliases its shared arrays")
        rows, cols = a[2], a[3]
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        # strict > / < scan from column 0: first index wins (:1523-1528, :1559-1564)
        r = (X.argmax(axis=1) if kind.startswith("argmax") else X.argmin(axis=1)).astype(F32)
        MEM.view(a[1], rows)[:] = r
        return
    if kind == "slice_2d":  # :1112-1198
        rows, cols, rs, re_, cs, ce, orows, ocols = a[2:10]
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        MEM.view(a[1], orows * ocols)[:] = X[rs:rs + orows, cs:cs + ocols].reshape(-1)
        return
    if kind == "slice_1d":  # :1200-1240
        start, n = a[2], a[3]
        MEM.view(a[1], n)[:] = MEM.view(a[0])[start:start + n]
        return
    if kind in ("linear_1d", "linear_2d"):  # :1584-1661
        if kind == "linear_1d":
            bsz, fin, fout = 1, a[4], a[5]
        else:
            bsz, fin, fout = a[4], a[5], a[6]
        X = MEM.view(a[0], bsz * fin).reshape(bsz, fin)
        W = MEM.view(a[1], fin * fout).reshape(fin, fout)
        b = MEM.view(a[2], fout)
        Y = np.zeros((bsz, fout), dtype=F32)
        for kk in range(fin):
            Y = (Y + np.outer(X[:, kk], W[kk, :]).astype(F32)).astype(F32)
        MEM.view(a[3], bsz * fout)[:] = (Y + b).astype(F32).reshape(-1)
        return
    if kind in ("layer_norm_2d", "layer_norm_axis0", "layer_norm_1d", "instance_norm_2d"):
        # :1667-1810, :2017-2061: two-pass population statistics, sqrtf(var+eps)
        if kind == "layer_norm_1d":
            rows, cols, eps, ax = 1, a[2], a[3], 1
        else:
            rows, cols, eps = a[2], a[3], a[4]
            ax = 0 if kind == "layer_norm_axis0" else 1
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        lines = X.T if ax == 0 else X
        out = np.empty_like(lines)
        for i, v in enumerate(lines):
            mean = F32(_seq_sum(v) / F32(v.size))
            d = (v - mean).astype(F32)
            var = F32(_seq_sum(d * d) / F32(v.size))
            sd = np.sqrt(F32(var + F32(eps)))
            out[i] = (d / sd).astype(F32)
        res = out.T if ax == 0 else out
        MEM.view(a[1], rows * cols)[:] = np.ascontiguousarray(res).reshape(-1)
        return
    if kind == "batch_norm_2d":  # :1978-2011 running statistics, no affine
        n, f, eps = a[4], a[5], a[6]
        X = MEM.view(a[0], n * f).reshape(n, f)
        mu = MEM.view(a[1], f)
        var = MEM.view(a[2], f)
        MEM.view(a[3], n * f)[:] = ((X - mu) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32).reshape(-1)
        return
    if kind == "cross_entropy":  # :1816-1885 class-index targets
        bsz, ncls = a[3], a[4]
        P = MEM.view(a[0], bsz * ncls).reshape(bsz, ncls)
        T = MEM.view(a[1], bsz)
        tot = F32(0.0)
        for i in range(bsz):
            c = max(0, min(int(T[i]), ncls - 1))
            p = min(max(P[i, c], F32(1e-7)), F32(1.0) - F32(1e-7))
            tot = F32(tot + F32(-np.log(F32(p))))
        MEM.view(a[2], 1)[0] = F32(tot / F32(bsz))
        return
    if kind == "mse_loss":  # :1891-1943
        n = a[3]
        d = (MEM.view(a[0], n) - MEM.view(a[1], n)).astype(F32)
        MEM.view(a[2], 1)[0] = F32(F32(np.sum(d * d, dtype=F32)) / F32(n))
        return
    if kind == "transpose_2d":  # :1949-1972
        rows, cols = a[2], a[3]
        X = MEM.view(a[0], rows * cols).reshape(rows, cols)
        MEM.view(a[1], rows * cols)[:] = X.T.reshape(-1)
        return
    if kind == "reshape":  # :2067-2086
        n = a[2]
        MEM.view(a[1], n)[:] = MEM.view(a[0], n)
        return
    if kind == "concat_axis0":  # :2092-2132
        r1, r2, cols = a[3], a[4], a[5]
        MEM.view(a[2], (r1 + r2) * cols)[:] = np.concatenate(
            [MEM.view(a[0], r1 * cols), MEM.view(a[1], r2 * cols)])
        return
    raise UndefinedBehaviour(f"no emulation for kernel kind {kind}")


# ---------------------------------------------------------------------------
# Run the reference executor on each program
# ---------------------------------------------------------------------------

def extract_expected(text):
    m = re.search(r"//\s*@EXPECTED\s*\n", text)
    if not m:
        return None
    lines = []
    for line in text[m.end():].split("\n"):
        mm = re.match(r"//\s*(.*)", line)
        if not mm:
            break
        lines.append(mm.group(1))
    try:
        return json.loads("\n".join(lines))
    except json.JSONDecodeError:
        return None


def run_reference_programs(ref: Path):
    sys.path.insert(0, str(ref))
    install_fake_pycuda()
    import tensorlang.compiler as tlc
    from tensorlang.kernel_generator import KernelGenerator

    global SCRATCH
    SCRATCH = Path(tempfile.mkdtemp(prefix="tl_golden_"))
    (SCRATCH / "tensorlang.lark").symlink_to(ref / "tensorlang.lark")
    (SCRATCH / "tests").symlink_to(ref / "tests")
    os.chdir(SCRATCH)

    captured = {}
    orig_build_ast, orig_tc = tlc.build_ast, tlc.type_checker

    def cap_build_ast(tree, *a, **kw):
        res = orig_build_ast(tree, *a, **kw)
        captured["ast"] = strip_ast(res[0])
        return res

    def cap_type_checker(ast, env, *a, **kw):
        ok, env2 = orig_tc(ast, env, *a, **kw)
        captured["env"] = strip_ast({k: {"dtype": v["dtype"], "shape": list(v["shape"])}
                                     for k, v in env2.items()})
        captured["typecheck_ok"] = bool(ok)
        return ok, env2

    tlc.build_ast = cap_build_ast
    tlc.type_checker = cap_type_checker

    kinfos = {}

    class RecordingGenerator(KernelGenerator):
        pass

    for meth in [m for m in dir(KernelGenerator) if not m.startswith("_")
                 and m not in ("cuda_header", "cuda_debug", "generate_unary_op_kernel")]:
        orig = getattr(KernelGenerator, meth)

        def wrap(orig=orig):
            def w(self, *args, **kw):
                res = orig(self, *args, **kw)
                if res is not None and res[1] is not None:
                    ki = res[1]
                    name = ki[2] if ki[0] == "general_broadcast" else ki[1]
                    kinfos[name] = ki
                return res
            return w
        setattr(RecordingGenerator, meth, wrap())
    tlc.KernelGenerator = RecordingGenerator

    tlc.subprocess = types.SimpleNamespace(run=lambda *a, **k: subprocess.CompletedProcess(a, 0),
                                           CalledProcessError=subprocess.CalledProcessError)
    ctypes.cdll.LoadLibrary = lambda path: KernelEmulator(kinfos)

    files = sorted(glob.glob("tests/*.tl"))
    # basics.tl writes the .npy files that the load_* programs read
    files.sort(key=lambda f: (0 if f.endswith("basics.tl") else 1, f))
    out = {}
    for f in files:
        name = Path(f).stem
        captured.clear()
        kinfos.clear()
        text = (ref / f).read_text()
        rec = {"file": f, "expected": extract_expected(text)}
        status = "ok"
        try:
            comp = tlc.TensorCompiler(debug_mode=False, cache_layers=True)
            with contextlib.redirect_stdout(io.StringIO()):
                comp.compile_and_execute(f)
        except UndefinedBehaviour as e:
            status = f"undefined: {e}"
        except SystemExit as e:
            status = f"exit: {e.code}"
        except Exception as e:  # noqa: BLE001 - recorded, not hidden
            status = f"error: {type(e).__name__}: {e}"
        rec["status"] = status
        rec["ast"] = captured.get("ast")
        rec["env"] = captured.get("env")
        rec["typecheck_ok"] = captured.get("typecheck_ok")
        outs = {}
        cdir = SCRATCH / "cache" / f
        if cdir.exists():
            for npy in sorted(cdir.glob("*.npy")):
                outs[npy.name[:-4]] = arr_to_json(np.load(npy))
        rec["outputs"] = outs
        # the load_* programs read files that basics.tl saved; keep them
        loads = {}
        for node in rec["ast"] or []:
            e = node.get("expr") if isinstance(node, dict) else None
            if isinstance(e, dict) and e.get("type") == "load":
                p = SCRATCH / e["file_path"]
                if p.exists():
                    loads[e["file_path"]] = arr_to_json(np.load(p))
        rec["load_files"] = loads
        out[name] = rec
    os.chdir(REPO)
    return out


# ---------------------------------------------------------------------------
# kernel_info dispatch tuples
# ---------------------------------------------------------------------------

KINFO_CALLS = [
    ("elementwise", ["add", "c", "a", "b", 12]),
    ("elementwise", ["div", "c", "a", "b", 7]),
    ("binary_broadcast", ["mult", "mult", "xs", "x", "s", [8, 8], [8], [8, 8]]),
    ("binary_broadcast", ["add", "add", "y", "x", "b", [3, 4], [4], [3, 4]]),
    ("binary_broadcast", ["minus", "minus", "y", "x", "b", [3, 4], [3], [3, 4]]),
    ("binary_1d_broadcast", ["mult", "g", "bg", "lr1", 10]),
    ("binary_general_broadcast", ["add", "u", "xs", "b", [8, 8], [8, 1], [8, 8]]),
    ("binary_general_broadcast", ["mult", "s", "lr", "wg", [1, 1], [4, 3], [4, 3]]),
    ("fill", ["fill", "z", None, None, 16, 0.5]),
    ("matmul", ["matmul", "c", "a", "b", 4, 3, 2]),
    ("relu", ["relu", "r", "h", 64]),
    ("sigmoid", ["sigmoid", "s", "h", 64]),
    ("tanh", ["tanh", "t", "h", 64]),
    ("softmax", ["softmax", "p", "z", [64, 10], 1]),
    ("softmax", ["softmax", "p", "z", [10], None]),
    ("greater_broadcast", ["greater", "m", "y", "zero", [8, 8], [8], [8, 8], 64]),
    ("greater_broadcast", ["greater", "m", "y", "z", [8, 8], [8, 8], [8, 8], 64]),
    ("less_broadcast", ["less", "m", "y", "z", [4, 5], [5], [4, 5]]),
    ("less_broadcast", ["less", "m", "y", "z", [4, 5], [4, 5], [4, 5]]),
    ("equal", ["equal", "m", "y", "z", [4, 5], [4, 5], [4, 5]]),
    ("sum", ["sum", "s", "x", None, [16, 4]]),
    ("sum", ["sum", "s", "x", 1, [16, 4]]),
    ("sum", ["sum", "s", "x", 0, [16, 4]]),
    ("mean", ["mean", "s", "x", None, [16, 4]]),
    ("mean", ["mean", "s", "x", 1, [16, 4]]),
    ("mean", ["mean", "s", "x", 0, [16, 4]]),
    ("max", ["max", "s", "x", None, [16, 4]]),
    ("max", ["max", "s", "x", 1, [16, 4]]),
    ("max", ["max", "s", "x", 0, [16, 4]]),
    ("min", ["min", "s", "x", None, [16, 4]]),
    ("min", ["min", "s", "x", 1, [16, 4]]),
    ("min", ["min", "s", "x", 0, [16, 4]]),
    ("argmax", ["argmax", "s", "x", 1, [16, 4]]),
    ("argmax", ["argmax", "s", "x", None, [16, 4]]),
    ("argmin", ["argmin", "s", "x", 1, [16, 4]]),
    ("slice", ["slice", "s", "x", [{"type": "slice", "start": 1, "end": 3},
                                  {"type": "full_slice"}], [4, 5], [2, 5]]),
    ("slice", ["slice", "s", "x", [{"type": "index", "value": 2}], [6], [1]]),
    ("linear", ["linear", "y", "x", "W", "b", [64, 128], [128, 256], [64, 256]]),
    ("linear", ["linear", "y", "x", "W", "b", [128], [128, 256], [256]]),
    ("layer_norm", ["layer_norm", "y", "x", 1, 1e-5, [16, 4]]),
    ("layer_norm", ["layer_norm", "y", "x", 0, 1e-5, [16, 4]]),
    ("layer_norm", ["layer_norm", "y", "x", None, 1e-5, [16]]),
    ("cross_entropy", ["cross_entropy", "l", "p", [64, 10], [64], "t"]),
    ("mse_loss", ["mse_loss", "l", "p", "t", 640]),
    ("transpose", ["transpose", "t", [3, 5], "x"]),
    ("batch_norm", ["batch_norm", "y", [8, 4], "x", "rm", 1e-5, "rv"]),
    ("instance_norm", ["instance_norm", "y", "x", [8, 4], 1e-5]),
    ("reshape", ["reshape", "y", "x", 24]),
]


def kinfo_cases(ref: Path):
    sys.path.insert(0, str(ref))
    from tensorlang.kernel_generator import KernelGenerator
    gen = KernelGenerator(False)
    cases = []
    for meth, args in KINFO_CALLS:
        call = [tuple(a) if isinstance(a, list) and a and not isinstance(a[0], dict) else a
                for a in args]
        with contextlib.redirect_stdout(io.StringIO()):
            res = getattr(gen, meth)(*call)
        kinfo = None if res is None else strip_ast(res[1])
        cases.append({"method": meth, "args": args, "kinfo": kinfo})
    # concat needs an env
    env = {"a": {"shape": (2, 3)}, "b": {"shape": (4, 3)}, "c": {"shape": (6, 3)}}
    res = gen.concat("concat", "c", ["a", "b"], 0, env)
    cases.append({"method": "concat", "args": ["concat", "c", ["a", "b"], 0,
                                               {k: {"shape": list(v["shape"])} for k, v in env.items()}],
                  "kinfo": strip_ast(res[1])})
    return cases


# ---------------------------------------------------------------------------
# Reference autograd on seeded inputs
# ---------------------------------------------------------------------------

def autograd_cases(ref: Path):
    sys.path.insert(0, str(ref))
    from tensorlang.autograd import ComputationGraph
    rng = np.random.default_rng(1234)
    f32 = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    cases = []

    def run(label, tensors, grad_names, nodes, loss):
        g = ComputationGraph(debug_mode=False)
        for k, v in tensors.items():
            g.register_tensor(k, v, k in grad_names)
        for op, out, ins, meta in nodes:
            g.add_operation(op, out, ins, meta)
        with contextlib.redirect_stdout(io.StringIO()):
            g.backward(loss)
        cases.append({
            "label": label,
            "tensors": {k: arr_to_json(v) for k, v in tensors.items()},
            "requires_grad": sorted(grad_names),
            "nodes": [[op, out, ins, meta] for op, out, ins, meta in nodes],
            "loss": loss,
            "gradients": {k: arr_to_json(v) for k, v in g.gradients.items()},
        })

    # linear -> relu -> linear -> softmax -> cross_entropy (one-hot), the
    # training graph of the MLP configurations (autograd.py:540,563,619,691)
    B, I, H, C = 6, 5, 7, 4
    x, W1, W2 = f32(B, I), f32(I, H) * 0.3, f32(H, C) * 0.3
    b1, b2 = f32(H) * 0.1, f32(C) * 0.1
    h = (x @ W1 + b1).astype(np.float32)
    a = np.maximum(h, 0).astype(np.float32)
    z = (a @ W2 + b2).astype(np.float32)
    e = np.exp(z - z.max(axis=1, keepdims=True))
    p = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    t = np.eye(C, dtype=np.float32)[rng.integers(0, C, B)]
    loss = np.array(-np.mean(np.log(np.clip((p * t).sum(1), 1e-7, 1 - 1e-7))), dtype=np.float32)
    run("mlp_ce", dict(x=x, W1=W1, b1=b1, h=h, a=a, W2=W2, b2=b2, z=z, p=p, t=t, loss=loss),
        {"W1", "b1", "W2", "b2"},
        [("linear", "h", ["x", "W1", "b1"], {}), ("relu", "a", ["h"], {}),
         ("linear", "z", ["a", "W2", "b2"], {}), ("softmax", "p", ["z"], {"axis": 1}),
         ("cross_entropy", "loss", ["p", "t"], {})], "loss")

    # linear -> relu -> mse (autograd.py:677)
    X, W, b, T = f32(5, 4), f32(4, 3), np.zeros(3, np.float32), f32(5, 3)
    zz = (X @ W + b).astype(np.float32)
    y = np.maximum(zz, 0).astype(np.float32)
    l2 = np.array(np.mean((y - T) ** 2), dtype=np.float32)
    run("linear_relu_mse", dict(X=X, W=W, b=b, z=zz, y=y, T=T, loss=l2), {"X", "W", "b"},
        [("linear", "z", ["X", "W", "b"], {}), ("relu", "y", ["z"], {}),
         ("mse_loss", "loss", ["y", "T"], {})], "loss")

    # broadcasting elementwise chain + reductions (autograd.py:491-616, _unbroadcast :350-488)
    A, Bv, Cc, D = f32(3, 4), f32(4), f32(3, 1), f32(1, 1)
    u = (A + Bv).astype(np.float32)
    v = (u * Cc).astype(np.float32)
    w = (v - D).astype(np.float32)
    q = (w / (np.abs(A) + 1.0)).astype(np.float32)
    Aabs = (np.abs(A) + 1.0).astype(np.float32)
    s = np.tanh(q).astype(np.float32)
    sg = (1 / (1 + np.exp(-s))).astype(np.float32)
    m0 = sg.mean(axis=0).astype(np.float32)
    s1 = np.array(m0.sum(), dtype=np.float32)
    run("broadcast_chain", dict(A=A, Bv=Bv, Cc=Cc, D=D, u=u, v=v, w=w, Aabs=Aabs, q=q,
                                s=s, sg=sg, m0=m0, s1=s1),
        {"A", "Bv", "Cc", "D", "Aabs"},
        [("add", "u", ["A", "Bv"], {}), ("mult", "v", ["u", "Cc"], {}),
         ("minus", "w", ["v", "D"], {}), ("div", "q", ["w", "Aabs"], {}),
         ("tanh", "s", ["q"], {}), ("sigmoid", "sg", ["s"], {}),
         ("mean", "m0", ["sg"], {"axis": 0}), ("sum", "s1", ["m0"], {"axis": None})], "s1")

    # matmul + sum(axis=1) + mean(full)
    M1, M2 = f32(4, 6), f32(6, 3)
    mm = (M1 @ M2).astype(np.float32)
    r = mm.sum(axis=1).astype(np.float32)
    mn = np.array(r.mean(), dtype=np.float32)
    run("matmul_sum_mean", dict(M1=M1, M2=M2, mm=mm, r=r, mn=mn), {"M1", "M2"},
        [("matmul", "mm", ["M1", "M2"], {}), ("sum", "r", ["mm"], {"axis": 1}),
         ("mean", "mn", ["r"], {"axis": None})], "mn")

    # layer_norm backward (autograd.py:649-674)
    L = f32(4, 8)
    mu = L.mean(axis=1, keepdims=True)
    ln = ((L - mu) / np.sqrt(L.var(axis=1, keepdims=True) + 1e-5)).astype(np.float32)
    Tl = f32(4, 8)
    lm = np.array(np.mean((ln - Tl) ** 2), dtype=np.float32)
    run("layer_norm_mse", dict(L=L, ln=ln, Tl=Tl, lm=lm), {"L"},
        [("layer_norm", "ln", ["L"], {"axis": 1, "eps": 1e-5}),
         ("mse_loss", "lm", ["ln", "Tl"], {})], "lm")
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TL_REFERENCE"),
                    required="TL_REFERENCE" not in os.environ,
                    help="checkout of the TensorLang reference (or set TL_REFERENCE)")
    args = ap.parse_args()
    ref = Path(args.reference).resolve()
    progs = run_reference_programs(ref)
    (HERE / "ref_programs.json").write_text(json.dumps(progs, indent=0, sort_keys=True))
    (HERE / "kinfo_cases.json").write_text(json.dumps(kinfo_cases(ref), indent=0))
    (HERE / "autograd_cases.json").write_text(json.dumps(autograd_cases(ref), indent=0))
    n_ok = sum(1 for r in progs.values() if r["status"] == "ok")
    print(f"programs: {len(progs)} ({n_ok} ran), statuses:")
    for k, r in sorted(progs.items()):
        if r["status"] != "ok":
            print(f"  {k}: {r['status']}")


if __name__ == "__main__":
    main()
