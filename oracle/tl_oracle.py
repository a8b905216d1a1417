"""NumPy restatement of the TensorLang reference execution path (test oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``; never by the GPU backend.

Three layers, each following the reference file it names:

* ``op_forward`` -- one ``let`` expression evaluated the way the CUDA that
  ``tensorlang/kernel_generator.py`` generates for it evaluates, with the
  dispatch rules of ``tensorlang/compiler.py:1110-1424`` (which generator a
  shape pair selects).
* ``_Graph`` -- ``tensorlang/autograd.py`` ``ComputationGraph``: zero-init,
  seed, reverse walk with the all-zero skip, per-op VJPs, ``_unbroadcast``.
* ``OracleProgram`` -- the phase order of ``TensorCompiler.compile_and_execute``
  (``compiler.py:1481-1661``) and ``_execute_for_loop`` (``compiler.py:168-352``),
  including which operations ``_record_operation`` (``compiler.py:47-54``)
  records into the autograd graph.

``dtype=np.float64`` is the correctness oracle; ``dtype=np.float32`` mirrors
the reference's own float32 arithmetic and is the timed CPU baseline.

Where the reference has no semantics (an op with no generator, a shape its
generator returns ``None`` for, or launcher code with undefined behaviour) the
oracle defines them; the list is ``SEMANTICS_EXTENSIONS`` and the GPU backend
implements the same definitions.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import numpy as np

try:  # exact erf for gelu; scipy is optional, math.erf is the fallback
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)

SEMANTICS_EXTENSIONS = {
    "gelu": "exact 0.5*x*(1+erf(x/sqrt(2))); the reference has grammar/type rules "
            "(tensorlang.lark:175, type_checker.py:274) but no kernel",
    "swish": "x*sigmoid(x); same gap as gelu",
    "cross_entropy_onehot": "targets (B,C): -mean_b log(clamp(sum_c t*p, 1e-7, 1-1e-7)); "
                            "the reference generator returns None (kernel_generator.py:1818)",
    "autograd_records": "linear, cross_entropy, layer_norm, gelu, swish are recorded into the "
                        "autograd graph (the reference records only the ops at "
                        "compiler.py:1114-1374 / 776-848)",
    "cross_entropy_vjp_class_index": "class-index targets use one-hot(t) in the VJP "
                                     "(autograd.py:702 would broadcast (B,C)-(B,))",
    "gelu_swish_vjp": "d gelu = Phi(x)+x*phi(x); d swish = s+x*s*(1-s)",
    "for_body_ops": "every op lowers inside a for body (compiler.py:767-851 lowers a subset)",
    "argmax_argmin_axes": "axis 0 and full argmax/argmin: NumPy first-index "
                          "(the reference generates axis 1 only; full argmax kernel is broken)",
    "compare_scalar_operand": "greater/less/equal against a (1,) or (1,1) operand broadcast "
                              "as NumPy does (kernel_generator.py:676 reads B[j] out of bounds)",
    "equal_broadcast": "equal with a 1-D operand uses B[j] like greater/less "
                       "(compiler.py:450-457 calls the launcher with a missing argument)",
    "nd_reductions": "sum/mean/max/min over any axis of an N-D tensor follow NumPy",
    "softmax_axis0": "softmax over axis 0 of a 2-D tensor follows the same formula column-wise",
    "matmul_matvec": "matmul(A[m,n], v[n]) is the matrix-vector product (the reference "
                     "kernel indexes B[k*P+j] with P=n, reading past v)",
    "scalar_arg1": "op(a[1], b[n]) broadcasts a[0] (binary_1d_broadcast assumes the scalar "
                   "is the second operand, kernel_generator.py:363-367)",
    "aliases": "let a = b copies b's value at that statement",
    "body_literals": "tensor literals inside a for body are initialised once",
}

_BIN = {"add": np.add, "minus": np.subtract, "mult": np.multiply, "div": np.divide}
_RECORDED_REFERENCE = {"add", "minus", "mult", "div", "matmul", "relu", "sigmoid", "tanh",
                       "softmax", "sum", "mean", "mse_loss"}
_RECORDED_EXTENDED = _RECORDED_REFERENCE | {"linear", "cross_entropy", "layer_norm", "gelu", "swish"}
KERNEL_FREE = ("name", "tensor_literal", "load")


def _shape(v) -> tuple:
    return tuple(int(d) for d in v)


# ---------------------------------------------------------------------------
# shapes (type_checker.py output shapes, restated for the ops on the path)
# ---------------------------------------------------------------------------

def _bcast(s1, s2):
    n = max(len(s1), len(s2))
    a = (1,) * (n - len(s1)) + tuple(s1)
    b = (1,) * (n - len(s2)) + tuple(s2)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ValueError(f"shapes {s1} and {s2} do not broadcast")
        out.append(max(x, y))
    return tuple(out)


def _slice_bounds(spec, size):
    """kernel_generator.py:1125-1160 -- start/end with Python-exclusive end, clamped."""
    t = spec.get("type")
    if t == "slice":
        start = spec.get("start")
        end = spec.get("end")
        start = 0 if start is None else int(start)
        end = size if end is None else int(end)
    elif t == "index":
        start = int(spec["value"])
        end = start + 1
    else:
        start, end = 0, size
    start = max(0, min(start, size))
    end = max(start, min(end, size))
    return start, end


def infer_shape(expr: dict, shapes: Dict[str, tuple]) -> tuple:
    """Output shape of one expression given its operand shapes."""
    t = expr["type"]
    if t in _BIN:
        s1, s2 = shapes[expr["args"][0]], shapes[expr["args"][1]]
        if s1 == s2:
            return s1
        if len(s1) == 2 and len(s2) == 1:
            return s1
        return _bcast(s1, s2)
    if t in ("relu", "sigmoid", "tanh", "gelu", "swish"):
        return shapes[expr["args"][0]]
    if t in ("greater", "less", "equal"):
        s1, s2 = shapes[expr["args"][0]], shapes[expr["args"][1]]
        if s1 == s2 or (len(s1) == 2 and len(s2) == 1):
            return s1
        return _bcast(s1, s2)
    if t == "fill":
        return _shape(expr["shape"])
    if t == "matmul":
        a, b = shapes[expr["args"][0]], shapes[expr["args"][1]]
        if len(a) == 2 and len(b) == 2:
            return (a[0], b[1])
        if len(a) == 2 and len(b) == 1:
            return (a[0],)
        if len(a) == 1 and len(b) == 2:
            return (b[1],)
        raise ValueError(f"matmul shapes {a} @ {b}")
    if t == "linear":
        x, w = shapes[expr["args"][0]], shapes[expr["args"][1]]
        return (w[1],) if len(x) == 1 else (x[0], w[1])
    if t in ("softmax", "layer_norm", "batch_norm", "instance_norm"):
        return shapes[expr["tensor"]]
    if t in ("sum", "mean", "max", "min", "argmax", "argmin"):
        s = shapes[expr["tensor"]]
        ax = expr.get("axis")
        if ax is None:
            return ()
        ax = int(ax) % len(s)
        return tuple(d for i, d in enumerate(s) if i != ax)
    if t in ("mse_loss", "cross_entropy"):
        return ()
    if t == "transpose":
        s = shapes[expr["tensor"]]
        axes = expr.get("axes")
        if axes:
            return tuple(s[int(i)] for i in axes)
        return tuple(reversed(s))
    if t == "reshape":
        return _shape(expr["new_shape"])
    if t == "concat":
        ss = [shapes[n] for n in expr["tensors"]]
        ax = int(expr.get("axis") or 0)
        out = list(ss[0])
        out[ax] = sum(s[ax] for s in ss)
        return tuple(out)
    if t == "slice":
        s = shapes[expr["tensor"]]
        specs = expr["specs"]
        out = []
        for i, d in enumerate(s):
            spec = specs[i] if i < len(specs) else {"type": "full_slice"}
            a, b = _slice_bounds(spec, d)
            out.append(b - a)
        return tuple(out)
    if t == "name":
        return shapes[expr["name"]]
    raise ValueError(f"no shape rule for {t}")


# ---------------------------------------------------------------------------
# forward ops
# ---------------------------------------------------------------------------

def _gelu(x):
    return 0.5 * x * (1.0 + _erf(x / np.sqrt(2.0)))


def _sigmoid(x):
    one = x.dtype.type(1.0)
    return one / (one + np.exp(-x))


def _argfirst(x, axis, largest):
    """First index of the max (min) along ``axis``; NaN-free inputs."""
    return (np.argmax(x, axis=axis) if largest else np.argmin(x, axis=axis))


def op_forward(expr: dict, vals: Dict[str, np.ndarray], dt=np.float64,
               numpy_broadcast: bool = False) -> np.ndarray:
    """Evaluate one ``let`` expression; ``vals`` maps operand names to arrays.

    ``numpy_broadcast``: a square 2-D op 1-D reads ``B[j]`` (NumPy) instead
    of the reference's ``B[i]``."""
    t = expr["type"]
    T = np.dtype(dt).type
    if t in _BIN:
        a, b = vals[expr["args"][0]], vals[expr["args"][1]]
        op = _BIN[t]
        if a.shape == b.shape:  # elementwise, kernel_generator.py:246-275
            return op(a, b).astype(dt)
        if a.ndim == 2 and b.ndim == 1:  # binary_broadcast :281-348
            square = numpy_broadcast and a.shape[1] == b.shape[0]
            if a.shape[0] == b.shape[0] and not square:
                return op(a, b[:, None]).astype(dt)  # B[i]
            return op(a, b[None, :]).astype(dt)  # B[j]
        if a.ndim == 1 and b.ndim == 1 and b.shape[0] == 1:  # binary_1d_broadcast :354-377
            return op(a, b[0]).astype(dt)
        return op(a, b).astype(dt)  # binary_general_broadcast :383-463 (NumPy rule)
    if t == "relu":  # fmaxf(0, x)
        x = vals[expr["args"][0]]
        return np.maximum(T(0), x).astype(dt)
    if t == "sigmoid":  # 1/(1+expf(-x))
        return _sigmoid(vals[expr["args"][0]]).astype(dt)
    if t == "tanh":
        return np.tanh(vals[expr["args"][0]]).astype(dt)
    if t == "gelu":
        x = vals[expr["args"][0]]
        return _gelu(x.astype(np.float64)).astype(dt)
    if t == "swish":
        x = vals[expr["args"][0]]
        return (x * _sigmoid(x)).astype(dt)
    if t in ("greater", "less", "equal"):  # :646-778 -> 1.0 / 0.0
        a, b = vals[expr["args"][0]], vals[expr["args"][1]]
        if a.shape != b.shape and a.ndim == 2 and b.ndim == 1 and b.shape[0] == a.shape[1]:
            b = b[None, :]  # always B[j]
        if t == "greater":
            c = a > b
        elif t == "less":
            c = a < b
        else:
            c = np.abs(a - b) < T(1e-6)
        return c.astype(dt)
    if t == "fill":
        return np.full(_shape(expr["shape"]), T(expr["value"]), dtype=dt)
    if t == "matmul":  # :501-525
        a, b = vals[expr["args"][0]], vals[expr["args"][1]]
        return (a @ b).astype(dt)
    if t == "linear":  # :1584-1661, y = x @ W + b with W [in, out]
        x, w, b = (vals[n] for n in expr["args"])
        return (x @ w + b).astype(dt)
    if t == "softmax":  # :564-640, max-subtracted
        x = vals[expr["tensor"]]
        ax = expr.get("axis")
        ax = x.ndim - 1 if ax is None else int(ax)
        m = x.max(axis=ax, keepdims=True)
        e = np.exp(x - m)
        return (e / e.sum(axis=ax, keepdims=True)).astype(dt)
    if t in ("sum", "mean", "max", "min"):
        x = vals[expr["tensor"]]
        ax = expr.get("axis")
        ax = None if ax is None else int(ax)
        if t in ("sum", "mean"):
            acc = x.astype(np.float64) if dt == np.float64 else x
            r = acc.sum(axis=ax) if t == "sum" else acc.mean(axis=ax)
        else:
            r = x.max(axis=ax) if t == "max" else x.min(axis=ax)
        return np.asarray(r, dtype=dt)
    if t in ("argmax", "argmin"):  # :1459-1578 strict compare -> first index
        x = vals[expr["tensor"]]
        ax = expr.get("axis")
        if ax is None:
            r = _argfirst(x.reshape(-1), 0, t == "argmax")
        else:
            r = _argfirst(x, int(ax), t == "argmax")
        return np.asarray(r, dtype=dt)
    if t == "layer_norm":  # :1667-1810 population variance, sqrtf(var+eps), no affine
        x = vals[expr["tensor"]]
        ax = expr.get("axis")
        ax = x.ndim - 1 if ax is None else int(ax)
        eps = T(expr.get("eps", 1e-5) if expr.get("eps") is not None else 1e-5)
        mu = x.mean(axis=ax, keepdims=True)
        d = x - mu
        var = (d * d).mean(axis=ax, keepdims=True)
        return (d / np.sqrt(var + eps)).astype(dt)
    if t == "instance_norm":  # :2017-2061 per-row
        x = vals[expr["tensor"]]
        eps = T(expr.get("eps", 1e-5) if expr.get("eps") is not None else 1e-5)
        mu = x.mean(axis=1, keepdims=True)
        d = x - mu
        var = (d * d).mean(axis=1, keepdims=True)
        return (d / np.sqrt(var + eps)).astype(dt)
    if t == "batch_norm":  # :1978-2011 running statistics
        x = vals[expr["tensor"]]
        rm, rv = vals[expr["running_mean"]], vals[expr["running_var"]]
        eps = T(expr.get("eps", 1e-5) if expr.get("eps") is not None else 1e-5)
        return ((x - rm) / np.sqrt(rv + eps)).astype(dt)
    if t == "mse_loss":  # :1891-1943 mean((p-t)^2)
        p, q = vals[expr["args"][0]], vals[expr["args"][1]]
        d = (p - q).astype(np.float64) if dt == np.float64 else (p - q)
        return np.asarray((d * d).sum() / T(d.size), dtype=dt)
    if t == "cross_entropy":  # :1816-1885
        p, q = vals[expr["args"][0]], vals[expr["args"][1]]
        lo, hi = T(1e-7), T(1.0) - T(1e-7)
        if q.ndim == 1:  # class indices stored as float, clamped to [0, C-1]
            c = np.clip(q.astype(np.int64), 0, p.shape[1] - 1)
            pp = p[np.arange(p.shape[0]), c]
        else:  # one-hot targets (extension)
            pp = (p * q).sum(axis=1)
        pp = np.minimum(np.maximum(pp, lo), hi)
        return np.asarray(-np.log(pp).sum() / T(p.shape[0]), dtype=dt)
    if t == "transpose":  # :1949-1972
        x = vals[expr["tensor"]]
        axes = expr.get("axes")
        return np.ascontiguousarray(np.transpose(x, axes if axes else None)).astype(dt)
    if t == "reshape":  # :2067-2086 copy
        x = vals[expr["tensor"]]
        return x.reshape(_shape(expr["new_shape"])).astype(dt)
    if t == "concat":  # :2092-2132
        xs = [vals[n] for n in expr["tensors"]]
        return np.concatenate(xs, axis=int(expr.get("axis") or 0)).astype(dt)
    if t == "slice":  # :1112-1240
        x = vals[expr["tensor"]]
        specs = expr["specs"]
        idx = []
        for i, d in enumerate(x.shape):
            spec = specs[i] if i < len(specs) else {"type": "full_slice"}
            a, b = _slice_bounds(spec, d)
            idx.append(slice(a, b))
        return np.ascontiguousarray(x[tuple(idx)]).astype(dt)
    raise ValueError(f"oracle has no rule for op {t}")


# ---------------------------------------------------------------------------
# autograd (tensorlang/autograd.py)
# ---------------------------------------------------------------------------

class _Node:
    __slots__ = ("op", "out", "ins", "meta")

    def __init__(self, op, out, ins, meta):
        self.op, self.out, self.ins, self.meta = op, out, list(ins), dict(meta or {})


def unbroadcast(g: np.ndarray, shape: tuple) -> np.ndarray:
    """autograd.py:350-488: sum prepended axes, then stretched axes (keepdims)."""
    shape = tuple(shape)
    if g.shape == shape:
        return g
    scalar = shape == ()
    tgt = (1,) if scalar else shape
    while g.ndim > len(tgt):
        g = g.sum(axis=0)
    for i in reversed(range(len(tgt))):
        if tgt[i] == 1 and g.shape[i] != 1:
            g = g.sum(axis=i, keepdims=True)
        elif tgt[i] != g.shape[i]:
            raise ValueError(f"unbroadcast {g.shape} -> {shape}")
    if scalar:
        g = g.reshape(())
    return g


class _Graph:
    def __init__(self, dt, textbook_ce=False):
        self.dt = dt
        # cross_entropy through a row softmax (its only consumer, 2-D, axis 1):
        # the textbook (p - t) / B for the logits, nothing for p
        self.textbook_ce = textbook_ce
        self.nodes: List[_Node] = []
        self.tensors: Dict[str, np.ndarray] = {}
        self.requires: set = set()
        self.grads: Dict[str, np.ndarray] = {}

    def register(self, name, value, requires_grad):
        self.tensors[name] = value
        if requires_grad:
            self.requires.add(name)
            self.grads[name] = np.zeros_like(value)

    def _acc(self, name, g):
        """autograd.py:317-333"""
        if name not in self.grads:
            if name not in self.tensors:
                return
            self.grads[name] = np.zeros_like(self.tensors[name])
        shp = self.tensors[name].shape
        g = np.asarray(g)
        if g.shape != shp:
            g = unbroadcast(g, shp)
        self.grads[name] = (self.grads[name] + g).astype(self.dt)

    def backward(self, loss):
        """autograd.py:100-228"""
        if loss not in self.tensors:
            raise ValueError(f"loss tensor {loss!r} not computed")
        need = set(self.requires) | {loss}
        for n in self.nodes:
            need.add(n.out)
            need.update(n.ins)
        for n in need:
            if n in self.tensors:
                self.grads[n] = np.zeros_like(self.tensors[n])
        self._consumers: Dict[str, int] = {}
        for n in self.nodes:
            for i in n.ins:
                self._consumers[i] = self._consumers.get(i, 0) + 1
        self.grads[loss] = np.ones_like(self.tensors[loss])
        for node in reversed(self.nodes):
            if node.out not in self.grads:
                continue
            g = self.grads[node.out]
            if not np.any(g != 0):
                continue
            self._vjp(node, g)

    def _vjp(self, node, g):
        """autograd.py:491-704 plus the extension rules for gelu/swish."""
        T, V = self.tensors, self.dt
        op, ins = node.op, node.ins
        if op == "add":
            self._acc(ins[0], g)
            self._acc(ins[1], g)
        elif op == "minus":
            self._acc(ins[0], g)
            self._acc(ins[1], -g)
        elif op == "mult":
            self._acc(ins[0], g * T[ins[1]])
            self._acc(ins[1], g * T[ins[0]])
        elif op == "div":
            b = T[ins[1]]
            self._acc(ins[0], g / b)
            self._acc(ins[1], -g * T[ins[0]] / (b ** 2))
        elif op == "matmul":
            a, b = T[ins[0]], T[ins[1]]
            self._acc(ins[0], g @ b.T)
            self._acc(ins[1], a.T @ g)
        elif op == "relu":
            x = T[ins[0]]
            self._acc(ins[0], g * (x > 0).astype(V))
        elif op == "sigmoid":
            s = T[node.out]
            self._acc(ins[0], g * s * (1 - s))
        elif op == "tanh":
            y = T[node.out]
            self._acc(ins[0], g * (1 - y ** 2))
        elif op == "gelu":
            x = T[ins[0]].astype(np.float64)
            d = 0.5 * (1.0 + _erf(x / np.sqrt(2.0))) + x * np.exp(-0.5 * x * x) / np.sqrt(2 * np.pi)
            self._acc(ins[0], g * d.astype(V))
        elif op == "swish":
            x = T[ins[0]]
            s = _sigmoid(x)
            self._acc(ins[0], g * (s + x * s * (1 - s)))
        elif op == "softmax":
            s = T[node.out]
            ax = node.meta.get("axis", -1)
            gs = g * s
            self._acc(ins[0], gs - s * np.sum(gs, axis=ax, keepdims=True))
        elif op == "sum":
            x = T[ins[0]]
            ax = node.meta.get("axis")
            if ax is None:
                gg = np.full_like(x, g.item() if g.size == 1 else g)
            else:
                gg = np.broadcast_to(np.expand_dims(g, axis=ax), x.shape)
            self._acc(ins[0], gg)
        elif op == "mean":
            x = T[ins[0]]
            ax = node.meta.get("axis")
            if ax is None:
                cnt = int(np.prod(x.shape))
                gg = np.full_like(x, (g.item() if g.size == 1 else g) / cnt)
            else:
                cnt = x.shape[ax]
                gg = np.broadcast_to(np.expand_dims(g / cnt, axis=ax), x.shape)
            self._acc(ins[0], gg)
        elif op == "linear":
            x, w = T[ins[0]], T[ins[1]]
            self._acc(ins[0], g @ w.T)
            self._acc(ins[1], np.outer(x, g) if x.ndim == 1 else x.T @ g)
            self._acc(ins[2], g if g.ndim == 1 else g.sum(axis=0))
        elif op == "layer_norm":
            x = T[ins[0]]
            ax = node.meta.get("axis", -1)
            eps = node.meta.get("eps", 1e-5)
            mean = x.mean(axis=ax, keepdims=True)
            var = x.var(axis=ax, keepdims=True)
            std = np.sqrt(var + eps)
            n = x.shape[ax]
            gv = np.sum(g * (x - mean) * -0.5 * (var + eps) ** -1.5, axis=ax, keepdims=True)
            gm = (np.sum(g * -1 / std, axis=ax, keepdims=True)
                  + gv * np.sum(-2 * (x - mean), axis=ax, keepdims=True) / n)
            self._acc(ins[0], g / std + gv * 2 * (x - mean) / n + gm / n)
        elif op == "mse_loss":
            p, q = T[ins[0]], T[ins[1]]
            sg = g.item() if g.size == 1 else g
            self._acc(ins[0], 2 * (p - q) / p.size * sg)
        elif op == "cross_entropy":
            p, q = T[ins[0]], T[ins[1]]
            if q.ndim == 1 and p.ndim == 2:
                c = np.clip(q.astype(np.int64), 0, p.shape[1] - 1)
                q = np.eye(p.shape[1], dtype=V)[c]
            sg = g.item() if g.size == 1 else g
            sm = next((n for n in self.nodes if n.out == ins[0] and n.op == "softmax"), None)
            if (self.textbook_ce and sm is not None and p.ndim == 2 and
                    sm.meta.get("axis") in (1, -1) and self._consumers.get(ins[0]) == 1):
                self._acc(sm.ins[0], (p - q) / p.shape[0] * sg)
                return
            self._acc(ins[0], (p - q) / p.shape[0] * sg)


# ---------------------------------------------------------------------------
# program executor (compiler.py phase order)
# ---------------------------------------------------------------------------

def _is_kernel_let(node) -> bool:
    return (node.get("type") == "let" and isinstance(node.get("expr"), dict)
            and node["expr"]["type"] not in KERNEL_FREE)


def _expr_inputs(expr) -> List[str]:
    t = expr["type"]
    if "args" in expr:
        return list(expr["args"])
    if t == "concat":
        return list(expr["tensors"])
    if t == "batch_norm":
        return [expr["tensor"], expr["running_mean"], expr["running_var"]]
    if "tensor" in expr:
        return [expr["tensor"]]
    return []


class OracleProgram:
    """Execute a lowered TensorLang program (reference AST + type environment).

    ``feeds`` replaces the initial value of named ``let`` tensors (used for
    seeded synthetic inputs).  ``load_files`` maps ``load("path")`` paths to
    arrays.  ``record="extended"`` applies the autograd-recording extension;
    ``record="reference"`` records only what the reference records.
    """

    def __init__(self, ast, env, dtype=np.float64, feeds=None, load_files=None,
                 record="extended", semantics="reference"):
        self.ast = ast
        self.env = {k: _shape(v["shape"]) for k, v in env.items()}
        self.dt = np.dtype(dtype).type
        self.feeds = {k: np.asarray(v) for k, v in (feeds or {}).items()}
        self.load_files = load_files or {}
        self.recorded_ops = _RECORDED_EXTENDED if record == "extended" else _RECORDED_REFERENCE
        if semantics not in ("reference", "numpy"):
            raise ValueError(f"semantics must be 'reference' or 'numpy', not {semantics!r}")
        self.numpy_broadcast = semantics == "numpy"
        self.graph = _Graph(self.dt, textbook_ce=semantics == "numpy")
        self.requires: set = set()
        self.tensors: Dict[str, np.ndarray] = {}
        self.outputs: Dict[str, np.ndarray] = {}
        self.saved: Dict[str, np.ndarray] = {}

    # -- recording (codegen-time, compiler.py:996-1424 / 725-851) ----------
    def _record(self, op, out, ins, meta=None):
        if op not in self.recorded_ops:
            return
        if any(i in self.requires for i in ins):
            self.graph.nodes.append(_Node(op, out, ins, meta))
            self.requires.add(out)

    def _record_let(self, node):
        e = node["expr"]
        t = e["type"]
        meta = None
        if t in ("softmax", "sum", "mean"):
            meta = {"axis": e.get("axis")}
        elif t == "layer_norm":
            ax = e.get("axis")
            if ax is None:
                ax = len(self.env[e["tensor"]]) - 1
            eps = e.get("eps")
            meta = {"axis": int(ax), "eps": 1e-5 if eps is None else float(eps)}
        self._record(t, node["name"], _expr_inputs(e), meta)

    def _literal(self, node):
        e = node["expr"]
        name = node["name"]
        if name in self.feeds:
            return self.feeds[name].astype(self.dt)
        if e["type"] == "tensor_literal":
            shp = self.env[name]
            return np.asarray(e["data"], dtype=np.float32).astype(self.dt).reshape(shp)
        if e["type"] == "load":
            arr = self.load_files[e["file_path"]]
            return np.asarray(arr, dtype=np.float32).astype(self.dt)
        raise ValueError(e["type"])

    def _compile(self):
        for node in self.ast:
            typ = node["type"]
            if typ in ("save", "backward", "rebind"):
                continue
            if typ == "for":
                for b in node["body"]:
                    if b["type"] == "let" and isinstance(b.get("expr"), dict):
                        if b["expr"]["type"] == "tensor_literal":
                            self.tensors[b["name"]] = self._literal(b)
                        elif _is_kernel_let(b):
                            self._record_let(b)
                continue
            if typ != "let":
                continue
            if node.get("requires_grad"):
                self.requires.add(node["name"])
            e = node.get("expr")
            if not isinstance(e, dict):
                continue
            if e["type"] in ("tensor_literal", "load"):
                self.tensors[node["name"]] = self._literal(node)
            elif e["type"] != "name":
                self._record_let(node)

    # -- execution ---------------------------------------------------------
    def _exec_let(self, node):
        name = node["name"]
        if name in self.feeds and node["expr"]["type"] in ("fill",):
            self.tensors[name] = self.feeds[name].astype(self.dt)
            return
        self.tensors[name] = op_forward(node["expr"], self.tensors, self.dt, self.numpy_broadcast)

    def _register_all(self):
        for k, v in self.tensors.items():
            self.graph.register(k, v, k in self.requires)

    def _backward(self, loss):
        self.graph.grads = {}
        self._register_all()
        self.graph.backward(loss)
        out = {}
        for n in sorted(self.graph.requires):
            if n in self.graph.grads:
                out[n] = self.graph.grads[n]
        return out

    def _run_for(self, node):
        body = node["body"]
        bw = next((i for i, b in enumerate(body) if b["type"] == "backward"), None)
        rebinds = [b for b in body if b["type"] == "rebind"]
        for _ in range(int(node["iterations"])):
            for i, b in enumerate(body):
                if _is_kernel_let(b) and (bw is None or i < bw):
                    self._exec_let(b)
                elif b["type"] == "let" and isinstance(b.get("expr"), dict) \
                        and b["expr"]["type"] == "name" and (bw is None or i < bw):
                    self.tensors[b["name"]] = self.tensors[b["expr"]["name"]].copy()
            if bw is not None:
                grads = self._backward(body[bw]["loss_tensor"])
                for n, g in grads.items():
                    self.tensors[f"{n}_grad"] = g
                for i, b in enumerate(body):
                    if i > bw and _is_kernel_let(b):
                        self._exec_let(b)
                    elif i > bw and b["type"] == "let" and isinstance(b.get("expr"), dict) \
                            and b["expr"]["type"] == "name":
                        self.tensors[b["name"]] = self.tensors[b["expr"]["name"]].copy()
            pending = {}
            for r in rebinds:
                src = r["expr"]
                if src.get("type") == "name" and src["name"] in self.tensors:
                    pending[r["name"]] = self.tensors[src["name"]]
            self.tensors.update(pending)

    def run(self) -> Dict[str, np.ndarray]:
        self._compile()
        ast = self.ast
        bw = next((i for i, n in enumerate(ast) if n["type"] == "backward"), None)

        def step(i):
            n = ast[i]
            if n["type"] == "for":
                self._run_for(n)
            elif _is_kernel_let(n):
                self._exec_let(n)
            elif n["type"] == "let" and isinstance(n.get("expr"), dict) \
                    and n["expr"]["type"] == "name":
                src = n["expr"]["name"]
                if src in self.tensors:
                    self.tensors[n["name"]] = self.tensors[src].copy()

        if bw is None:
            for i in range(len(ast)):
                step(i)
        else:
            for i in range(bw):
                step(i)
            for n in ast:
                if n["type"] == "backward":
                    grads = self._backward(n["loss_tensor"])
                    for g_name, g in grads.items():
                        self.tensors[f"{g_name}_grad"] = g
                        self.outputs[f"{g_name}.grad"] = g
            for i in range(bw + 1, len(ast)):
                if _is_kernel_let(ast[i]):
                    self._exec_let(ast[i])
                elif ast[i]["type"] == "let" and isinstance(ast[i].get("expr"), dict) \
                        and ast[i]["expr"]["type"] == "name":
                    step(i)
        for n in ast:
            if n["type"] == "save" and n["tensor"] in self.tensors:
                self.saved[n["file_path"]] = self.tensors[n["tensor"]]
        self.outputs.update(self.tensors)
        return self.outputs
