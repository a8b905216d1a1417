"""The benchmark programs as ASTs, plus their .tl source text.

Each program is built directly in the AST form the reference frontend
produces (``tensorlang/ast_builder.py``: ``let``/``for``/``backward``/
``rebind`` dicts), so the GPU host needs no parser.  ``tl_source()`` gives
the same program as .tl text; where the reference frontend is importable the
test-suite checks that it parses the text into exactly these ASTs.

Inputs are ``fill`` placeholders overwritten through ``Program(feeds=...)``
with seeded synthetic data; ``inputs()`` generates that data with
``numpy.random.default_rng(seed)`` (PCG64), drawing in float64 and casting to
float32, in a fixed order.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np


def _let(name, expr, shape=None, grad=False):
    return {"type": "let", "name": name,
            "ty": {"dtype": "f32", "shape": tuple(shape)} if shape is not None else None,
            "expr": expr, "requires_grad": bool(grad)}


def _fill(shape, value=0.0):
    return {"type": "fill", "value": float(value), "shape": tuple(int(d) for d in shape)}


def _call(op, *args):
    return {"type": op, "args": list(args)}


def _lit(values, shape):
    return {"type": "tensor_literal", "data": [float(v) for v in values],
            "is_1d": len(shape) == 1}


def _sgd_lets(params: List[Tuple[str, int]]) -> List[dict]:
    """``let p_step = mult(lr, p_grad); let p_new = minus(p, p_step)``.  Weights use
    the (1,1) rate through general broadcasting; biases use the (1,) rate as the
    second operand, because ``mult(lr(1,1), b_grad(n,))`` does not type-check in
    the reference (type_checker.py:656-663)."""
    out = []
    for p, nd in params:
        if nd == 2:
            out.append(_let(f"{p}_step", _call("mult", "lr", f"{p}_grad")))
        else:
            out.append(_let(f"{p}_step", _call("mult", f"{p}_grad", "lr1")))
        out.append(_let(f"{p}_new", _call("minus", p, f"{p}_step")))
    return out


# ---------------------------------------------------------------------------
# 2-layer MLP, one forward + backward + SGD step (the CPU-runnable case)
# ---------------------------------------------------------------------------

def mlp2_step(B=64, I=128, H=256, C=10, lr=0.01) -> list:
    ast = [
        _let("x", _fill((B, I)), (B, I)),
        _let("W1", _fill((I, H)), (I, H), grad=True),
        _let("b1", _fill((H,)), (H,), grad=True),
        _let("W2", _fill((H, C)), (H, C), grad=True),
        _let("b2", _fill((C,)), (C,), grad=True),
        _let("t", _fill((B, C)), (B, C)),
        _let("lr", _lit([lr], (1, 1)), (1, 1)),
        _let("lr1", _lit([lr], (1,)), (1,)),
        _let("h", _call("linear", "x", "W1", "b1")),
        _let("a", _call("relu", "h")),
        _let("z", _call("linear", "a", "W2", "b2")),
        _let("p", {"type": "softmax", "tensor": "z", "axis": 1}),
        _let("loss", _call("cross_entropy", "p", "t")),
        {"type": "backward", "loss_tensor": "loss"},
    ]
    ast += _sgd_lets([("W1", 2), ("b1", 1), ("W2", 2), ("b2", 1)])
    return ast


def mlp2_inputs(B=64, I=128, H=256, C=10, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, I)).astype(np.float32)
    W1 = (rng.standard_normal((I, H)) * 0.02).astype(np.float32)
    W2 = (rng.standard_normal((H, C)) * 0.02).astype(np.float32)
    labels = rng.integers(0, C, B)
    t = np.eye(C, dtype=np.float32)[labels]
    return {"x": x, "W1": W1, "b1": np.zeros(H, np.float32), "W2": W2,
            "b2": np.zeros(C, np.float32), "t": t}


# ---------------------------------------------------------------------------
# fused broadcast chain gelu(add(mult(x, s), b)) + greater mask
# ---------------------------------------------------------------------------

def fused_chain(N=8192) -> list:
    return [
        _let("x", _fill((N, N)), (N, N)),
        _let("s", _fill((N,)), (N,)),
        _let("b", _fill((N, 1)), (N, 1)),
        _let("zero", _fill((N,), 0.0), (N,)),
        _let("xs", _call("mult", "x", "s")),
        _let("u", _call("add", "xs", "b")),
        _let("y", _call("gelu", "u")),
        _let("m", _call("greater", "y", "zero")),
    ]


def fused_chain_inputs(N=8192, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((N, N), dtype=np.float32)
    s = rng.uniform(0.5, 1.5, N).astype(np.float32)
    b = (rng.standard_normal((N, 1)) * 0.1).astype(np.float32)
    return {"x": x, "s": s, "b": b, "zero": np.zeros(N, np.float32)}


# ---------------------------------------------------------------------------
# reductions / softmax / layer_norm on one matrix
# ---------------------------------------------------------------------------

REDUCTION_OPS = [
    ("sum1", "sum", 1), ("mean1", "mean", 1), ("max1", "max", 1), ("argmax1", "argmax", 1),
    ("sum0", "sum", 0), ("mean0", "mean", 0), ("max0", "max", 0), ("argmax0", "argmax", 0),
    ("sumall", "sum", None), ("minall", "min", None),
    ("argmin1", "argmin", 1), ("argmin0", "argmin", 0),
]


def reductions(R=16384, C=4096) -> list:
    ast = [_let("x", _fill((R, C)), (R, C)),
           _let("xa1", _fill((R, C)), (R, C)),   # copy with tied maxima per row
           _let("xa0", _fill((R, C)), (R, C)),   # copy with tied maxima per column
           _let("xi1", _fill((R, C)), (R, C)),   # tied minima per row
           _let("xi0", _fill((R, C)), (R, C))]   # tied minima per column
    src = {"argmax1": "xa1", "argmax0": "xa0", "argmin1": "xi1", "argmin0": "xi0"}
    for name, op, ax in REDUCTION_OPS:
        ast.append(_let(name, {"type": op, "tensor": src.get(name, "x"), "axis": ax}))
    ast.append(_let("sm", {"type": "softmax", "tensor": "x", "axis": 1}))
    ast.append(_let("ln", {"type": "layer_norm", "tensor": "x", "axis": 1, "eps": 0.00001}))
    return ast


def tie_copy(x: np.ndarray, axis: int, largest: bool, rng) -> np.ndarray:
    """Set 1% of each row (axis=1) / column (axis=0) to that line's extreme,
    at positions other than one kept original position."""
    y = x.copy()
    lines = y if axis == 1 else y.T
    n = lines.shape[1]
    k = max(1, n // 100)
    for i in range(lines.shape[0]):
        ext = lines[i].max() if largest else lines[i].min()
        keep = int(np.argmax(lines[i]) if largest else np.argmin(lines[i]))
        cand = rng.choice(n - 1, size=k, replace=False)
        cand = cand + (cand >= keep)
        lines[i, cand] = ext
    return np.ascontiguousarray(y)


def reductions_inputs(R=16384, C=4096, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, C)).astype(np.float32)
    return {"x": x,
            "xa1": tie_copy(x, 1, True, rng), "xa0": tie_copy(x, 0, True, rng),
            "xi1": tie_copy(x, 1, False, rng), "xi0": tie_copy(x, 0, False, rng)}


def unary_vjp(op="gelu", R=4096, C=4096) -> list:
    """``y = op(x); loss = mse_loss(y, T); backward(loss)`` with ``x`` tracked:
    the activation's forward and its VJP (autograd.py:540-561 for relu,
    sigmoid and tanh; gelu and swish have no reference VJP)."""
    return [
        _let("x", _fill((R, C)), (R, C), grad=True),
        _let("T", _fill((R, C)), (R, C)),
        _let("y", _call(op, "x")),
        _let("loss", _call("mse_loss", "y", "T")),
        {"type": "backward", "loss_tensor": "loss"},
    ]


def unary_vjp_inputs(R=4096, C=4096, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((R, C)) * 2.0).astype(np.float32)
    T = rng.standard_normal((R, C)).astype(np.float32)
    return {"x": x, "T": T}


def layer_norm_vjp(R=16384, C=4096, eps=0.00001) -> list:
    """``y = layer_norm(x, axis=1); loss = mse_loss(y, T); backward(loss)``:
    the row normalisation and its VJP (autograd.py:649-674)."""
    return [
        _let("x", _fill((R, C)), (R, C), grad=True),
        _let("T", _fill((R, C)), (R, C)),
        _let("y", {"type": "layer_norm", "tensor": "x", "axis": 1, "eps": float(eps)}),
        _let("loss", _call("mse_loss", "y", "T")),
        {"type": "backward", "loss_tensor": "loss"},
    ]


def layer_norm_vjp_inputs(R=16384, C=4096, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    # rows with their own offset and scale, so the VJP's mean and variance
    # terms both matter
    x = (rng.standard_normal((R, C)) * rng.uniform(0.5, 2.0, (R, 1))
         + rng.standard_normal((R, 1))).astype(np.float32)
    T = rng.standard_normal((R, C)).astype(np.float32)
    return {"x": x, "T": T}


def norms(R=16384, C=4096, eps=0.00001) -> list:
    """batch_norm with running statistics (kernel_generator.py:1978-2011) and
    instance_norm per row (:2017-2061) of one matrix."""
    return [
        _let("x", _fill((R, C)), (R, C)),
        _let("rm", _fill((C,)), (C,)),
        _let("rv", _fill((C,)), (C,)),
        _let("bn", {"type": "batch_norm", "tensor": "x", "running_mean": "rm",
                    "running_var": "rv", "eps": float(eps)}),
        _let("inn", {"type": "instance_norm", "tensor": "x", "eps": float(eps)}),
    ]


def norms_inputs(R=16384, C=4096, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((R, C)) * 1.5 + 0.25).astype(np.float32)
    rm = (rng.standard_normal(C) * 0.3).astype(np.float32)
    rv = rng.uniform(0.5, 3.0, C).astype(np.float32)
    return {"x": x, "rm": rm, "rv": rv}


# ---------------------------------------------------------------------------
# linear layer with autograd
# ---------------------------------------------------------------------------

def linear_layer(M=8192, K=4096, N=4096) -> list:
    return [
        _let("X", _fill((M, K)), (M, K), grad=True),
        _let("W", _fill((K, N)), (K, N), grad=True),
        _let("b", _fill((N,)), (N,), grad=True),
        _let("T", _fill((M, N)), (M, N)),
        _let("z", _call("linear", "X", "W", "b")),
        _let("y", _call("relu", "z")),
        _let("loss", _call("mse_loss", "y", "T")),
        {"type": "backward", "loss_tensor": "loss"},
    ]


def linear_layer_inputs(M=8192, K=4096, N=4096, seed=0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    T = rng.standard_normal((M, N)).astype(np.float32)
    return {"X": X, "W": W, "b": np.zeros(N, np.float32), "T": T}


# ---------------------------------------------------------------------------
# data-parallel MLP training loop
# ---------------------------------------------------------------------------

def mlp3_train(B=65536, I=1024, H=4096, C=10, epochs=100, lr=0.01) -> list:
    ast = [
        _let("x", _fill((B, I)), (B, I)),
        _let("t", _fill((B, C)), (B, C)),
        _let("W1", _fill((I, H)), (I, H), grad=True),
        _let("b1", _fill((H,)), (H,), grad=True),
        _let("W2", _fill((H, H)), (H, H), grad=True),
        _let("b2", _fill((H,)), (H,), grad=True),
        _let("W3", _fill((H, C)), (H, C), grad=True),
        _let("b3", _fill((C,)), (C,), grad=True),
        _let("lr", _lit([lr], (1, 1)), (1, 1)),
        _let("lr1", _lit([lr], (1,)), (1,)),
    ]
    body = [
        _let("h1", _call("linear", "x", "W1", "b1")),
        _let("a1", _call("relu", "h1")),
        _let("h2", _call("linear", "a1", "W2", "b2")),
        _let("a2", _call("relu", "h2")),
        _let("z", _call("linear", "a2", "W3", "b3")),
        _let("p", {"type": "softmax", "tensor": "z", "axis": 1}),
        _let("loss", _call("cross_entropy", "p", "t")),
        {"type": "backward", "loss_tensor": "loss"},
    ]
    params = [("W1", 2), ("b1", 1), ("W2", 2), ("b2", 1), ("W3", 2), ("b3", 1)]
    body += _sgd_lets(params)
    body += [{"type": "rebind", "name": p, "expr": {"type": "name", "name": f"{p}_new"}}
             for p, _ in params]
    ast.append({"type": "for", "loop_var": "epoch", "iterations": int(epochs), "body": body})
    return ast


def mlp3_inputs(B=65536, I=1024, H=4096, C=10, seed=0, rows=None) -> Dict[str, np.ndarray]:
    """Full-batch data; ``rows=(r0, r1)`` returns that contiguous shard of x and t
    (parameters are generated identically on every rank)."""
    rng = np.random.default_rng(seed)
    r0, r1 = rows if rows else (0, B)
    x = rng.standard_normal((B, I), dtype=np.float32)
    labels = rng.integers(0, C, B)
    W1 = (rng.standard_normal((I, H), dtype=np.float32) * np.float32(0.02))
    W2 = (rng.standard_normal((H, H), dtype=np.float32) * np.float32(0.02))
    W3 = (rng.standard_normal((H, C), dtype=np.float32) * np.float32(0.02))
    t = np.zeros((r1 - r0, C), np.float32)
    t[np.arange(r1 - r0), labels[r0:r1]] = 1.0
    return {"x": np.ascontiguousarray(x[r0:r1]), "t": t, "W1": W1, "b1": np.zeros(H, np.float32),
            "W2": W2, "b2": np.zeros(H, np.float32), "W3": W3, "b3": np.zeros(C, np.float32)}


# ---------------------------------------------------------------------------
# .tl source text of the same programs
# ---------------------------------------------------------------------------

def _ty(shape):
    return "Tensor[f32, (" + ", ".join(str(d) for d in shape) + (",)" if len(shape) == 1 else ")") + "]"


def tl_source(ast: list) -> str:
    """Render an AST built here as .tl text (the grammar of tensorlang.lark)."""
    def num(v):
        s = repr(float(v))
        if "e" in s or "E" in s:
            s = f"{float(v):.10f}".rstrip("0")
            if s.endswith("."):
                s += "0"
        return s

    def expr(e):
        t = e["type"]
        if t == "fill":
            return f"fill({num(e['value'])}, ({', '.join(str(d) for d in e['shape'])}" + \
                   ("," if len(e["shape"]) == 1 else "") + "))"
        if t == "tensor_literal":
            return None
        if "args" in e:
            return f"{t}({', '.join(e['args'])})"
        if t in ("softmax", "sum", "mean", "max", "min", "argmax", "argmin"):
            ax = e.get("axis")
            return f"{t}({e['tensor']}" + (f", axis={ax}" if ax is not None else "") + ")"
        if t == "layer_norm":
            return f"layer_norm({e['tensor']}, axis={e['axis']}, eps={num(e['eps'])})"
        raise ValueError(t)

    def stmt(n, ind=""):
        if n["type"] == "let":
            e = n["expr"]
            ty = f": {_ty(n['ty']['shape'])}" if n.get("ty") else ""
            if e["type"] == "tensor_literal":
                shape = n["ty"]["shape"]
                d = [num(v) for v in e["data"]]
                body = "[" + ", ".join(d) + "]" if len(shape) == 1 else \
                    "[" + ", ".join("[" + ", ".join(d[r * shape[1]:(r + 1) * shape[1]]) + "]"
                                    for r in range(shape[0])) + "]"
            else:
                body = expr(e)
            return f"{ind}let {n['name']}{ty} = {body}" + (" with grad" if n.get("requires_grad") else "")
        if n["type"] == "backward":
            return f"{ind}backward({n['loss_tensor']})"
        if n["type"] == "rebind":
            return f"{ind}{n['name']} = {n['expr']['name']}"
        if n["type"] == "for":
            inner = "\n".join(stmt(b, ind + "    ") for b in n["body"])
            return f"{ind}for {n['loop_var']} in range({n['iterations']}) {{\n{inner}\n{ind}}}"
        raise ValueError(n["type"])

    return "\n".join(stmt(n) for n in ast) + "\n"
