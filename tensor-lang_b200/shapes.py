"""Output-shape rules of the TensorLang ops on the execution path.

The reference computes these in ``tensorlang/type_checker.py`` (per-op rules
at :100-781, gradient tensors at :541-571 and :783-825).  The backend needs
them itself to (a) fill in shapes the checker's environment lacks (gradient
tensors, programs assembled without the reference frontend) and (b) re-derive
per-rank shapes when a training loop is sharded across GPUs.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np

Shape = Tuple[int, ...]


def _t(s) -> Shape:
    return tuple(int(d) for d in s)


def broadcast(s1: Shape, s2: Shape) -> Shape:
    n = max(len(s1), len(s2))
    a = (1,) * (n - len(s1)) + tuple(s1)
    b = (1,) * (n - len(s2)) + tuple(s2)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ValueError(f"shapes {s1} and {s2} do not broadcast")
        out.append(max(x, y))
    return tuple(out)


def slice_bounds(spec: dict, size: int) -> Tuple[int, int]:
    """Python-exclusive end, clamped (kernel_generator.py:1125-1160)."""
    t = spec.get("type")
    if t == "slice":
        s, e = spec.get("start"), spec.get("end")
        s = 0 if s is None else int(s)
        e = size if e is None else int(e)
    elif t == "index":
        s = int(spec["value"])
        e = s + 1
    else:
        s, e = 0, size
    s = max(0, min(s, size))
    e = max(s, min(e, size))
    return s, e


def expr_inputs(expr: dict) -> List[str]:
    t = expr["type"]
    if "args" in expr:
        return list(expr["args"])
    if t == "concat":
        return list(expr["tensors"])
    if t == "batch_norm":
        return [expr["tensor"], expr["running_mean"], expr["running_var"]]
    if "tensor" in expr:
        return [expr["tensor"]]
    if t == "name":
        return [expr["name"]]
    return []


def out_shape(expr: dict, shapes: Dict[str, Shape]) -> Shape:
    t = expr["type"]
    if t in ("add", "minus", "mult", "div", "greater", "less", "equal"):
        s1, s2 = _t(shapes[expr["args"][0]]), _t(shapes[expr["args"][1]])
        if s1 == s2 or (len(s1) == 2 and len(s2) == 1):
            return s1
        if len(s1) == 1 and len(s2) == 1 and s2[0] == 1:
            return s1
        return broadcast(s1, s2)
    if t in ("relu", "sigmoid", "tanh", "gelu", "swish"):
        return _t(shapes[expr["args"][0]])
    if t == "fill":
        return _t(expr["shape"])
    if t == "matmul":
        a, b = _t(shapes[expr["args"][0]]), _t(shapes[expr["args"][1]])
        if len(a) == 2 and len(b) == 2:
            return (a[0], b[1])
        if len(a) == 2 and len(b) == 1:
            return (a[0],)
        if len(a) == 1 and len(b) == 2:
            return (b[1],)
        raise ValueError(f"matmul shapes {a} @ {b}")
    if t == "linear":
        x, w = _t(shapes[expr["args"][0]]), _t(shapes[expr["args"][1]])
        return (w[1],) if len(x) == 1 else (x[0], w[1])
    if t in ("softmax", "layer_norm", "batch_norm", "instance_norm"):
        return _t(shapes[expr["tensor"]])
    if t in ("sum", "mean", "max", "min", "argmax", "argmin"):
        s = _t(shapes[expr["tensor"]])
        ax = expr.get("axis")
        if ax is None:
            return ()
        ax = int(ax) % len(s)
        return tuple(d for i, d in enumerate(s) if i != ax)
    if t in ("mse_loss", "cross_entropy"):
        return ()
    if t == "transpose":
        s = _t(shapes[expr["tensor"]])
        axes = expr.get("axes")
        return tuple(s[int(i)] for i in axes) if axes else tuple(reversed(s))
    if t == "reshape":
        return _t(expr["new_shape"])
    if t == "concat":
        ss = [_t(shapes[n]) for n in expr["tensors"]]
        ax = int(expr.get("axis") or 0)
        o = list(ss[0])
        o[ax] = sum(s[ax] for s in ss)
        return tuple(o)
    if t == "slice":
        s = _t(shapes[expr["tensor"]])
        specs = expr["specs"]
        res = []
        for i, d in enumerate(s):
            spec = specs[i] if i < len(specs) else {"type": "full_slice"}
            a, b = slice_bounds(spec, d)
            res.append(b - a)
        return tuple(res)
    if t == "name":
        return _t(shapes[expr["name"]])
    if t == "tensor_literal":
        n = len(expr["data"])
        return (n,)
    raise ValueError(f"no shape rule for op {t}")


def numel(shape: Shape) -> int:
    return int(np.prod(shape)) if len(shape) else 1


def complete_env(ast: list, env: Dict[str, dict]) -> Dict[str, Shape]:
    """Shapes for every name the program defines, plus ``<name>_grad``."""
    shapes: Dict[str, Shape] = {k: _t(v["shape"]) for k, v in (env or {}).items()}
    for k in list(shapes):
        if not k.endswith("_grad"):
            shapes.setdefault(f"{k}_grad", shapes[k])

    def visit(nodes):
        for n in nodes:
            if n["type"] == "for":
                visit(n["body"])
                continue
            if n["type"] != "let":
                continue
            name = n["name"]
            e = n.get("expr")
            if name not in shapes and isinstance(e, dict):
                ty = n.get("ty")
                if isinstance(ty, dict) and ty.get("shape") is not None:
                    shapes[name] = _t(ty["shape"])
                else:
                    shapes[name] = out_shape(e, shapes)
                shapes.setdefault(f"{name}_grad", shapes[name])

    visit(ast)
    for k in list(shapes):
        if not k.endswith("_grad") and f"{k}_grad" not in shapes:
            shapes[f"{k}_grad"] = shapes[k]
    return shapes
