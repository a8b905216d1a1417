"""Reverse mode on the device: ``tensorlang/autograd.py`` as a step list.

The reference copies every tensor to the host, runs
``ComputationGraph.backward`` in NumPy and copies every gradient back, each
iteration of a training loop (tensorlang/compiler.py:237-289).  Here the same
recorded node list is turned, once, into a list of device steps:

* gradients flow only where the reference's would be non-zero: from the loss
  back through recorded nodes to tracked tensors (``with grad`` leaves and
  the outputs of recorded ops), autograd.py:100-228;
* each tracked tensor's gradient lives in ``<name>_grad``; the first
  contribution writes it, later ones accumulate (the reference zero-fills and
  accumulates, autograd.py:135-155, 317-333); tracked tensors that receive
  nothing are zero-filled;
* broadcast operands are reduced back to their shape the way
  ``_unbroadcast`` does (autograd.py:350-488): NumPy rules, prepended axes
  summed first;
* VJPs are the reference's (autograd.py:491-704): elementwise ones become
  fusable elementwise ops, matmul/linear become GEMMs with accumulate, softmax
  followed by cross_entropy becomes one fused row kernel, bias gradients are
  column reductions.

``divisors`` lets the data-parallel executor substitute the global batch for
the per-rank one in the cross_entropy and mse_loss VJPs (autograd.py:686,700),
so that the sum of the ranks' gradients equals the single-GPU gradient.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

from . import runtime as rt
from .shapes import Shape, numel
from .steps import EW, Copy, LibCall, Memset0, Step


class Node:
    __slots__ = ("op", "out", "ins", "meta")

    def __init__(self, op, out, ins, meta=None):
        self.op, self.out, self.ins, self.meta = op, out, list(ins), dict(meta or {})

    def __repr__(self):
        return f"Node({self.op}: {self.ins} -> {self.out})"


def grad_name(n: str) -> str:
    return f"{n}_grad"


class BackwardPlanner:
    def __init__(self, nodes: List[Node], requires: set, shapes: Dict[str, Shape],
                 prefix: str = "bw", divisors: Optional[Dict[str, float]] = None,
                 textbook_ce: bool = False):
        self.nodes = nodes
        # cross_entropy through a row softmax: the textbook (p - t) / B for the
        # logits instead of the reference's chained softmax VJP
        self.textbook_ce = textbook_ce
        self.requires = set(requires)
        self.shapes = shapes
        self.prefix = prefix
        self.divisors = divisors or {}
        self.steps: List[Step] = []
        self.written: Dict[str, int] = {}
        self._ntmp = 0

    # -- helpers -------------------------------------------------------------
    def _tmp(self, shape) -> str:
        name = f"__{self.prefix}{self._ntmp}"
        self._ntmp += 1
        self.shapes[name] = tuple(shape)
        return name

    def _ew(self, shape, opcode, operands) -> str:
        t = self._tmp(shape)
        self.steps.append(EW(t, shape, opcode, operands))
        return t

    def _first(self, target: str) -> bool:
        g = grad_name(target)
        first = self.written.get(g, 0) == 0
        self.written[g] = self.written.get(g, 0) + 1
        return first

    def _accumulate_value(self, target: str, value: str, vshape: Shape):
        """grad(target) (+)= unbroadcast(value) -- autograd.py:317-333, 350-488."""
        tshape = tuple(self.shapes[target])
        vshape = tuple(vshape)
        g = grad_name(target)
        self.shapes.setdefault(g, tshape)
        if vshape == tshape or numel(vshape) == numel(tshape) and _same_order(vshape, tshape):
            if self._first(target):
                self.steps.append(EW(g, tshape, "copy", [("name", value, "full")]))
            else:
                self.steps.append(EW(g, tshape, "add", [("name", g, "full"), ("name", value, "full")]))
            return
        first = self._first(target)
        dst = g if first else self._tmp(tshape)
        self._unbroadcast(value, vshape, dst, tshape)
        if not first:
            self.steps.append(EW(g, tshape, "add", [("name", g, "full"), ("name", dst, "full")]))

    def _unbroadcast(self, src: str, sshape: Shape, dst: str, tshape: Shape):
        """NumPy-rule reduction of ``src`` (shape sshape) to ``tshape`` into ``dst``."""
        sshape, tshape = tuple(sshape), tuple(tshape)
        target = (1,) if tshape == () else tshape
        lead = len(sshape) - len(target)
        if lead < 0:
            raise ValueError(f"unbroadcast {sshape} -> {tshape}")
        kept = sshape[lead:]
        summed_axes = list(range(lead)) + [lead + i for i, (a, b) in enumerate(zip(kept, target))
                                           if b == 1 and a != 1]
        for i, (a, b) in enumerate(zip(kept, target)):
            if b != 1 and a != b:
                raise ValueError(f"unbroadcast error: {sshape} -> {tshape}")
        nsum = numel(tuple(sshape[i] for i in summed_axes))
        n = numel(sshape)
        if nsum == n:  # everything summed
            self.steps.append(LibCall(f"unbcast_full:{dst}", "tl_reduce_full",
                                      [("int", rt.RED_SUM), ("ptr", src), ("ptr", dst), ("int", n),
                                       ("scratch",)], [src], [dst]))
            return
        # a leading block of axes summed -> column reduction; a trailing block -> rows
        if summed_axes == list(range(len(summed_axes))):
            rows = numel(tuple(sshape[:len(summed_axes)]))
            self.steps.append(LibCall(f"unbcast_cols:{dst}", "tl_reduce_cols",
                                      [("int", rt.RED_SUM), ("ptr", src), ("ptr", dst),
                                       ("int", rows), ("int", n // rows), ("scratch",)], [src], [dst]))
            return
        ns = len(sshape)
        if summed_axes == list(range(ns - len(summed_axes), ns)):
            cols = numel(tuple(sshape[ns - len(summed_axes):]))
            self.steps.append(LibCall(f"unbcast_rows:{dst}", "tl_reduce_rows",
                                      [("int", rt.RED_SUM), ("ptr", src), ("ptr", dst),
                                       ("int", n // cols), ("int", cols)], [src], [dst]))
            return
        raise NotImplementedError(f"gradient reduction {sshape} -> {tshape}")

    def _val(self, name, access=None):
        return ("name", name, access)

    # -- planning ------------------------------------------------------------
    def plan(self, loss: str) -> Tuple[List[Step], List[str]]:
        """Steps computing every tracked gradient for ``backward(loss)``."""
        shapes = self.shapes
        has_grad = {loss}
        active: List[Node] = []
        for node in reversed(self.nodes):
            if node.out in has_grad:
                active.append(node)
                for i in node.ins:
                    if i in self.requires:
                        has_grad.add(i)
        # seed: d loss / d loss = 1 (autograd.py:160)
        lg = grad_name(loss)
        shapes.setdefault(lg, tuple(shapes[loss]))
        self.steps.append(EW(lg, shapes[lg], "copy", [("const", 1.0)]))
        self.written[lg] = 1

        consumers: Dict[str, List[Node]] = {}
        for node in active:
            for i in node.ins:
                consumers.setdefault(i, []).append(node)
        fused_softmax = set()
        for node in active:
            if node.op == "cross_entropy":
                p = node.ins[0]
                prod = next((n for n in active if n.out == p and n.op == "softmax"), None)
                if prod is not None and len(consumers.get(p, [])) == 1 and \
                        len(shapes[p]) == 2 and prod.meta.get("axis") in (1, -1) and \
                        tuple(shapes[node.ins[1]]) in (tuple(shapes[p]), (shapes[p][0],)):
                    fused_softmax.add(p)

        for node in active:
            self._vjp(node, fused_softmax, active)

        exposed = sorted(n for n in self.requires if n in shapes and not n.startswith("__"))
        for n in exposed:
            g = grad_name(n)
            shapes.setdefault(g, tuple(shapes[n]))
            if self.written.get(g, 0) == 0:
                self.steps.append(Memset0(g))
                self.written[g] = 1
        return self.steps, exposed

    def _vjp(self, node: Node, fused_softmax: set, active: List[Node]):
        S = self.shapes
        op, out, ins = node.op, node.out, node.ins
        g = grad_name(out)
        oshape = tuple(S[out])
        req = self.requires

        if op in ("add", "minus"):
            a, b = ins
            if a in req:
                self._accumulate_value(a, g, oshape)
            if b in req:
                if op == "add":
                    self._accumulate_value(b, g, oshape)
                else:
                    t = self._ew(oshape, "neg", [self._val(g, "full")])
                    self._accumulate_value(b, t, oshape)
        elif op == "mult":
            a, b = ins
            if a in req:
                t = self._ew(oshape, "mult", [self._val(g, "full"), self._val(b)])
                self._accumulate_value(a, t, oshape)
            if b in req:
                t = self._ew(oshape, "mult", [self._val(g, "full"), self._val(a)])
                self._accumulate_value(b, t, oshape)
        elif op == "div":
            a, b = ins
            if a in req:
                t = self._ew(oshape, "div", [self._val(g, "full"), self._val(b)])
                self._accumulate_value(a, t, oshape)
            if b in req:
                # -g * a / b**2
                t1 = self._ew(oshape, "neg", [self._val(g, "full")])
                t2 = self._ew(oshape, "mult", [self._val(t1, "full"), self._val(a)])
                t3 = self._ew(oshape, "square", [self._val(b)])
                t4 = self._ew(oshape, "div", [self._val(t2, "full"), self._val(t3, "full")])
                self._accumulate_value(b, t4, oshape)
        elif op in ("matmul", "linear"):
            self._vjp_gemm(node)
        elif op in ("relu", "gelu", "swish"):
            x = ins[0]
            if x in req:
                opc = {"relu": "relu_mask", "gelu": "gelu_bwd", "swish": "swish_bwd"}[op]
                t = self._ew(oshape, opc, [self._val(g, "full"), self._val(x, "full")])
                self._accumulate_value(x, t, oshape)
        elif op in ("sigmoid", "tanh"):
            x = ins[0]
            if x in req:
                t = self._ew(oshape, f"{op}_bwd", [self._val(g, "full"), self._val(out, "full")])
                self._accumulate_value(x, t, oshape)
        elif op == "softmax":
            x = ins[0]
            if out in fused_softmax or x not in req:
                return
            ax = node.meta.get("axis")
            if len(oshape) == 1 or (len(oshape) == 2 and ax in (1, -1)):
                rows, cols = (1, oshape[0]) if len(oshape) == 1 else oshape
                first = self._first(x)
                gx = grad_name(x)
                S.setdefault(gx, tuple(S[x]))
                self.steps.append(LibCall(f"softmax_bwd:{gx}", "tl_softmax_backward_rows",
                                          [("ptr", out), ("ptr", g), ("ptr", gx), ("int", rows),
                                           ("int", cols), ("int", 0 if first else 1)],
                                          [out, g] + ([] if first else [gx]), [gx]))
            else:
                # axis=None on a 2-D tensor: the reference sums over every element
                t = self._ew(oshape, "mult", [self._val(g, "full"), self._val(out, "full")])
                tot = self._tmp(())
                self.steps.append(LibCall(f"softmax_bwd_sum:{tot}", "tl_reduce_full",
                                          [("int", rt.RED_SUM), ("ptr", t), ("ptr", tot),
                                           ("int", numel(oshape)), ("scratch",)], [t], [tot]))
                t2 = self._ew(oshape, "mult", [self._val(out, "full"), self._val(tot, "scalar")])
                t3 = self._ew(oshape, "minus", [self._val(t, "full"), self._val(t2, "full")])
                self._accumulate_value(x, t3, oshape)
        elif op in ("sum", "mean"):
            x = ins[0]
            if x not in req:
                return
            xs = tuple(S[x])
            ax = node.meta.get("axis")
            if ax is None:
                acc = "scalar"
            else:
                ax = int(ax) % len(xs)
                if len(xs) == 1:
                    acc = "scalar"
                elif len(xs) == 2:
                    acc = "row" if ax == 1 else "col"
                else:
                    raise NotImplementedError(f"{op} backward over axis {ax} of {xs}")
            if op == "sum":
                t = self._ew(xs, "copy", [self._val(g, acc)])
            else:
                cnt = numel(xs) if ax is None else xs[ax]
                t = self._ew(xs, "div", [self._val(g, acc), ("const", float(cnt))])
            self._accumulate_value(x, t, xs)
        elif op == "mse_loss":
            p, tgt = ins
            if p in req:
                n = self.divisors.get(("mse", out), float(numel(S[p])))
                ps = tuple(S[p])
                d = self._ew(ps, "minus", [self._val(p, "full"), self._val(tgt, "full")])
                d2 = self._ew(ps, "mult", [("const", 2.0), self._val(d, "full")])
                d3 = self._ew(ps, "div", [self._val(d2, "full"), ("const", float(n))])
                d4 = self._ew(ps, "mult", [self._val(d3, "full"), self._val(g, "scalar")])
                self._accumulate_value(p, d4, ps)
        elif op == "cross_entropy":
            self._vjp_ce(node, fused_softmax, active)
        elif op == "layer_norm":
            x = ins[0]
            if x not in req:
                return
            xs = tuple(S[x])
            ax = int(node.meta.get("axis", len(xs) - 1)) % len(xs)
            if ax != len(xs) - 1:
                raise NotImplementedError("layer_norm backward along a non-last axis")
            rows, cols = (1, xs[0]) if len(xs) == 1 else xs
            first = self._first(x)
            gx = grad_name(x)
            S.setdefault(gx, xs)
            self.steps.append(LibCall(f"layer_norm_bwd:{gx}", "tl_layer_norm_backward_rows",
                                      [("ptr", x), ("ptr", g), ("ptr", gx), ("int", rows),
                                       ("int", cols), ("float", float(node.meta.get("eps", 1e-5))),
                                       ("int", 0 if first else 1)],
                                      [x, g] + ([] if first else [gx]), [gx]))
        else:
            # the reference prints "No backward implemented" and skips (autograd.py:309-311)
            return

    def _vjp_gemm(self, node: Node):
        """matmul autograd.py:520-537; linear :619-646."""
        S = self.shapes
        g = grad_name(node.out)
        x, w = node.ins[0], node.ins[1]
        xs, ws, gs = tuple(S[x]), tuple(S[w]), tuple(S[node.out])
        if len(xs) == 1:  # vector input: treat as one row
            xs2, gs2 = (1, xs[0]), (1, gs[0])
        else:
            xs2, gs2 = xs, gs
        if len(ws) != 2 or len(xs2) != 2:
            raise NotImplementedError(f"{node.op} backward for {xs} @ {ws}")
        M, K = xs2
        N = ws[1]
        # parameter gradients (dW, db) first, then dX: in data-parallel training
        # a layer's weight gradient is then final before the (larger) dX product
        # of that layer runs, and its all-reduce overlaps that product
        if w in self.requires:  # dW[K,N] = X^T @ G
            first = self._first(w)
            gw = grad_name(w)
            S.setdefault(gw, ws)
            self.steps.append(LibCall(f"dW:{gw}", "tl_gemm",
                                      [("int", 1), ("int", 0), ("int", K), ("int", N), ("int", M),
                                       ("ptr", x), ("int", K), ("ptr", g), ("int", N), ("ptr", gw),
                                       ("int", N), ("null",), ("int", 0 if first else 1), ("int", 0)],
                                      [x, g] + ([] if first else [gw]), [gw]))
        if node.op == "linear" and len(node.ins) > 2 and node.ins[2] in self.requires:
            b = node.ins[2]
            bs = tuple(S[b])
            if len(gs) == 1:
                self._accumulate_value(b, g, gs)
            else:
                first = self._first(b)
                gb = grad_name(b)
                S.setdefault(gb, bs)
                dst = gb if first else self._tmp(bs)
                self.steps.append(LibCall(f"db:{gb}", "tl_reduce_cols",
                                          [("int", rt.RED_SUM), ("ptr", g), ("ptr", dst),
                                           ("int", gs[0]), ("int", gs[1]), ("scratch",)], [g], [dst]))
                if not first:
                    self.steps.append(EW(gb, bs, "add", [("name", gb, "full"), ("name", dst, "full")]))
        if x in self.requires:  # dX[M,K] = G[M,N] @ W^T
            first = self._first(x)
            gx = grad_name(x)
            S.setdefault(gx, xs)
            self.steps.append(LibCall(f"dX:{gx}", "tl_gemm",
                                      [("int", 0), ("int", 1), ("int", M), ("int", K), ("int", N),
                                       ("ptr", g), ("int", N), ("ptr", w), ("int", N), ("ptr", gx),
                                       ("int", K), ("null",), ("int", 0 if first else 1), ("int", 0)],
                                      [g, w] + ([] if first else [gx]), [gx]))

    def _vjp_ce(self, node: Node, fused_softmax: set, active: List[Node]):
        """cross_entropy autograd.py:691-704 (+ the softmax VJP when fused)."""
        S = self.shapes
        p, tgt = node.ins
        g = grad_name(node.out)
        ps, ts = tuple(S[p]), tuple(S[tgt])
        onehot = 1 if ts == ps else 0
        B = self.divisors.get(("ce", node.out), float(ps[0]))
        if p in fused_softmax and self.textbook_ce:
            # d loss / d z = (p - t) / B * g, in the order of the literal VJP's
            # minus, div, mult; p itself gets nothing from this path
            z = next(n for n in active if n.out == p and n.op == "softmax").ins[0]
            if z not in self.requires:
                return
            if not onehot:
                raise NotImplementedError("the textbook cross_entropy gradient takes one-hot targets")
            d = self._ew(ps, "minus", [self._val(p, "full"), self._val(tgt, "full")])
            d2 = self._ew(ps, "div", [self._val(d, "full"), ("const", float(B))])
            d3 = self._ew(ps, "mult", [self._val(d2, "full"), self._val(g, "scalar")])
            self._accumulate_value(z, d3, ps)
            return
        if p in fused_softmax:
            sm = next(n for n in active if n.out == p and n.op == "softmax")
            z = sm.ins[0]
            dp = grad_name(p) if p in self.requires else None
            if dp is not None:
                self.shapes.setdefault(dp, ps)
                if not self._first(p):
                    raise NotImplementedError("softmax output with several gradient sources")
            if z not in self.requires:
                return
            first = self._first(z)
            gz = grad_name(z)
            S.setdefault(gz, tuple(S[z]))
            args = [("ptr", p), ("ptr", tgt), ("int", onehot), ("ptr", g), ("float", float(B)),
                    ("ptr", dp) if dp else ("null",), ("ptr", gz), ("int", ps[0]), ("int", ps[1]),
                    ("int", 0 if first else 1)]
            writes = [gz] + ([dp] if dp else [])
            self.steps.append(LibCall(f"ce_softmax_bwd:{gz}", "tl_ce_softmax_backward", args,
                                      [p, tgt, g] + ([] if first else [gz]), writes))
            return
        if p not in self.requires:
            return
        if not onehot:
            raise NotImplementedError("cross_entropy backward with class-index targets outside a "
                                      "softmax -> cross_entropy pair")
        d = self._ew(ps, "minus", [self._val(p, "full"), self._val(tgt, "full")])
        d2 = self._ew(ps, "div", [self._val(d, "full"), ("const", float(B))])
        d3 = self._ew(ps, "mult", [self._val(d2, "full"), self._val(g, "scalar")])
        self._accumulate_value(p, d3, ps)


def _same_order(a: Shape, b: Shape) -> bool:
    """Shapes that differ only by size-1 axes enumerate elements in the same order."""
    return tuple(d for d in a if d != 1) == tuple(d for d in b if d != 1)
