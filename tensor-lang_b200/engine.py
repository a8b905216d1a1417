"""Program executor: the execution half of ``TensorCompiler.compile_and_execute``.

Mirrors the reference's phases (tensorlang/compiler.py:1481-1661):

1. every ``let`` is lowered in program order through ``KernelGenerator``
   (compiler.py:996-1424; ``for`` bodies as in ``_generate_kernels_for_nodes``
   :725-765) and autograd operations are recorded as ``_record_operation``
   does (:47-54);
2. top-level statements before the first top-level ``backward`` run in order,
   ``for`` loops included (:1527-1560);
3. each top-level ``backward`` computes gradients (:1597-1635);
4. top-level kernels after it run (:1640-1648), then ``save`` statements.

Differences that are the point of this backend: results stay on the device
(no device-to-host copy per kernel, :675-685), backward runs on the device,
elementwise runs are fused, a ``for`` body is captured once as a CUDA graph
and replayed, and a rebind (:309-347) updates a parameter in place when the
update is elementwise instead of swapping buffers.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Dict, Iterable, List, Optional

import numpy as np

from . import runtime as rt
from .autograd import BackwardPlanner, Node, grad_name
from .dataio import check_shape, load_data_file
from .epilogue import fuse_gemm_epilogues
from .head import fuse_classifier_head
from .pairs import fuse_bias_colsums, plan_gemm_pairs
from .kernel_generator import KernelGenerator
from .shapes import Shape, broadcast, complete_env, expr_inputs, numel
from .steps import EW, Copy, LibCall, Memset0, RegionStep, Step, fuse, kinfo_to_step

KERNEL_FREE = ("name", "tensor_literal", "load")
RECORDED_REFERENCE = {"add", "minus", "mult", "div", "matmul", "relu", "sigmoid", "tanh",
                      "softmax", "sum", "mean", "mse_loss"}
RECORDED_EXTENDED = RECORDED_REFERENCE | {"linear", "cross_entropy", "layer_norm", "gelu", "swish"}


def lower_let(name: str, expr: dict, shapes: Dict[str, Shape], gen: KernelGenerator) -> tuple:
    """Choose the generator method exactly as compiler.py:1110-1424 does."""
    t = expr["type"]
    if t in ("add", "minus", "mult", "div"):
        a, b = expr["args"]
        s1, s2, out = tuple(shapes[a]), tuple(shapes[b]), tuple(shapes[name])
        if s1 == s2:
            return gen.elementwise(t, name, a, b, numel(out))[1]
        if len(s1) == 2 and len(s2) == 1:
            return gen.binary_broadcast(t, t, name, a, b, s1, s2, out)[1]
        if len(s1) == 1 and len(s2) == 1 and (s1[0] == 1 or s2[0] == 1):
            return gen.binary_1d_broadcast(t, name, a, b, numel(out))[1]
        broadcast(s1, s2)  # raises like compiler.py:1180-1184 when incompatible
        return gen.binary_general_broadcast(t, name, a, b, s1, s2, out)[1]
    if t == "fill":
        return gen.fill("fill", name, None, None, numel(tuple(expr["shape"])), expr["value"])[1]
    if t == "matmul":
        a, b = expr["args"]
        sa, sb = shapes[a], shapes[b]
        if len(sa) == 2 and len(sb) == 2:
            m, n, p = sa[0], sa[1], sb[1]
        elif len(sa) == 2 and len(sb) == 1:
            m, n, p = sa[0], sa[1], sb[0]
        elif len(sa) == 1 and len(sb) == 2:
            m, n, p = 1, sa[0], sb[1]
        else:
            raise TypeError(f"Unsupported matmul shapes: {sa} @ {sb}")
        return gen.matmul("matmul", name, a, b, int(m), int(n), int(p))[1]
    if t in ("relu", "sigmoid", "tanh", "gelu", "swish"):
        a = expr["args"][0]
        return getattr(gen, t)(t, name, a, numel(shapes[a]))[1]
    if t == "softmax":
        return gen.softmax("softmax", name, expr["tensor"], shapes[expr["tensor"]], expr.get("axis"))[1]
    if t in ("greater", "less", "equal"):
        a, b = expr["args"]
        s1, s2, out = shapes[a], shapes[b], shapes[name]
        if t == "greater":
            return gen.greater_broadcast(t, name, a, b, s1, s2, out, numel(out))[1]
        if t == "less":
            return gen.less_broadcast(t, name, a, b, s1, s2, out)[1]
        return gen.equal(t, name, a, b, s1, s2, out)[1]
    if t in ("sum", "mean", "max", "min", "argmax", "argmin"):
        return getattr(gen, t)(t, name, expr["tensor"], expr.get("axis"), shapes[expr["tensor"]])[1]
    if t == "slice":
        return gen.slice("slice", name, expr["tensor"], expr["specs"], shapes[expr["tensor"]],
                         shapes[name])[1]
    if t == "linear":
        x, w, b = expr["args"]
        return gen.linear("linear", name, x, w, b, shapes[x], shapes[w], shapes[name])[1]
    if t == "layer_norm":
        eps = expr.get("eps")
        return gen.layer_norm("layer_norm", name, expr["tensor"], expr.get("axis"),
                              1e-5 if eps is None else eps, shapes[expr["tensor"]])[1]
    if t == "cross_entropy":
        p, q = expr["args"]
        return gen.cross_entropy("cross_entropy", name, p, shapes[p], shapes[q], q)[1]
    if t == "mse_loss":
        p, q = expr["args"]
        return gen.mse_loss("mse_loss", name, p, q, numel(shapes[p]))[1]
    if t == "transpose":
        return gen.transpose("transpose", name, shapes[expr["tensor"]], expr["tensor"])[1]
    if t == "reshape":
        return gen.reshape("reshape", name, expr["tensor"], numel(shapes[expr["tensor"]]))[1]
    if t == "concat":
        env = {k: {"shape": v} for k, v in shapes.items()}
        return gen.concat("concat", name, expr["tensors"], expr["axis"], env)[1]
    if t == "batch_norm":
        eps = expr.get("eps")
        return gen.batch_norm("batch_norm", name, shapes[expr["tensor"]], expr["tensor"],
                              expr["running_mean"], 1e-5 if eps is None else eps,
                              expr["running_var"])[1]
    if t == "instance_norm":
        eps = expr.get("eps")
        return gen.instance_norm("instance_norm", name, expr["tensor"], shapes[expr["tensor"]],
                                 1e-5 if eps is None else eps)[1]
    raise NotImplementedError(f"op {t} has no lowering")


class _Loop(Step):
    """A ``for`` statement: body phases, rebinds, CUDA-graph replay.

    ``hoisted`` holds steps on values the body never writes (for example the
    GEMM operand pairs of a loop-invariant input); they run before the body on
    every eager run and are not part of the captured per-iteration graph."""

    def __init__(self, iterations: int, pre: List[Step], bw: List[Step], post: List[Step],
                 rebind: List[Step], label: str):
        self.iterations = int(iterations)
        self.pre, self.bw, self.post, self.rebind = pre, bw, post, rebind
        self.hoisted: List[Step] = []
        self.label = label
        self.reads = sorted({r for s in self.body() for r in s.reads})
        self.writes = sorted({w for s in self.body() for w in s.writes})
        self.graph = None
        self.graph_nodes = (0, 0)

    def body(self) -> List[Step]:
        return self.pre + self.bw + self.post + self.rebind

    def steps(self) -> List[Step]:
        """Everything the loop runs: hoisted steps, then the body."""
        return self.hoisted + self.body()

    def compile(self, P):
        for s in self.steps():
            s.compile(P)

    def bind(self, P):
        self._hoisted_calls = [s.bind(P) for s in self.hoisted]
        self._calls = [s.bind(P) for s in self.body()]
        self._stream = P.stream
        self._use_graph = P.use_graphs
        return lambda: self.iterate(self.iterations, first=True)

    def run_hoisted(self):
        """Re-run the hoisted steps, for a caller that has rewritten a
        loop-invariant input (a new batch) between iterations."""
        for c in self._hoisted_calls:
            c()

    def run_eager(self):
        """One iteration, kernel by kernel (after the hoisted steps)."""
        self.run_hoisted()
        for c in self._calls:
            c()

    def capture(self):
        """Record one iteration into a CUDA graph (nothing executes)."""
        if self.graph is not None:
            return
        rt.check(rt.lib().tl_graph_begin(self._stream), "graph_begin")
        try:
            for c in self._calls:
                c()
        finally:
            ge = ctypes.c_void_p()
            rt.check(rt.lib().tl_graph_end(self._stream, ctypes.byref(ge)), "graph_end")
        self.graph = ge.value
        k, pr = ctypes.c_int(), ctypes.c_int()
        rt.check(rt.lib().tl_graph_last_stats(ctypes.byref(k), ctypes.byref(pr)), "graph_stats")
        self.graph_nodes = (k.value, pr.value)  # kernel nodes, of them prioritised

    def replay(self, n: int = 1):
        L = rt.lib()
        for _ in range(n):
            rt.check(L.tl_graph_launch(self.graph, self._stream), "graph_launch")

    def iterate(self, n: int, first: bool = False):
        """Run ``n`` iterations: the first eagerly (it also warms caches), the
        rest as replays of one captured graph."""
        if n <= 0:
            return
        if first or not self._use_graph:
            self.run_eager()
            n -= 1
        if n <= 0:
            return
        if not self._use_graph:
            for _ in range(n):
                self.run_eager()
            return
        self.capture()
        self.replay(n)

    def release(self):
        if self.graph is not None:
            rt.lib().tl_graph_destroy(self.graph)
            self.graph = None


class Program:
    """A lowered TensorLang program bound to one device.

    ast/env: the reference frontend's output (``ast_builder.build_ast`` and
    ``type_checker.type_checker``).  ``feeds`` replaces initial values of
    named tensors; ``fetch`` names the tensors the caller will read (None =
    every named tensor, like the reference's cache of every result); anything
    else may be fused away.

    ``semantics="reference"`` (default) keeps the reference's literal rules;
    ``"numpy"`` switches two of them to the textbook ones: a square 2-D op
    1-D broadcast reads ``B[j]`` as NumPy does (the reference reads ``B[i]``
    whenever the row counts match, kernel_generator.py:303-348), and the
    gradient of cross_entropy through a row softmax is ``(p - t) / B``
    (the reference chains the softmax VJP after cross_entropy's,
    autograd.py:563-580, 691-704).  One-hot targets only in that mode.
    """

    def __init__(self, ast: list, env: Optional[dict] = None, *, device: int = 0,
                 feeds: Optional[Dict[str, np.ndarray]] = None, fetch: Optional[Iterable[str]] = None,
                 load_files: Optional[Dict[str, np.ndarray]] = None, record: str = "extended",
                 use_graphs: bool = True, fuse_ops: bool = True, fuse_head: bool = True,
                 fuse_colsum: bool = True,
                 save_dir: Optional[str] = None,
                 shapes: Optional[Dict[str, Shape]] = None, divisors: Optional[dict] = None,
                 grad_hook=None, semantics: str = "reference"):
        if semantics not in ("reference", "numpy"):
            raise ValueError(f"semantics must be 'reference' or 'numpy', not {semantics!r}")
        self.semantics = semantics
        self.ast = ast
        self.device_index = int(device)
        self.shapes: Dict[str, Shape] = dict(shapes) if shapes else complete_env(ast, env or {})
        self.feeds = {k: np.asarray(v, dtype=np.float32) for k, v in (feeds or {}).items()}
        self.fetch = None if fetch is None else list(fetch)
        self.load_files = load_files or {}
        self.recorded = RECORDED_EXTENDED if record == "extended" else RECORDED_REFERENCE
        self.use_graphs = use_graphs
        self.fuse_ops = fuse_ops
        self.fuse_head = fuse_head  # classifier-head fusion (head.py), with fuse_ops
        self.fuse_colsum = fuse_colsum  # bias sums folded into pair steps (pairs.py)
        self.save_dir = Path(save_dir) if save_dir else Path.cwd()
        self.divisors = divisors or {}
        self.grad_hook = grad_hook  # (program, exposed grads, backward steps) -> backward steps
        self.arena_names: List[str] = []  # allocated contiguously (one all-reduce span)
        self.gen = KernelGenerator(False, numpy_broadcast=semantics == "numpy")
        self.nodes: List[Node] = []
        self.requires: set = set()
        self.kinfos: List[tuple] = []
        self.initial: Dict[str, np.ndarray] = {}
        self.exposed_grads: List[str] = []
        self.top_grads: List[str] = []
        self.buffers: Dict[str, rt.DeviceBuffer] = {}
        self.alias: Dict[str, str] = {}
        self.dev = None
        self.stream = None
        self.scratch = None
        self.scratch_ptr = None
        self._calls = None
        self._lower()

    # -------------------------------------------------------------- lowering
    def _record(self, op, out, ins, meta=None):
        if op in self.recorded and any(i in self.requires for i in ins):
            self.nodes.append(Node(op, out, ins, meta))
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
                ax = len(self.shapes[e["tensor"]]) - 1
            eps = e.get("eps")
            meta = {"axis": int(ax), "eps": 1e-5 if eps is None else float(eps)}
        self._record(t, node["name"], expr_inputs(e), meta)

    def _literal_value(self, node) -> np.ndarray:
        name, e = node["name"], node["expr"]
        shp = self.shapes[name]
        if name in self.feeds:
            return self.feeds[name].reshape(shp)
        if e["type"] == "tensor_literal":
            return np.asarray(e["data"], dtype=np.float32).reshape(shp)
        if e["type"] == "load":
            src = self.load_files.get(e["file_path"])
            if src is not None:
                return np.asarray(src, dtype=np.float32).reshape(shp)
            data, _meta = load_data_file(e["file_path"], e.get("array_name"))
            return check_shape(name, e["file_path"], data, shp)
        raise ValueError(e["type"])

    def _let_step(self, node) -> Optional[Step]:
        name, e = node["name"], node["expr"]
        if name in self.feeds and e["type"] == "fill":
            self.initial[name] = self.feeds[name].reshape(self.shapes[name])
            return None
        k = lower_let(name, e, self.shapes, self.gen)
        self.kinfos.append(k)
        return kinfo_to_step(k, self.shapes)

    def _lower(self):
        ast = self.ast
        # codegen pass: literals, autograd recording, kernel_info per let
        self._let_steps: Dict[int, Step] = {}
        loops: Dict[int, dict] = {}
        for i, node in enumerate(ast):
            typ = node["type"]
            if typ == "for":
                body_steps = {}
                for j, b in enumerate(node["body"]):
                    if b["type"] != "let" or not isinstance(b.get("expr"), dict):
                        continue
                    if b["expr"]["type"] in ("tensor_literal", "load"):
                        self.initial[b["name"]] = self._literal_value(b)
                    elif b["expr"]["type"] == "name":
                        body_steps[j] = Copy(b["name"], b["expr"]["name"])
                    else:
                        self._record_let(b)
                        st = self._let_step(b)
                        if st is not None:
                            body_steps[j] = st
                loops[i] = body_steps
                continue
            if typ != "let":
                continue
            if node.get("requires_grad"):
                self.requires.add(node["name"])
            e = node.get("expr")
            if not isinstance(e, dict):
                continue
            if e["type"] in ("tensor_literal", "load"):
                self.initial[node["name"]] = self._literal_value(node)
            elif e["type"] == "name":
                self._let_steps[i] = Copy(node["name"], e["name"])
            else:
                self._record_let(node)
                st = self._let_step(node)
                if st is not None:
                    self._let_steps[i] = st

        # phases
        bw_idx = next((i for i, n in enumerate(ast) if n["type"] == "backward"), None)
        self.phase_pre: List[Step] = []
        self.phase_bw: List[Step] = []
        self.phase_post: List[Step] = []
        nbw = 0
        for i, node in enumerate(ast):
            if bw_idx is not None and i > bw_idx:
                if i in self._let_steps:
                    self.phase_post.append(self._let_steps[i])
                continue
            if node["type"] == "for" and (bw_idx is None or i < bw_idx):
                self.phase_pre.append(self._build_loop(node, loops[i], f"L{i}"))
            elif i in self._let_steps:
                self.phase_pre.append(self._let_steps[i])
        if bw_idx is not None:
            for node in ast:
                if node["type"] == "backward":
                    planner = BackwardPlanner(self.nodes, self.requires, self.shapes,
                                              prefix=f"tb{nbw}_", divisors=self.divisors,
                                              textbook_ce=self.semantics == "numpy")
                    nbw += 1
                    steps, exposed = planner.plan(node["loss_tensor"])
                    self.phase_bw += steps
                    self.top_grads = sorted(set(self.top_grads) | set(exposed))
                    self.exposed_grads = sorted(set(self.exposed_grads) | set(exposed))
        self.saves = [n for n in ast if n["type"] == "save"]

    def _build_loop(self, node, body_steps: Dict[int, Step], label: str) -> _Loop:
        body = node["body"]
        bw = next((j for j, b in enumerate(body) if b["type"] == "backward"), None)
        pre = [body_steps[j] for j in sorted(body_steps) if bw is None or j < bw]
        post = [body_steps[j] for j in sorted(body_steps) if bw is not None and j > bw]
        bw_steps: List[Step] = []
        if bw is not None:
            planner = BackwardPlanner(self.nodes, self.requires, self.shapes, prefix=f"{label}b_",
                                      divisors=self.divisors,
                                      textbook_ce=self.semantics == "numpy")
            bw_steps, exposed = planner.plan(body[bw]["loss_tensor"])
            self.exposed_grads = sorted(set(self.exposed_grads) | set(exposed))
            if self.grad_hook is not None:
                bw_steps = self.grad_hook(self, exposed, bw_steps)
        rebinds = [b for b in body if b["type"] == "rebind" and b["expr"].get("type") == "name"]
        reb_steps = self._plan_rebinds(rebinds, pre + bw_steps + post)
        return _Loop(int(node["iterations"]), pre, bw_steps, post, reb_steps, label)

    def _plan_rebinds(self, rebinds, body: List[Step]) -> List[Step]:
        """compiler.py:309-347 swaps buffer pointers.  Here: when the new value
        is produced elementwise and the old value is not read after that, the
        producer writes in place (same buffer); otherwise the value is copied
        at the end of the iteration.  Either way pointers stay fixed, so the
        loop body can be replayed as one CUDA graph."""
        targets = {r["name"]: r["expr"]["name"] for r in rebinds}
        srcs = set(targets.values())
        steps: List[Step] = []
        if srcs & set(targets):
            # a = b; b = a  -> simultaneous assignment through temporaries
            tmps = {}
            for t, s in targets.items():
                tmp = f"__rebind_{t}"
                self.shapes[tmp] = self.shapes[t]
                tmps[t] = tmp
                steps.append(Copy(tmp, s))
            for t in targets:
                steps.append(Copy(t, tmps[t]))
            return steps
        for t, s in targets.items():
            prod_idx = max((i for i, st in enumerate(body) if s in st.writes), default=None)
            ok = prod_idx is not None and isinstance(body[prod_idx], EW) and \
                tuple(self.shapes[t]) == tuple(self.shapes[s]) and \
                not any(t in st.reads for st in body[prod_idx + 1:]) and \
                not any(t in st.writes for st in body) and \
                not any(s in st.reads for st in body[:prod_idx]) and \
                s not in self.alias and t not in self.alias.values()
            if ok:
                self.alias[s] = t  # s lives in t's buffer
            else:
                steps.append(Copy(t, s))
        return steps

    # -------------------------------------------------------------- binding
    def _all_steps(self) -> List[Step]:
        out = []

        def walk(lst):
            for s in lst:
                if isinstance(s, _Loop):
                    walk(s.steps())
                else:
                    out.append(s)
        walk(self.phase_pre + self.phase_bw + self.phase_post)
        return out

    def _fuse_all(self):
        if self.fuse_ops:
            fuse_gemm_epilogues(self)
            if self.fuse_head:
                fuse_classifier_head(self)
            plan_gemm_pairs(self)
            if self.fuse_colsum:
                fuse_bias_colsums(self)
        live = set(self.shapes) if self.fetch is None else set(self.fetch)
        live |= set(self.initial)
        live |= {sv["tensor"] for sv in self.saves}
        if self.fetch is None:
            live |= {grad_name(g) for g in self.exposed_grads}
        read_count: Dict[str, int] = {}
        for s in self._all_steps():
            for r in s.reads:
                read_count[r] = read_count.get(r, 0) + 1
        # a rebound value lives on in its target's buffer (the in-place
        # update of a parameter); any other value a loop writes is kept only
        # if some step reads it, or the caller fetches or saves it
        live |= set(self.alias)
        self.live = live

        def dead_zero(st) -> bool:
            # a gradient that receives nothing is zero-filled (autograd.py:151-153);
            # when nothing reads or keeps it, the fill is skipped
            return isinstance(st, Memset0) and st.name not in live and \
                read_count.get(st.name, 0) == 0

        def fz(lst, label):
            res, chunk = [], []
            lst = [st for st in lst if not dead_zero(st)]

            def flush():
                if not chunk:
                    return
                if self.fuse_ops:
                    res.extend(fuse(chunk, self.shapes, live, read_count, label, canon=self.alias))
                else:
                    for st in chunk:
                        if isinstance(st, EW):
                            res.extend(fuse([st], self.shapes, live | {st.out}, read_count, label,
                                            horizontal=False, canon=self.alias))
                        else:
                            res.append(st)
                chunk.clear()

            for s in lst:
                if isinstance(s, _Loop):
                    flush()
                    s.hoisted = fz(s.hoisted, s.label + "h")
                    s.pre = fz(s.pre, s.label + "f")
                    s.bw = fz(s.bw, s.label + "b")
                    s.post = fz(s.post, s.label + "p")
                    s.rebind = fz(s.rebind, s.label + "r")
                    res.append(s)
                else:
                    chunk.append(s)
            flush()
            return res

        self.phase_pre = fz(self.phase_pre, "pre")
        self.phase_bw = fz(self.phase_bw, "bw")
        self.phase_post = fz(self.phase_post, "post")

    def ptr(self, name: str) -> int:
        return self.buffers[self.alias.get(name, name)].ptr

    def prepare(self):
        """Allocate, upload initial values, compile regions, bind pointers."""
        if self._calls is not None:
            return
        self.dev = rt.Device.get(self.device_index)
        self.stream = self.dev.stream
        self._fuse_all()
        needed = set(self.initial)
        for s in self._all_steps():
            needed.update(s.reads)
            needed.update(s.writes)
        if self.fetch is not None:
            needed.update(n for n in self.fetch if n in self.shapes)
        if self.arena_names:
            bases = []
            for n in self.arena_names:
                b = self.alias.get(n, n)
                if b not in bases:
                    bases.append(b)
            # 64-float (256-byte) aligned slots: every tensor keeps the
            # alignment TMA and vector loads need; the padding is all-reduced too
            pad = lambda n: (n + 63) // 64 * 64  # noqa: E731
            total = sum(pad(numel(self.shapes[b])) for b in bases)
            self._arena = rt.DeviceBuffer(self.dev, (total,), zero=True)
            off = 0
            for b in bases:
                self.buffers[b] = rt.DeviceBuffer.view(self._arena, off, self.shapes[b])
                off += pad(numel(self.shapes[b]))
        for n in sorted(needed):
            base = self.alias.get(n, n)
            if base in self.buffers:
                continue
            if base not in self.shapes:
                raise KeyError(f"no shape known for tensor {base!r}")
            self.buffers[base] = rt.DeviceBuffer(self.dev, self.shapes[base])
        for n, v in self.initial.items():
            self.buffers[self.alias.get(n, n)].upload(v)
        scratch_bytes = self._scratch_bytes()
        self.scratch = rt.DeviceBuffer(self.dev, (max(scratch_bytes // 4, 1),), zero=True)
        self.scratch_ptr = self.scratch.ptr
        for s in self.phase_pre + self.phase_bw + self.phase_post:
            s.compile(self)
        self._calls = [s.bind(self) for s in self.phase_pre + self.phase_bw + self.phase_post]
        self.dev.sync()

    def _scratch_bytes(self) -> int:
        L = rt.lib()
        need = 1 << 16
        for s in self._all_steps():
            if not isinstance(s, LibCall) or not any(a[0] == "scratch" for a in s.args):
                continue
            f = s.fname
            a = s.args
            if f == "tl_reduce_cols":
                need = max(need, L.tl_reduce_cols_scratch_bytes(a[0][1], a[3][1], a[4][1]))
            elif f == "tl_reduce_full":
                need = max(need, L.tl_reduce_full_scratch_bytes(a[0][1], a[3][1]))
            elif f == "tl_layer_norm_cols":
                need = max(need, L.tl_norm_cols_scratch_bytes(a[2][1], a[3][1]))
            elif f in ("tl_mse_loss", "tl_cross_entropy"):
                need = max(need, L.tl_loss_scratch_bytes(1))
        return int(need)

    def execute(self):
        """Enqueue the whole program on the device stream (no host sync)."""
        self.prepare()
        for c in self._calls:
            c()

    def sync(self):
        self.dev.sync()

    # -------------------------------------------------------------- results
    def read(self, name: str) -> np.ndarray:
        return self.buffers[self.alias.get(name, name)].download()

    def run(self) -> Dict[str, np.ndarray]:
        """Execute and return the fetched tensors (and ``<name>.grad`` for the
        gradients of a top-level backward, as the reference caches them)."""
        self.execute()
        self.sync()
        if self.fetch is not None:
            names = self.fetch
        else:
            # every value the program names (the frontend's own temporaries,
            # such as inlined function results, included), none of the
            # backend's internal buffers
            lets = self._let_names()
            names = [n for n in self.buffers if not n.startswith("__") or n in lets] + \
                [a for a in self.alias if not a.startswith("__") or a in lets]
        out = {}
        for n in names:
            base = self.alias.get(n, n)
            if base in self.buffers:
                out[n] = self.read(n)
        for g in self.top_grads:
            gn = grad_name(g)
            if gn in out:
                out[f"{g}.grad"] = out[gn]
            elif self.alias.get(gn, gn) in self.buffers:
                out[f"{g}.grad"] = self.read(gn)
        for sv in self.saves:
            if sv["tensor"] in self.shapes and self.alias.get(sv["tensor"], sv["tensor"]) in self.buffers:
                p = Path(sv["file_path"])
                if not p.is_absolute():
                    p = self.save_dir / p
                p.parent.mkdir(parents=True, exist_ok=True)
                np.save(p, self.read(sv["tensor"]))
        return out

    def _let_names(self) -> set:
        out = set()

        def walk(nodes):
            for n in nodes:
                if n.get("type") == "for":
                    walk(n["body"])
                elif n.get("type") == "let":
                    out.add(n["name"])
        walk(self.ast)
        return out

    def arena_span(self):
        """(pointer, float count) of the packed gradient arena, or None."""
        a = getattr(self, "_arena", None)
        return (a.ptr, a.size) if a is not None else None

    @property
    def loops(self) -> List[_Loop]:
        return [s for s in self.phase_pre if isinstance(s, _Loop)]

    def free(self):
        for lp in self.loops:
            lp.release()
        for b in self.buffers.values():
            b.free()
        if getattr(self, "_arena", None) is not None:
            self._arena.free()
            self._arena = None
        self.buffers.clear()
        if self.scratch is not None:
            self.scratch.free()
            self.scratch = None
