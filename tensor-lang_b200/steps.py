"""Executable steps of a lowered program and the kernel_info dispatch.

``kinfo_to_step`` is this backend's ``TensorCompiler._execute_single_kernel``
(tensorlang/compiler.py:365-673): it switches on ``kernel_info[0]`` and turns
the tuple into either an elementwise op (``EW``, fused later into a region
kernel) or a call into libtlb200 (``LibCall``).  Steps only name tensors;
pointers are bound once, after allocation, so a bound program can be captured
into a CUDA graph and replayed.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from . import runtime as rt
from . import views as V
from .region import Region, Seg, classify
from .shapes import Shape, numel


class Step:
    label = "step"
    reads: List[str] = []
    writes: List[str] = []

    def bind(self, P) -> Callable[[], None]:
        raise NotImplementedError

    def compile(self, P):
        pass


class EW(Step):
    """One elementwise op over the iteration shape ``shape``.

    operands: ("name", tensor, access) with access in full|row|col|scalar|None
    (None = NumPy broadcasting), ("map", m) -- a view read through the index
    map ``m`` (``views.py``) -- or ("const", value).
    """

    def __init__(self, out: str, shape: Shape, opcode: str, operands: list, label: str = ""):
        self.out, self.shape, self.opcode, self.operands = out, tuple(shape), opcode, operands
        self.label = label or f"{opcode}:{out}"
        self.writes = [out]
        self._set_reads()

    def _set_reads(self):
        reads = []
        for o in self.operands:
            if o[0] == "name":
                reads.append(o[1])
            elif o[0] == "map":
                reads += [n for n in V.leaves(o[1]) if n not in reads]
        self.reads = reads


class LibCall(Step):
    """A libtlb200 entry point.

    args: ("ptr", name) | ("int", v) | ("float", v) | ("scratch",) | ("bytes", name)
          | ("null",)
    The stream argument is appended.
    """

    def __init__(self, label: str, fname: str, args: list, reads: Sequence[str],
                 writes: Sequence[str]):
        self.label, self.fname, self.args = label, fname, args
        self.reads, self.writes = list(reads), list(writes)

    def bind(self, P):
        fn = getattr(rt.lib(), self.fname)
        vals = []
        for a in self.args:
            k = a[0]
            if k == "ptr":
                vals.append(c_void_p(P.ptr(a[1])))
            elif k == "int":
                vals.append(a[1])
            elif k == "float":
                vals.append(c_float(a[1]))
            elif k == "scratch":
                vals.append(c_void_p(P.scratch_ptr))
            elif k == "bytes":
                vals.append(ctypes.c_size_t(P.buffers[P.alias.get(a[1], a[1])].nbytes))
            elif k == "null":
                vals.append(c_void_p(None))
            elif k == "handle":
                vals.append(c_void_p(a[1]() if callable(a[1]) else a[1]))
            elif k == "size":
                vals.append(ctypes.c_size_t(a[1]))
            else:
                raise ValueError(k)
        vals.append(P.stream)
        vals = tuple(vals)
        label = self.label

        def run():
            st = fn(*vals)
            if st:
                rt.check(st, label)
        return run


class Copy(Step):
    def __init__(self, dst: str, src: str):
        self.dst, self.src = dst, src
        self.reads, self.writes = [src], [dst]
        self.label = f"copy:{dst}<-{src}"

    def bind(self, P):
        d, s = P.ptr(self.dst), P.ptr(self.src)
        nbytes = 4 * numel(P.shapes[self.dst])
        L, stream = rt.lib(), P.stream
        if d == s:
            return lambda: None

        def run():
            rt.check(L.tl_memcpy_d2d(d, s, nbytes, stream), self.label)
        return run


class Memset0(Step):
    def __init__(self, name: str):
        self.name = name
        self.reads, self.writes = [], [name]
        self.label = f"zero:{name}"

    def bind(self, P):
        p, nbytes = P.ptr(self.name), 4 * numel(P.shapes[self.name])
        L, stream = rt.lib(), P.stream

        def run():
            rt.check(L.tl_memset(p, 0, nbytes, stream), self.label)
        return run


class RegionStep(Step):
    """A fused elementwise kernel (one or more segments)."""

    def __init__(self, region: Region, key_of: Dict[str, str], reads, writes):
        self.region = region
        self.key_of = key_of          # region key -> tensor name
        self.reads, self.writes = list(reads), list(writes)
        self.label = region.label

    def compile(self, P):
        self.region.compile(P.dev)

    def bind(self, P):
        ptrs = {k: P.ptr(n) for k, n in self.key_of.items()}
        bound = self.region.bind(ptrs)
        region, stream = self.region, P.stream
        return lambda: region.launch(bound, stream)


class ViewStep(Step):
    """A movement op (slice, transpose, reshape, concat).  ``resolve_views``
    either folds it into the elementwise kernels that read it, as an index map
    (``views.py``), or writes it: with ``fallback`` (the dedicated library
    kernel or copy) when its inputs are in memory, else as a region copy
    through the composed map."""

    def __init__(self, view: V.View, fallback: Step):
        self.view, self.fallback = view, fallback
        self.out = view.out
        self.reads, self.writes = list(view.sources), [view.out]
        self.label = f"{view.kind}:{view.out}"

    def bind(self, P):  # only reached when fusion is bypassed
        return self.fallback.bind(P)

    def compile(self, P):
        self.fallback.compile(P)


# ---------------------------------------------------------------------------
# kernel_info -> step
# ---------------------------------------------------------------------------

_BIN = ("add", "minus", "mult", "div")
_CMP = ("greater", "less", "equal")
_UNARY = ("relu", "sigmoid", "tanh", "gelu", "swish")


def _vec_access(out_shape: Shape, arg_shape: Shape) -> str:
    """Access of a 1-D compare/binary operand that the reference reads as B[j]."""
    if numel(arg_shape) == 1:
        return "scalar"
    return "col"


def kinfo_to_step(k: tuple, shapes: Dict[str, Shape], divisor_scale: Optional[dict] = None) -> Step:
    kind = k[0]
    if kind == "general_broadcast":
        _, op, name, a, b, _p1, _p2, out, _tot = k
        return EW(name, shapes[name], op, [("name", a, None), ("name", b, None)])
    name = k[1]
    out = shapes[name]
    if kind in _BIN + _CMP and len(k) == 5:  # same shape (elementwise :246-275, compare :646-778)
        return EW(name, out, kind, [("name", k[2], "full"), ("name", k[3], "full")])
    if kind.endswith("_scalar") and kind.split("_")[0] in _BIN:  # binary_1d_broadcast :354-377
        a, b = k[2], k[3]
        if numel(shapes[b]) == 1:
            ops = [("name", a, "full"), ("name", b, "scalar")]
        else:  # scalar first operand: broadcast it
            ops = [("name", a, "scalar"), ("name", b, "full")]
        return EW(name, out, kind.split("_")[0], ops)
    if kind.endswith("_broadcast_rows"):  # B[i], :303-325
        return EW(name, out, kind.split("_")[0], [("name", k[2], "full"), ("name", k[3], "row")])
    if kind in ("add_broadcast", "minus_broadcast", "mult_broadcast", "div_broadcast",
                "greater_broadcast", "less_broadcast") or (kind == "equal" and len(k) == 6):
        op = kind.split("_")[0]
        b = k[3]
        return EW(name, out, op, [("name", k[2], "full"), ("name", b, _vec_access(out, shapes[b]))])
    if kind == "fill":  # :469-488
        return EW(name, out, "copy", [("const", float(k[5]))])
    if kind in _UNARY:
        return EW(name, out, kind, [("name", k[2], "full")])

    R = rt
    if kind == "matmul":  # :501-525
        a, b = k[2], k[3]
        m, n, p = (int(v) for v in k[4:7])
        sa, sb = shapes[a], shapes[b]
        if len(sa) == 2 and len(sb) == 2:
            M, K, N = sa[0], sa[1], sb[1]
            return LibCall(f"matmul:{name}", "tl_gemm",
                           [("int", 0), ("int", 0), ("int", M), ("int", N), ("int", K),
                            ("ptr", a), ("int", K), ("ptr", b), ("int", N), ("ptr", name),
                            ("int", N), ("null",), ("int", 0), ("int", 0)], [a, b], [name])
        if len(sa) == 2 and len(sb) == 1:  # matrix-vector
            M, K = sa
            return LibCall(f"matmul:{name}", "tl_gemm",
                           [("int", 0), ("int", 0), ("int", M), ("int", 1), ("int", K),
                            ("ptr", a), ("int", K), ("ptr", b), ("int", 1), ("ptr", name),
                            ("int", 1), ("null",), ("int", 0), ("int", 0)], [a, b], [name])
        if len(sa) == 1 and len(sb) == 2:
            K, N = sb
            return LibCall(f"matmul:{name}", "tl_gemm",
                           [("int", 0), ("int", 0), ("int", 1), ("int", N), ("int", K),
                            ("ptr", a), ("int", K), ("ptr", b), ("int", N), ("ptr", name),
                            ("int", N), ("null",), ("int", 0), ("int", 0)], [a, b], [name])
        raise NotImplementedError(f"matmul {sa} @ {sb}")
    if kind in ("linear_1d", "linear_2d"):  # :1584-1661
        x, w, bias = k[2], k[3], k[4]
        if kind == "linear_1d":
            M, K, N = 1, int(k[5]), int(k[6])
        else:
            M, K, N = int(k[5]), int(k[6]), int(k[7])
        return LibCall(f"linear:{name}", "tl_gemm",
                       [("int", 0), ("int", 0), ("int", M), ("int", N), ("int", K),
                        ("ptr", x), ("int", K), ("ptr", w), ("int", N), ("ptr", name),
                        ("int", N), ("ptr", bias), ("int", 0), ("int", 0)], [x, w, bias], [name])
    if kind == "softmax":  # :564-640
        rows, cols = int(k[4]), int(k[5])
        return LibCall(f"softmax:{name}", "tl_softmax_rows",
                       [("ptr", k[2]), ("ptr", name), ("int", rows), ("int", cols)], [k[2]], [name])
    if kind == "softmax_1d":
        return LibCall(f"softmax:{name}", "tl_softmax_rows",
                       [("ptr", k[2]), ("ptr", name), ("int", 1), ("int", int(k[4]))], [k[2]], [name])
    red = {"sum": R.RED_SUM, "mean": R.RED_MEAN, "max": R.RED_MAX, "min": R.RED_MIN,
           "argmax": R.RED_ARGMAX, "argmin": R.RED_ARGMIN}
    base = kind.split("_")[0]
    if base in red and (kind.endswith("_full") or kind.endswith("_axis") or kind.endswith("_axis0")):
        op, t = red[base], k[2]
        if kind.endswith("_full") or (kind == "argmax_axis" and len(k) == 5):
            n = numel(shapes[t])
            return LibCall(f"{base}:{name}", "tl_reduce_full",
                           [("int", op), ("ptr", t), ("ptr", name), ("int", n), ("scratch",)],
                           [t], [name])
        rows, cols = int(k[4]), int(k[5])
        if kind.endswith("_axis0"):
            return LibCall(f"{base}0:{name}", "tl_reduce_cols",
                           [("int", op), ("ptr", t), ("ptr", name), ("int", rows), ("int", cols),
                            ("scratch",)], [t], [name])
        return LibCall(f"{base}1:{name}", "tl_reduce_rows",
                       [("int", op), ("ptr", t), ("ptr", name), ("int", rows), ("int", cols)],
                       [t], [name])
    if kind in ("layer_norm_2d", "instance_norm_2d", "layer_norm_1d"):  # :1667-1810, :2017-2061
        t = k[2]
        if kind == "layer_norm_1d":
            rows, cols, eps = 1, int(k[4]), float(k[5])
        elif kind == "instance_norm_2d":
            rows, cols, eps = int(k[5]), int(k[6]), float(k[7])
        else:
            rows, cols, eps = int(k[4]), int(k[5]), float(k[6])
        return LibCall(f"{kind}:{name}", "tl_layer_norm_rows",
                       [("ptr", t), ("ptr", name), ("int", rows), ("int", cols), ("float", eps)],
                       [t], [name])
    if kind == "layer_norm_axis0":
        t, rows, cols, eps = k[2], int(k[4]), int(k[5]), float(k[6])
        return LibCall(f"layer_norm0:{name}", "tl_layer_norm_cols",
                       [("ptr", t), ("ptr", name), ("int", rows), ("int", cols), ("float", eps),
                        ("scratch",)], [t], [name])
    if kind == "batch_norm_2d":  # :1978-2011
        t, rm, rows, cols, eps, rv = k[2], k[3], int(k[4]), int(k[5]), float(k[6]), k[7]
        return LibCall(f"batch_norm:{name}", "tl_batch_norm",
                       [("ptr", t), ("ptr", rm), ("ptr", rv), ("ptr", name), ("int", rows),
                        ("int", cols), ("float", eps)], [t, rm, rv], [name])
    if kind in ("cross_entropy", "cross_entropy_onehot"):  # :1816-1885
        p, t, B, C = k[2], k[3], int(k[4]), int(k[5])
        return LibCall(f"cross_entropy:{name}", "tl_cross_entropy",
                       [("ptr", p), ("ptr", t), ("ptr", name), ("int", B), ("int", C),
                        ("int", 1 if kind.endswith("onehot") else 0), ("scratch",)], [p, t], [name])
    if kind == "mse_loss":  # :1891-1943
        p, t, n = k[2], k[3], int(k[4])
        return LibCall(f"mse_loss:{name}", "tl_mse_loss",
                       [("ptr", p), ("ptr", t), ("ptr", name), ("int", n), ("scratch",)],
                       [p, t], [name])
    if kind == "transpose_2d":  # :1949-1972
        t, rows, cols = k[2], int(k[4]), int(k[5])
        lib = LibCall(f"transpose:{name}", "tl_transpose2d",
                      [("ptr", t), ("ptr", name), ("int", rows), ("int", cols)], [t], [name])
        return ViewStep(V.View("transpose", name, out, [t], ()), lib)
    if kind == "reshape":  # :2067-2086
        return ViewStep(V.View("reshape", name, out, [k[2]], ()), Copy(name, k[2]))
    if kind == "slice_2d":  # :1112-1198
        t, rows, cols, r0, r1, c0, c1, orows, ocols = k[2], *[int(v) for v in k[4:12]]
        lib = LibCall(f"slice:{name}", "tl_slice2d",
                      [("ptr", t), ("ptr", name), ("int", cols), ("int", r0), ("int", c0),
                       ("int", orows), ("int", ocols)], [t], [name])
        return ViewStep(V.View("slice", name, out, [t], (r0, c0)), lib)
    if kind == "slice_1d":  # :1200-1240
        t, start, n = k[2], int(k[4]), int(k[5])
        lib = LibCall(f"slice:{name}", "tl_slice2d",
                      [("ptr", t), ("ptr", name), ("int", max(1, start + n)), ("int", 0),
                       ("int", start), ("int", 1 if n > 0 else 0), ("int", n)], [t], [name])
        return ViewStep(V.View("slice", name, out, [t], (start,)), lib)
    if kind == "concat_axis0":  # :2092-2132
        a, b, r1, r2, cols = k[2], k[3], int(k[4]), int(k[5]), int(k[6])
        lib = LibCall(f"concat:{name}", "tl_concat_rows",
                      [("ptr", a), ("ptr", b), ("ptr", name), ("int", r1), ("int", r2),
                       ("int", cols)], [a, b], [name])
        return ViewStep(V.View("concat0", name, out, [a, b], ()), lib)
    raise NotImplementedError(f"no backend dispatch for kernel_info {k[0]!r}")


# ---------------------------------------------------------------------------
# fusion
# ---------------------------------------------------------------------------

def fuse(steps: List[Step], shapes: Dict[str, Shape], live: set, read_count: Dict[str, int],
         label: str = "region", horizontal: bool = True,
         canon: Optional[Dict[str, str]] = None) -> List[Step]:
    """Merge runs of same-shape EW ops into region kernels.

    A value produced inside a run is written to memory only if it is in
    ``live`` (fetched, saved, rebound) or some read of that name is not an
    in-run consumer of it (``read_count`` counts reads over the whole program,
    loops and backward included).  With ``horizontal``, neighbouring runs with
    no data hazard between them become segments of one launch.  ``canon``
    maps a name to the tensor whose buffer it shares (in-place updates).
    """
    steps = resolve_views(steps, shapes, live, read_count, canon or {})
    out: List[Step] = []
    run: List[EW] = []

    def flush():
        if run:
            out.append(_RunMarker(list(run)))
            run.clear()

    for st in steps:
        if isinstance(st, EW):
            if run and run[0].shape != st.shape:
                flush()
            elif run and _maps_read_run(st, run):
                flush()  # a view of a value this run computes: written first
            run.append(st)
        else:
            flush()
            out.append(st)
    flush()

    merged: List = []
    for st in out:
        if isinstance(st, _RunMarker) and horizontal and merged and isinstance(merged[-1], _RunGroup):
            grp = merged[-1]
            if not grp.hazard(st, canon or {}):
                grp.runs.append(st)
                continue
        if isinstance(st, _RunMarker):
            merged.append(_RunGroup([st]))
        else:
            merged.append(st)

    result: List[Step] = []
    for st in merged:
        if isinstance(st, _RunGroup):
            result.append(st.build(shapes, live, read_count, label, canon or {}))
        else:
            result.append(st)
    return result


def _maps_read_run(st: EW, run: List[EW]) -> bool:
    written = {op.out for op in run}
    return any(o[0] == "map" and set(V.leaves(o[1])) & written for o in st.operands)


def resolve_views(steps: List[Step], shapes: Dict[str, Shape], live: set,
                  read_count: Dict[str, int], canon: Dict[str, str]) -> List[Step]:
    """Fold each ``ViewStep`` into the elementwise steps that read it, as an
    index map, or write it where it stands.

    A view folds when nothing else needs it in memory: it is not live, every
    read of it in the whole program is by a later step of this list that is
    either an elementwise op reading it element for element (same shape,
    ``full`` access) or another view that composes with it, and no step up to
    its last reader writes the tensors the map reads."""
    c = lambda n: canon.get(n, n)  # noqa: E731
    maps: Dict[str, tuple] = {}
    out: List[Step] = []
    for i, st in enumerate(steps):
        if isinstance(st, ViewStep):
            v = st.view
            in_maps = [maps.get(src) or V.identity(shapes[src], src) for src in v.sources]
            m = v.build(in_maps, [shapes[src] for src in v.sources])
            if m is not None and _view_folds(v.out, m, steps, i, shapes, live, read_count, c):
                maps[v.out] = m
                continue
            if m is None or any(src in maps for src in v.sources):
                if m is None:
                    raise NotImplementedError(f"{st.label}: a view of a view that does not compose")
                out.append(EW(v.out, v.out_shape, "copy", [("map", m)], label=f"{st.label}(map)"))
            else:
                out.append(st.fallback)
            continue
        if isinstance(st, EW) and any(o[0] == "name" and o[1] in maps for o in st.operands):
            ops = [("map", maps[o[1]]) if o[0] == "name" and o[1] in maps else o
                   for o in st.operands]
            st = EW(st.out, st.shape, st.opcode, ops, label=st.label)
        out.append(st)
    return out


def _view_folds(name, m, steps, i, shapes, live, read_count, c) -> bool:
    if name in live:
        return False
    shape = tuple(shapes[name])
    nreads, last = 0, i
    for j in range(i + 1, len(steps)):
        st = steps[j]
        n = st.reads.count(name)
        if not n:
            continue
        nreads += n
        last = j
        if isinstance(st, ViewStep):
            if st.view.kind == "reshape" and not V.is_whole(m, shape):
                return False
            continue
        if not isinstance(st, EW) or tuple(st.shape) != shape:
            return False
        if any(o[0] == "name" and o[1] == name and o[2] != "full" for o in st.operands):
            return False
    if nreads == 0 or nreads != read_count.get(name, 0):
        return False
    srcs = {c(n) for n in V.leaves(m)}
    return not any(c(w) in srcs for st in steps[i + 1:last + 1] for w in st.writes)


class _RunMarker:
    def __init__(self, ops: List[EW]):
        self.ops = ops
        self.reads = set()
        self.writes = set()
        defined = set()
        for op in ops:
            for r in op.reads:
                if r not in defined:
                    self.reads.add(r)
            defined.add(op.out)
            self.writes.add(op.out)


class _RunGroup:
    def __init__(self, runs: List[_RunMarker]):
        self.runs = runs

    def hazard(self, other: _RunMarker, canon: Dict[str, str]) -> bool:
        c = lambda names: {canon.get(n, n) for n in names}  # noqa: E731
        ow, orr = c(other.writes), c(other.reads)
        for r in self.runs:
            rw, rr = c(r.writes), c(r.reads)
            if rw & orr or rr & ow or rw & ow:
                return True
        return False

    def build(self, shapes, live, read_count, label, canon) -> RegionStep:
        segs = []
        key_of: Dict[str, str] = {}
        name_key: Dict[str, str] = {}
        reads, writes = set(), set()

        def key(name):
            base = canon.get(name, name)
            if base not in name_key:
                k = f"k{len(name_key)}"
                name_key[base] = k
                key_of[k] = name
            return name_key[base]

        labels = []
        for run in self.runs:
            shape = run.ops[0].shape
            seg = Seg(shape)
            cur = {}       # name -> Ref of its latest in-run value
            consumed = {}  # name -> reads served from the in-run value
            for op in run.ops:
                args = []
                for o in op.operands:
                    if o[0] == "const":
                        args.append(seg.const(o[1]))
                        continue
                    if o[0] == "map":
                        keyed = V.rename(o[1], key)
                        ref = seg.add_input(None, shape, "map", keyed)
                        reads.update(V.leaves(o[1]))
                        args.append(ref)
                        continue
                    nm, acc = o[1], o[2]
                    if nm in cur and numel(shapes[nm]) == numel(shape):
                        args.append(cur[nm])
                        consumed[nm] = consumed.get(nm, 0) + 1
                        continue
                    if acc is None:
                        ref = seg.add_input(key(nm), shapes[nm])
                    else:
                        ref = seg.add_input(key(nm), shapes[nm], acc)
                    reads.add(nm)
                    args.append(ref)
                r = seg.op(op.opcode, *args)
                cur[op.out] = r
            for nm, ref in cur.items():
                external = read_count.get(nm, 0) - consumed.get(nm, 0)
                if nm in live or external > 0:
                    seg.output(key(nm), ref)
                    writes.add(nm)
            if not seg.outputs:
                last = run.ops[-1].out
                seg.output(key(last), cur[last])
                writes.add(last)
            segs.append(seg)
            labels.append("+".join(op.opcode for op in run.ops))
        region = Region(segs, label=f"{label}[{';'.join(labels)}]")
        return RegionStep(region, key_of, reads, writes)
