"""Fused elementwise regions: IR and sm_100a CUDA code generation.

The reference emits one kernel per elementwise op, each a separate launch
with ``cudaDeviceSynchronize`` and a full device-to-host copy of its result
(kernel_generator.py:209-488, 646-778; compiler.py:675-685).  Here a run of
elementwise ops over one iteration shape becomes a single *segment*, and
independent segments (for example the SGD update of every parameter) share
one kernel launch.  Intermediates that nothing else reads live only in
registers.

Operand access rules follow the reference's lowering (compiler.py:1155-1186):

* same shape                -> ``full``    (element e)
* 2-D op 1-D, s1[0]==s2[0]  -> ``row``     (B[i], binary_broadcast :303-325)
* 2-D op 1-D otherwise      -> ``col``     (B[j], :327-348)
* 1-D op (1,)               -> ``scalar``  (B[0], binary_1d_broadcast :354-377)
* anything else             -> NumPy broadcasting (binary_general_broadcast
  :383-463), classified into the cheapest of the above when possible, else
  a ``strided`` gather with zero strides on broadcast axes.

Arithmetic is IEEE float32 with every binary op rounded separately
(``__fadd_rn`` and friends) -- the reference computes each op in its own
kernel, so no multiply-add contraction may merge them.

Generated kernels are compiled by NVRTC inside libtlb200 (``tl_jit_compile``)
for ``sm_100a`` and cached by content hash under ``_jit/``.
"""
from __future__ import annotations

import ctypes
import hashlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import runtime as rt
from . import views as V

BLOCK = 256
UNROLL = 1          # units per thread per loop trip (more raised register use and lost
                    # occupancy on B200: 1 unit at 16 blocks/SM measured fastest)
BLOCKS_PER_SM = 16  # grid size cap, as a multiple of the SM count

# opcode -> (arity, C expression template over a, b, c)
OPS = {
    "add": (2, "__fadd_rn({a}, {b})"),
    "minus": (2, "__fsub_rn({a}, {b})"),
    "mult": (2, "__fmul_rn({a}, {b})"),
    "div": (2, "__fdiv_rn({a}, {b})"),
    "relu": (1, "fmaxf(0.0f, {a})"),
    "sigmoid": (1, "__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-{a})))"),
    "tanh": (1, "tanhf({a})"),
    # gelu(x) = x * Phi(x), Phi(x) = erfc(-x/sqrt(2))/2: no cancellation for x < 0
    "gelu": (1, "__fmul_rn(__fmul_rn(0.5f, {a}), erfcf(__fmul_rn(-{a}, 0.70710678118654752f)))"),
    "swish": (1, "__fdiv_rn({a}, __fadd_rn(1.0f, expf(-{a})))"),
    "greater": (2, "(({a}) > ({b}) ? 1.0f : 0.0f)"),
    "less": (2, "(({a}) < ({b}) ? 1.0f : 0.0f)"),
    "equal": (2, "(fabsf(__fsub_rn({a}, {b})) < 1e-6f ? 1.0f : 0.0f)"),
    "neg": (1, "(-({a}))"),
    "copy": (1, "({a})"),
    # reverse-mode helpers (tensorlang/autograd.py VJPs)
    "relu_mask": (2, "__fmul_rn({a}, ({b}) > 0.0f ? 1.0f : 0.0f)"),          # g * (x > 0)
    "sigmoid_bwd": (2, "__fmul_rn(__fmul_rn({a}, {b}), __fsub_rn(1.0f, {b}))"),  # g*s*(1-s)
    "tanh_bwd": (2, "__fmul_rn({a}, __fsub_rn(1.0f, __fmul_rn({b}, {b})))"),    # g*(1-y^2)
    "gelu_bwd": (2, "__fmul_rn({a}, __fadd_rn(__fmul_rn(0.5f, erfcf(__fmul_rn(-{b}, "
                    "0.70710678118654752f))), __fmul_rn(__fmul_rn({b}, 0.39894228040143268f), "
                    "expf(__fmul_rn(-0.5f, __fmul_rn({b}, {b}))))))"),
    "swish_bwd": (2, "tl_swish_bwd({a}, {b})"),
    "square": (1, "__fmul_rn({a}, {a})"),
}

PRELUDE = r"""
__device__ __forceinline__ float4 tl_ld4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float4 tl_ldc4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void tl_st4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
__device__ __forceinline__ float tl_swish_bwd(float g, float x) {
  float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  return __fmul_rn(g, __fadd_rn(s, __fmul_rn(__fmul_rn(x, s), __fsub_rn(1.0f, s))));
}
"""


@dataclass
class Ref:
    kind: str  # "in" | "tmp" | "const"
    idx: int = 0
    value: float = 0.0


@dataclass
class Input:
    key: Optional[str]
    access: str            # full | row | col | scalar | strided | map
    strides: Tuple[int, ...] = ()  # for strided: per output axis, in elements
    mapspec: tuple = ()    # for map: a views.py index map over buffer keys

    def keys(self) -> List[str]:
        return V.leaves(self.mapspec) if self.access == "map" else [self.key]


@dataclass
class Seg:
    """One iteration space: ``shape`` elements, each computed independently."""

    shape: Tuple[int, ...]
    inputs: List[Input] = field(default_factory=list)
    body: List[Tuple[str, List[Ref]]] = field(default_factory=list)
    outputs: List[Tuple[str, Ref]] = field(default_factory=list)

    @property
    def total(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def add_input(self, key: Optional[str], in_shape: Sequence[int], access: Optional[str] = None,
                  mapspec: tuple = ()) -> Ref:
        in_shape = tuple(int(d) for d in in_shape)
        if access is None:
            access, strides = classify(self.shape, in_shape)
        else:
            strides = ()
        for i, inp in enumerate(self.inputs):
            if inp.key == key and inp.access == access and inp.strides == strides \
                    and inp.mapspec == mapspec:
                return Ref("in", i)
        self.inputs.append(Input(key, access, strides, tuple(mapspec)))
        return Ref("in", len(self.inputs) - 1)

    def const(self, v: float) -> Ref:
        return Ref("const", value=float(v))

    def op(self, opcode: str, *args: Ref) -> Ref:
        if opcode not in OPS:
            raise ValueError(f"unknown elementwise opcode {opcode}")
        if len(args) != OPS[opcode][0]:
            raise ValueError(f"{opcode} takes {OPS[opcode][0]} operands")
        self.body.append((opcode, list(args)))
        return Ref("tmp", len(self.body) - 1)

    def output(self, key: str, ref: Ref):
        self.outputs.append((key, ref))

    def signature(self) -> str:
        parts = [f"S{self.shape}"]
        for i in self.inputs:
            parts.append(f"I{i.access}{i.strides}{i.mapspec}")
        for opc, args in self.body:
            parts.append(opc + "(" + ",".join(f"{a.kind}{a.idx}{a.value!r}" for a in args) + ")")
        for k, r in self.outputs:
            parts.append(f"O{r.kind}{r.idx}{r.value!r}")
        return "|".join(parts)


def classify(out_shape: Tuple[int, ...], in_shape: Tuple[int, ...]) -> Tuple[str, Tuple[int, ...]]:
    """NumPy-broadcast access of ``in_shape`` over ``out_shape``."""
    n = len(out_shape)
    if tuple(in_shape) == tuple(out_shape):
        return "full", ()
    if int(np.prod(in_shape)) == 1:
        return "scalar", ()
    pad = (1,) * (n - len(in_shape)) + tuple(in_shape)
    if len(pad) != n:
        raise ValueError(f"cannot broadcast {in_shape} to {out_shape}")
    for a, b in zip(pad, out_shape):
        if a != b and a != 1:
            raise ValueError(f"cannot broadcast {in_shape} to {out_shape}")
    if n >= 2:
        lead = int(np.prod(out_shape[:-1]))
        # varies only along the last axis
        if all(d == 1 for d in pad[:-1]) and pad[-1] == out_shape[-1]:
            return "col", ()
        # varies only along the leading axes, constant along the last
        if pad[-1] == 1 and tuple(pad[:-1]) == tuple(out_shape[:-1]) and lead > 0:
            return "row", ()
    strides = []
    acc = 1
    for d in reversed(pad):
        strides.append(0 if d == 1 else acc)
        acc *= d
    strides.reverse()
    return "strided", tuple(int(s) for s in strides)


def _fmt_const(v: float) -> str:
    if np.isnan(v):
        return "__int_as_float(0x7fc00000)"
    if np.isinf(v):
        return "__int_as_float(0x7f800000)" if v > 0 else "__int_as_float(0xff800000)"
    return repr(float(np.float32(v))) + "f"


class Region:
    """A kernel made of one or more independent segments."""

    def __init__(self, segs: List[Seg], label: str = "region"):
        self.segs = segs
        self.label = label
        self.params: List[str] = []      # buffer keys in kernel-parameter order
        self._fn = None
        self.grid = 0
        self._seg_blocks: List[Tuple[int, int]] = []
        self.source = ""
        self.name = ""

    # -- planning -----------------------------------------------------------
    def _plan(self, sm_count: int):
        keys: List[str] = []
        for s in self.segs:
            for i in s.inputs:
                for k in i.keys():
                    if k not in keys:
                        keys.append(k)
            for k, _ in s.outputs:
                if k not in keys:
                    keys.append(k)
        self.params = keys
        # blocks per segment: enough unrolled float4 work per thread, at most
        # BLOCKS_PER_SM blocks per SM overall
        work = []
        for s in self.segs:
            units = (s.total + 3) // 4 if self._vec_ok(s) else s.total
            work.append(max(1, (units + UNROLL * BLOCK - 1) // (UNROLL * BLOCK)))
        cap = BLOCKS_PER_SM * sm_count
        total = sum(work)
        if total > cap:
            scale = cap / total
            work = [max(1, int(w * scale)) for w in work]
        self._seg_blocks = []
        b0 = 0
        for w in work:
            self._seg_blocks.append((b0, b0 + w))
            b0 += w
        self.grid = b0

    @staticmethod
    def _vec_ok(s: Seg) -> bool:
        if not s.shape or s.shape[-1] % 4 != 0 or s.total % 4 != 0:
            return False
        for i in s.inputs:
            if i.access == "strided" and i.strides[-1] not in (0, 1):
                return False
            if i.access == "map" and not V.vec4_ok(i.mapspec, len(s.shape)):
                return False
        return True

    # -- code generation -----------------------------------------------------
    def _seg_code(self, si: int, s: Seg) -> str:
        b0, b1 = self._seg_blocks[si]
        vec = self._vec_ok(s)
        shape = s.shape if s.shape else (1,)
        C = int(shape[-1])
        cond = f"blockIdx.x < {b1}u" if b0 == 0 else f"blockIdx.x >= {b0}u && blockIdx.x < {b1}u"
        lines = [f"  if ({cond}) {{",
                 f"    const long long nb = {b1 - b0}LL * {BLOCK}LL;",
                 f"    const long long t0 = (long long)(blockIdx.x - {b0}u) * {BLOCK}LL + threadIdx.x;"]
        pidx = {k: i for i, k in enumerate(self.params)}
        lanes = 4 if vec else 1
        comp = ["x", "y", "z", "w"]

        # hoisted scalar inputs
        for ii, inp in enumerate(s.inputs):
            if inp.access == "scalar":
                lines.append(f"    const float s{ii} = p{pidx[inp.key]}[0];")

        def coord_code(e: str, x: str) -> List[str]:
            """row / column / strided offsets of flat element ``e`` (suffix x)"""
            out = []
            if any(i.access == "row" for i in s.inputs):
                out.append(f"      const long long r{x} = {e} / {C}LL;")
            if any(i.access == "col" for i in s.inputs):
                out.append(f"      const long long c{x} = {e} % {C}LL;")
            strided = [ii for ii, i in enumerate(s.inputs) if i.access == "strided"]
            mapped = [ii for ii, i in enumerate(s.inputs) if i.access == "map"]
            if strided or mapped:
                out.append(f"      long long rem{x} = {e};")
                for ax in reversed(range(len(shape))):
                    out.append(f"      const long long k{ax}{x} = rem{x} % {int(shape[ax])}LL; "
                               f"rem{x} /= {int(shape[ax])}LL;")
                for ii in strided:
                    terms = [f"k{ax}{x} * {st}LL" for ax, st in enumerate(s.inputs[ii].strides) if st]
                    out.append(f"      const long long o{ii}{x} = {' + '.join(terms) if terms else '0LL'};")
            return out

        def map_load(m: tuple, x: str, four: bool) -> str:
            """Expression loading one element (or float4) through index map ``m``."""
            if m[0] == "aff":
                terms = [f"{m[2]}LL"] + [f"k{ax}{x} * {st}LL" for ax, st in enumerate(m[3]) if st]
                p = f"p{pidx[m[1]]} + ({' + '.join(terms)})"
                return f"tl_ldc4({p})" if four else f"__ldg({p})"
            return (f"(k{m[1]}{x} < {m[2]}LL ? {map_load(m[3], x, four)} : "
                    f"{map_load(m[4], x, four)})")

        def is4(inp: Input) -> bool:
            return vec and (inp.access in ("full", "col", "map") or
                            (inp.access == "strided" and inp.strides[-1] == 1))

        def load_code(e: str, x: str) -> List[str]:
            out = []
            for ii, inp in enumerate(s.inputs):
                p = f"p{pidx[inp.key]}" if inp.key is not None else ""
                if inp.access == "full":
                    out.append(f"      const float4 v{ii}{x} = tl_ld4({p} + {e});" if vec
                               else f"      const float v{ii}{x} = __ldg({p} + {e});")
                elif inp.access == "row":
                    out.append(f"      const float v{ii}{x} = __ldg({p} + r{x});")
                elif inp.access == "col":
                    out.append(f"      const float4 v{ii}{x} = tl_ldc4({p} + c{x});" if vec
                               else f"      const float v{ii}{x} = __ldg({p} + c{x});")
                elif inp.access == "strided":
                    if is4(inp):
                        out.append(f"      const float4 v{ii}{x} = tl_ldc4({p} + o{ii}{x});")
                    else:
                        out.append(f"      const float v{ii}{x} = __ldg({p} + o{ii}{x});")
                elif inp.access == "map":
                    t = "float4" if is4(inp) else "float"
                    out.append(f"      const {t} v{ii}{x} = {map_load(inp.mapspec, x, is4(inp))};")
            return out

        def val(ref: Ref, lane: int, x: str) -> str:
            if ref.kind == "const":
                return _fmt_const(ref.value)
            if ref.kind == "tmp":
                return f"t{ref.idx}_{lane}{x}"
            inp = s.inputs[ref.idx]
            if inp.access == "scalar":
                return f"s{ref.idx}"
            return f"v{ref.idx}{x}.{comp[lane]}" if is4(inp) else f"v{ref.idx}{x}"

        def body_code(x: str) -> List[str]:
            out = []
            for lane in range(lanes):
                for ti, (opc, args) in enumerate(s.body):
                    tmpl = OPS[opc][1]
                    kw = {"a": val(args[0], lane, x)}
                    if len(args) > 1:
                        kw["b"] = val(args[1], lane, x)
                    out.append(f"      const float t{ti}_{lane}{x} = {tmpl.format(**kw)};")
            return out

        def store_code(e: str, x: str) -> List[str]:
            out = []
            for key, ref in s.outputs:
                p = f"p{pidx[key]}"
                if vec:
                    vals = ", ".join(val(ref, l, x) for l in range(4))
                    out.append(f"      tl_st4({p} + {e}, make_float4({vals}));")
                else:
                    out.append(f"      {p}[{e}] = {val(ref, 0, x)};")
            return out

        units = s.total // 4 if vec else s.total
        step = 4 if vec else 1
        # UNROLL-way unrolled grid-stride loop: each trip issues the loads of
        # all UNROLL units before any arithmetic; the remainder runs one unit
        # at a time
        lines.append("    long long u = t0;")
        lines.append(f"    for (; u + {UNROLL - 1}LL * nb < {units}LL; u += {UNROLL}LL * nb) {{")
        for q in range(UNROLL):
            lines.append(f"      const long long e_{q} = (u + {q}LL * nb) * {step}LL;")
        for q in range(UNROLL):
            lines += coord_code(f"e_{q}", f"_{q}")
        for q in range(UNROLL):
            lines += load_code(f"e_{q}", f"_{q}")
        for q in range(UNROLL):
            lines += body_code(f"_{q}")
            lines += store_code(f"e_{q}", f"_{q}")
        lines.append("    }")
        lines.append(f"    for (; u < {units}LL; u += nb) {{")
        lines.append(f"      const long long e_r = u * {step}LL;")
        lines += coord_code("e_r", "_r")
        lines += load_code("e_r", "_r")
        lines += body_code("_r")
        lines += store_code("e_r", "_r")
        lines.append("    }")
        lines.append("    return;")
        lines.append("  }")
        return "\n".join(lines)

    def codegen(self, sm_count: int) -> Tuple[str, str]:
        self._plan(sm_count)
        sig = "||".join(s.signature() for s in self.segs) + \
            f"|G{self.grid}|P{len(self.params)}|U{UNROLL}|B{BLOCK}"
        digest = hashlib.sha1(sig.encode()).hexdigest()[:20]
        name = f"tl_region_{digest}"
        written = set()
        for s in self.segs:
            for k, _ in s.outputs:
                written.add(k)
        params = []
        for i, k in enumerate(self.params):
            if k in written:
                params.append(f"float* __restrict__ p{i}")
            else:
                params.append(f"const float* __restrict__ p{i}")
        src = [PRELUDE,
               f'extern "C" __global__ void __launch_bounds__({BLOCK}) {name}({", ".join(params)}) {{']
        for si, s in enumerate(self.segs):
            src.append(self._seg_code(si, s))
        src.append("}")
        self.source = "\n".join(src)
        self.name = name
        return self.source, name

    # -- compile / launch ------------------------------------------------------
    def compile(self, dev: rt.Device):
        if self._fn is not None:
            return
        src, name = self.codegen(dev.sm_count)
        rt.JIT_DIR.mkdir(parents=True, exist_ok=True)
        fn = ctypes.c_void_p()
        rt.check(rt.lib().tl_jit_compile(src.encode(), name.encode(), name.encode(),
                                         str(rt.JIT_DIR).encode(), ctypes.byref(fn)),
                 f"jit {self.label}")
        self._fn = fn.value

    def bind(self, ptrs: Dict[str, int]):
        """Pre-build the argument array for the given buffer pointers."""
        n = len(self.params)
        vals = (ctypes.c_void_p * n)(*[ptrs[k] for k in self.params])
        argv = (ctypes.c_void_p * n)(*[ctypes.addressof(vals) + i * ctypes.sizeof(ctypes.c_void_p)
                                       for i in range(n)])
        return (vals, argv)

    def launch(self, bound, stream):
        _, argv = bound
        rt.check(rt.lib().tl_jit_launch(self._fn, self.grid, BLOCK, 0, argv, stream),
                 f"launch {self.label}")
