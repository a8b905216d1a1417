"""GEMM epilogue fusion: a peephole pass over a lowered program.

The reference runs every op as its own kernel: linear (kernel_generator.py
:1584-1661), then relu (:1462-1478); in backward the relu VJP multiplies the
incoming gradient by (x > 0) (autograd.py:540-544) after the GEMM of the next
layer's VJP produced that gradient (autograd.py:619-646), and the result is
copied into the gradient buffer (autograd.py:317-333).  Each of those passes
reads and writes a full activation.  This pass moves them into the epilogue
of the GEMM that produces their input:

  A  ``h = gemm(...); a = relu(h)``      ->  ``a = gemm(..., relu)``; every
     ``relu_mask(g, h)`` becomes ``relu_mask(g, a)`` (a > 0 exactly where
     h > 0, NaN included, since relu is fmaxf(0, h)).
  B  ``y = gemm(...); t = relu_mask(y, m)``  ->  ``t = tl_gemm_masked(..., m)``
     (the epilogue rounds y * (m > 0 ? 1 : 0) like the region kernel).
  C  ``y = gemm(...); d = copy(y)``      ->  ``d = gemm(...)``.

Each rewrite requires that the intermediate (h, y) is written once, read only
by the ops being folded, not fetched, saved, given an initial value or
sharing a buffer (in-place rebinding), and that no step between the two
touches the tensors involved.  Results are bit-identical to the unfused
program.  With ``fetch=None`` (every tensor visible) nothing is rewritten.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

from .shapes import numel
from .steps import EW, LibCall

_GEMMS = ("tl_gemm", "tl_gemm_masked")
# tl_gemm argument slots (steps.kinfo_to_step / autograd._vjp_gemm layout)
_C, _LDC, _BIAS, _ACC, _EPI = 9, 10, 11, 12, 13


def _flat(P) -> List[Tuple[list, object]]:
    """(owning list, step) for every step, in execution order."""
    from .engine import _Loop

    out: List[Tuple[list, object]] = []

    def walk(lst):
        for s in lst:
            if isinstance(s, _Loop):
                for sub in (s.pre, s.bw, s.post, s.rebind):
                    walk(sub)
            else:
                out.append((lst, s))
    walk(P.phase_pre)
    walk(P.phase_bw)
    walk(P.phase_post)
    return out


def _counts(flat):
    reads: Dict[str, int] = {}
    writes: Dict[str, int] = {}
    for _, s in flat:
        for r in s.reads:
            reads[r] = reads.get(r, 0) + 1
        for w in s.writes:
            writes[w] = writes.get(w, 0) + 1
    return reads, writes


def _is_gemm(s) -> bool:
    return isinstance(s, LibCall) and s.fname in _GEMMS


def _full(o, name: Optional[str] = None) -> bool:
    return o[0] == "name" and o[2] in ("full", None) and (name is None or o[1] == name)


def _between(flat, i: int, j: int):
    return [s for _, s in flat[i + 1:j]]


def fuse_gemm_epilogues(P) -> int:
    """Apply rewrites A, B, C until none applies; returns how many were made."""
    if P.fetch is None:
        return 0
    pinned = set(P.fetch) | set(P.initial) | {sv["tensor"] for sv in P.saves}
    aliased = set(P.alias) | set(P.alias.values())
    blocked = pinned | aliased
    total = 0
    while True:
        flat = _flat(P)
        reads, writes = _counts(flat)
        done = _rewrite_once(P, flat, reads, writes, blocked, aliased)
        if not done:
            return total
        total += 1


def _rewrite_once(P, flat, reads, writes, blocked, aliased) -> bool:
    shapes = P.shapes
    for k, (lst, g) in enumerate(flat):
        if not _is_gemm(g) or g.args[_ACC] != ("int", 0):
            continue
        y = g.args[_C][1]
        if y in blocked or writes.get(y, 0) != 1:
            continue
        readers = [(kk, s) for kk, (_, s) in enumerate(flat) if y in s.reads]
        if not readers:
            continue
        k1, first = readers[0]
        if k1 < k:
            continue  # read before it is produced (a value carried across iterations)
        same_list = flat[k1][0] is lst

        # A: relu of the product
        if (g.fname == "tl_gemm" and g.args[_EPI] == ("int", 0) and same_list
                and isinstance(first, EW) and first.opcode == "relu"
                and len(first.operands) == 1 and _full(first.operands[0], y)
                and numel(shapes[first.out]) == numel(shapes[y])):
            a = first.out
            others = [s for _, s in readers[1:]]
            ok = (a not in aliased and writes.get(a, 0) == 1
                  and all(isinstance(s, EW) and s.opcode == "relu_mask"
                          and _full(s.operands[1], y) and s.operands[0][1] != y
                          for s in others)
                  and not any(a in s.reads or a in s.writes for s in _between(flat, k, k1)))
            if ok:
                g.args[_C] = ("ptr", a)
                g.args[_EPI] = ("int", 1)  # TL_EPI_RELU
                g.writes = [a]
                g.label += "+relu"
                lst.remove(first)
                for s in others:
                    s.operands[1] = ("name", a, "full")
                    s.reads = [o[1] for o in s.operands if o[0] == "name"]
                return True

        if len(readers) != 1 or not same_list or not isinstance(first, EW):
            continue
        between = _between(flat, k, k1)

        # B: relu mask of the product
        if (first.opcode == "relu_mask" and _full(first.operands[0], y)
                and _full(first.operands[1]) and first.operands[1][1] != y
                and g.fname == "tl_gemm"):
            m, t = first.operands[1][1], first.out
            ok = (t not in aliased and writes.get(t, 0) == 1
                  and tuple(shapes[m]) == tuple(shapes[y]) == tuple(shapes[t])
                  and len(shapes[m]) == 2
                  and not any(m in s.writes or t in s.reads or t in s.writes for s in between))
            if ok:
                g.fname = "tl_gemm_masked"
                g.args[_C] = ("ptr", t)
                g.args = list(g.args) + [("ptr", m), ("int", int(shapes[m][1]))]
                g.reads = list(g.reads) + [m]
                g.writes = [t]
                g.label += "+mask"
                lst.remove(first)
                return True

        # C: copy of the product
        if (first.opcode == "copy" and len(first.operands) == 1 and _full(first.operands[0], y)
                and tuple(shapes[first.out]) == tuple(shapes[y])):
            d = first.out
            ok = d not in aliased and not any(d in s.reads or d in s.writes for s in between)
            if ok:
                g.args[_C] = ("ptr", d)
                g.writes = [d]
                g.label += f"->{d}"
                lst.remove(first)
                return True
    return False
