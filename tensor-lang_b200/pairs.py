"""GEMM operand pairs, prepared once per operand value.

The pair GEMM schemes (BF16X3, the default, and TF32+bf16) need a bf16 pair
matrix of each fp32 operand (values and lows, see include/tlb200.h); ``tl_gemm`` builds
those with a pre-pass on every call.  In a training iteration one activation
feeds several products in different roles -- a1 is the K-major A operand of
the next layer's forward GEMM and the MN-major A operand of that layer's dW;
h2's gradient is the K-major A operand of dX and the MN-major B operand of
dW -- and the batch input never changes.  This pass, run on each loop body
after epilogue fusion, gives every such operand value one pair step right
after the step that writes it (both layouts from one read,
``tl_gemm_pair_prepare``) or, for a value the body never writes, one step
hoisted out of the per-iteration graph; the GEMMs then take the prepared
pairs (``tl_gemm_pairs``).  The pairs are computed exactly as the per-call
pre-passes would compute them, so results are unchanged.

Only products that take a pair-scheme tensor-core path with contiguous
operands are planned (``tl_gemm_uses_pairs``); operands sharing a buffer
through in-place rebinding (updated weights) keep the per-call pre-pass.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

from . import runtime as rt
from .steps import LibCall

_GEMMS = ("tl_gemm", "tl_gemm_masked")
KMAJOR, MNMAJOR = 0, 1


def plan_gemm_pairs(P) -> int:
    """Plan pairs in every loop of program ``P``; returns the pair steps added."""
    from .engine import _Loop

    try:
        L = rt.lib()
    except Exception:  # no library: nothing to query, nothing planned
        return 0
    return sum(_plan_loop(P, L, s) for s in P.phase_pre if isinstance(s, _Loop))


def _plan_loop(P, L, loop) -> int:
    flat: List[Tuple[list, object]] = [(lst, s) for lst in (loop.pre, loop.bw, loop.post, loop.rebind)
                                       for s in lst]
    writers: Dict[str, List[int]] = {}
    for k, (_, s) in enumerate(flat):
        for w in s.writes:
            writers.setdefault(w, []).append(k)
    shared = set(P.alias) | set(P.alias.values())
    # (tensor, source) -> {(layout, lo_first): [(consumer, operand slot)]}
    wanted: Dict[Tuple[str, object], Dict[Tuple[int, int], list]] = {}
    for k, (_, g) in enumerate(flat):
        if not (isinstance(g, LibCall) and g.fname in _GEMMS):
            continue
        ta, tb, M, N, K = (int(g.args[i][1]) for i in range(5))
        A, lda, B, ldb = g.args[5][1], int(g.args[6][1]), g.args[7][1], int(g.args[8][1])
        sa, sb = tuple(P.shapes.get(A, ())), tuple(P.shapes.get(B, ()))
        if sa != ((K, M) if ta else (M, K)) or lda != sa[1]:
            continue
        if sb != ((N, K) if tb else (K, N)) or ldb != sb[1]:
            continue
        if not L.tl_gemm_uses_pairs(ta, tb, M, N, K, lda, ldb):
            continue
        for X, layout, lo, slot in ((A, MNMAJOR if ta else KMAJOR, 0, "a"),
                                    (B, KMAJOR if tb else MNMAJOR, 1, "b")):
            if X in shared:
                continue
            ws = writers.get(X, [])
            before = [w for w in ws if w < k]
            if before:
                src = before[-1]
            elif not ws:
                src = "hoist"  # the body never writes X
            else:
                continue  # a value carried over from the previous iteration
            wanted.setdefault((X, src), {}).setdefault((layout, lo), []).append((g, slot))

    added = 0
    pair_of: Dict[Tuple[int, str], str] = {}  # (id(consumer), slot) -> pair tensor
    for (X, src), combos in wanted.items():
        rows, cols = (int(d) for d in P.shapes[X])
        todo = sorted(combos)
        while todo:
            # one step: at most one K-major and one MN-major pair, from one read of X
            km = next(((lay, lo) for lay, lo in todo if lay == KMAJOR), None)
            mn = next(((lay, lo) for lay, lo in todo if lay == MNMAJOR), None)
            names = {}
            for combo in (km, mn):
                if combo is None:
                    continue
                todo.remove(combo)
                tag = "k" if combo[0] == KMAJOR else "m"
                name = f"__pair_{X}_{src}_{tag}{combo[1]}"
                nbytes = int(L.tl_gemm_pair_bytes(rows, cols, combo[0]))
                P.shapes[name] = ((nbytes + 3) // 4,)
                names[combo] = name
                for g, slot in combos[combo]:
                    pair_of[(id(g), slot)] = name
            args = [("ptr", X), ("int", cols), ("int", rows), ("int", cols),
                    ("ptr", names[km]) if km else ("null",), ("int", km[1] if km else 0),
                    ("ptr", names[mn]) if mn else ("null",), ("int", mn[1] if mn else 0)]
            step = LibCall(f"pairs:{X}", "tl_gemm_pair_prepare", args, [X], list(names.values()))
            if src == "hoist":
                loop.hoisted.append(step)
            else:
                lst, w = flat[src]
                lst.insert(lst.index(w) + 1 + added_after(lst, w), step)
            added += 1
    for _, g in flat:
        if not (isinstance(g, LibCall) and g.fname in _GEMMS):
            continue
        pa, pb = pair_of.get((id(g), "a")), pair_of.get((id(g), "b"))
        if pa is None and pb is None:
            continue
        a = list(g.args)
        mask = a[14:16] if g.fname == "tl_gemm_masked" else [("null",), ("int", 0)]
        g.args = (a[:7] + [("ptr", pa) if pa else ("null",)] + a[7:9] +
                  [("ptr", pb) if pb else ("null",)] + a[9:14] + mask)
        g.fname = "tl_gemm_pairs"
        g.reads = list(g.reads) + [n for n in (pa, pb) if n]
        g.label += "+pairs"
    return added


def added_after(lst: list, w) -> int:
    """Pair steps already inserted right after step ``w`` (keeps them in order)."""
    i, n = lst.index(w) + 1, 0
    while i + n < len(lst) and isinstance(lst[i + n], LibCall) and \
            lst[i + n].fname == "tl_gemm_pair_prepare":
        n += 1
    return n


PARTIALS = "__colsum_partials"


def fuse_bias_colsums(P) -> int:
    """Fold a bias gradient into the pair step of the same gradient.

    A linear layer's backward sums dY over rows for db (``tl_reduce_cols``,
    autograd.py:619-646) and converts the same dY into pairs for its dW and
    dX products.  Where the pair step of X is followed, in the same step
    list, by the row sum of X -- with nothing in between writing X or
    touching the sum's output -- the pair step also writes the sum
    (``tl_gemm_pair_prepare_colsum``: one read of X instead of two) and the
    sum's own step is dropped.  Its per-block partial sums go to a buffer of
    their own (``__colsum_partials``, shared by these steps, which run one
    after another on the program's stream), not to the program's scratch,
    whose counters the reduction and loss kernels keep at zero between
    calls.  Returns the number of sums folded."""
    from .engine import _Loop

    total = 0
    for loop in (s for s in P.phase_pre if isinstance(s, _Loop)):
        for lst in (loop.pre, loop.bw, loop.post, loop.rebind):
            total += _fold_list(P, lst)
    return total


def _fold_list(P, lst: list) -> int:
    folded = 0
    i = 0
    while i < len(lst):
        st = lst[i]
        if not (isinstance(st, LibCall) and st.fname == "tl_gemm_pair_prepare"):
            i += 1
            continue
        X, ld, rows, cols = st.args[0][1], st.args[1][1], st.args[2][1], st.args[3][1]
        j = next((k for k in range(i + 1, len(lst))
                  if isinstance(lst[k], LibCall) and lst[k].fname == "tl_reduce_cols"
                  and lst[k].args[1] == ("ptr", X)), None)
        if j is None or ld != cols or cols > 8192:
            i += 1
            continue
        red = lst[j]
        a = red.args
        if (a[0] != ("int", rt.RED_SUM) or a[2][0] != "ptr" or a[3] != ("int", rows)
                or a[4] != ("int", cols)):
            i += 1
            continue
        out = a[2][1]
        between = lst[i + 1:j]
        if any(X in b.writes or out in b.writes or out in b.reads for b in between):
            i += 1
            continue
        if out in P.alias or out in P.alias.values():
            i += 1
            continue
        floats = (int(rt.lib().tl_gemm_pair_colsum_scratch_bytes(rows, cols)) + 3) // 4
        have = P.shapes.get(PARTIALS, (0,))[0]
        P.shapes[PARTIALS] = (max(have, floats),)
        lst[i] = LibCall(st.label + "+colsum:" + out, "tl_gemm_pair_prepare_colsum",
                         list(st.args) + [("ptr", out), ("ptr", PARTIALS), ("bytes", PARTIALS)],
                         list(st.reads), list(st.writes) + [out, PARTIALS])
        del lst[j]
        folded += 1
        i += 1
    return folded
