"""Classifier-head fusion: a peephole pass over a lowered program.

A training step ends in ``z = linear(a, W, b); p = softmax(z, axis=1);
loss = cross_entropy(p, t)`` (kernel_generator.py:1584-1661, :564-640,
:1816-1885), and its backward starts with the cross_entropy VJP chained
through the softmax VJP (autograd.py:691-704, :563-580), then the linear
VJP's dW, db and dX (:619-646), the last with the relu-VJP mask of the layer
below (folded into it by ``epilogue.py``).  With a narrow head (N <= 16) the
forward product, softmax, the chained VJP and dX are four passes over the
[M, K] input or the [M, N] logits, plus their launches.  This pass replaces
them with one ``tl_head_ce`` call placed where the chained VJP ran (after
the loss seed is written), followed by the loss kernel, which reads ``p``;
dW and db keep their own kernels.  The fused kernel computes every value in
the order of the kernels it replaces, so the program's results are
bit-identical (``tests/test_gpu_epilogue.py``).

The rewrite requires: the forward product is a plain ``tl_gemm`` (no
transpose, no accumulate, no epilogue) whose output only the softmax reads
(or that is fetched: then the fused call also writes it); the softmax output
is read before the VJP only by the loss; the VJP writes its gradient
first-hand (no accumulate); the dX product is the masked nt product of that
gradient with the same weight, first-hand; nothing between the forward
product and the VJP writes the product's operands or the targets, and
nothing between the VJP and dX touches dX's operands or result; and the
shapes are ones ``tl_head_ce_ok`` accepts.
"""
from __future__ import annotations

from typing import Dict, List

from . import runtime as rt
from .epilogue import _counts, _flat
from .steps import LibCall

# tl_gemm / tl_gemm_masked argument slots
_TA, _TB, _M, _N, _K, _A, _LDA, _B, _LDB, _C, _LDC, _BIAS, _ACC, _EPI = range(14)
_MASK, _LDM = 14, 15


def _lib(s, name):
    return isinstance(s, LibCall) and s.fname == name


def _val(a):
    return a[1] if a[0] in ("int", "float", "ptr") else None


def fuse_classifier_head(P) -> int:
    """Apply the rewrite wherever it matches; returns how many were made."""
    if P.fetch is None:
        return 0
    pinned = set(P.fetch) | set(P.initial) | {sv["tensor"] for sv in P.saves}
    aliased = set(P.alias) | set(P.alias.values())
    total = 0
    while _rewrite_once(P, pinned, aliased):
        total += 1
    return total


def _rewrite_once(P, pinned, aliased) -> bool:
    flat = _flat(P)
    steps = [s for _, s in flat]
    reads, writes = _counts(flat)
    pos = {id(s): i for i, s in enumerate(steps)}
    for ice, ce in enumerate(steps):
        if not _lib(ce, "tl_ce_softmax_backward") or ce.args[9] != ("int", 0):
            continue
        p, tgt, onehot = ce.args[0][1], ce.args[1][1], ce.args[2][1]
        upstream = _val(ce.args[3])
        divisor = ce.args[4][1]
        dp = ce.args[5][1] if ce.args[5][0] == "ptr" else None
        gz = ce.args[6][1]
        rows, cols = ce.args[7][1], ce.args[8][1]
        # the softmax that wrote p, and the forward product that wrote its input
        sm = next((s for s in steps[:ice] if _lib(s, "tl_softmax_rows") and p in s.writes), None)
        if sm is None or writes.get(p, 0) != 1:
            continue
        z = sm.args[0][1]
        fz = next((s for s in steps[:pos[id(sm)]] if _lib(s, "tl_gemm") and z in s.writes), None)
        if fz is None or writes.get(z, 0) != 1 or z in aliased or p in aliased:
            continue
        a = fz.args
        if (_val(a[_TA]), _val(a[_TB]), _val(a[_ACC]), _val(a[_EPI])) != (0, 0, 0, 0):
            continue
        M, N, K = _val(a[_M]), _val(a[_N]), _val(a[_K])
        A, lda, W, ldw = a[_A][1], _val(a[_LDA]), a[_B][1], _val(a[_LDB])
        bias = a[_BIAS][1] if a[_BIAS][0] == "ptr" else None
        if (M, N) != (rows, cols) or _val(a[_LDC]) != N:
            continue
        # the masked dX product of the gradient with the same weight
        dx = next((s for s in steps[ice + 1:] if _lib(s, "tl_gemm_masked") and gz in s.reads
                   and s.args[_A] == ("ptr", gz)), None)
        if dx is None:
            continue
        d = dx.args
        if ((_val(d[_TA]), _val(d[_TB]), _val(d[_ACC]), _val(d[_EPI])) != (0, 1, 0, 0)
                or (_val(d[_M]), _val(d[_N]), _val(d[_K])) != (M, K, N)
                or d[_B] != ("ptr", W) or _val(d[_LDA]) != N or _val(d[_LDB]) != ldw):
            continue
        gx, lddx = d[_C][1], _val(d[_LDC])
        mask, ldm = d[_MASK][1], _val(d[_LDM])
        if gx in aliased or writes.get(gx, 0) != 1:
            continue
        # readers: z only by the softmax (or fetched); p before the VJP only by the loss
        iz, ism, idx = pos[id(fz)], pos[id(sm)], pos[id(dx)]
        z_readers = [s for s in steps if z in s.reads]
        if any(s is not sm for s in z_readers):
            continue
        loss = [s for s in steps[ism + 1:ice] if p in s.reads]
        if len(loss) > 1 or (loss and not _lib(loss[0], "tl_cross_entropy")):
            continue
        operands = {A, W, tgt} | ({bias} if bias else set())
        if any(operands & set(s.writes) for s in steps[iz + 1:ice]):
            continue
        if any({gz, W, mask, gx} & set(s.writes) or gx in s.reads for s in steps[ice + 1:idx]):
            continue
        if upstream is not None and any(upstream in s.writes for s in steps[ice + 1:idx]):
            continue
        if not _shape_ok(M, N, K, lda, lddx, ldm, ldw):
            continue
        keep_z = z in pinned
        fused = LibCall(
            f"head_ce:{z}+{p}+{gz}+{gx}", "tl_head_ce",
            [("ptr", A), ("int", lda), ("ptr", W), ("int", ldw),
             ("ptr", bias) if bias else ("null",), ("ptr", tgt), ("int", onehot),
             ("ptr", upstream) if upstream else ("null",), ("float", divisor),
             ("ptr", z) if keep_z else ("null",), ("ptr", p), ("ptr", dp) if dp else ("null",),
             ("ptr", gz), ("ptr", gx), ("int", lddx), ("ptr", mask), ("int", ldm),
             ("int", M), ("int", N), ("int", K)],
            reads=[A, W, tgt, mask] + ([bias] if bias else []) + ([upstream] if upstream else []),
            writes=([z] if keep_z else []) + [p] + ([dp] if dp else []) + [gz, gx])
        lst_of = {id(s): lst for lst, s in flat}
        lst_of[id(fz)].remove(fz)
        lst_of[id(sm)].remove(sm)
        for s in loss:
            lst_of[id(s)].remove(s)
        ce_list = lst_of[id(ce)]
        i = ce_list.index(ce)
        ce_list[i:i + 1] = [fused] + loss
        lst_of[id(dx)].remove(dx)
        return True
    return False


def _shape_ok(M, N, K, lda, lddx, ldm, ldw) -> bool:
    if ldm is None or ldm % 4 or ldw is None or ldw < N:
        return False
    # pool allocations are 256-byte aligned: stand in an aligned address
    return rt.lib().tl_head_ce_ok(M, N, K, 256, lda, 256, lddx) == 1
