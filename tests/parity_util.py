"""Checks of large GPU products against float64 without a float64 product of
the whole matrix.

A full float64 product at the benchmark sizes (65536 x 4096 x 4096) costs
minutes of CPU; these checks cost a fraction of a second and still see every
output tile of the tensor-core kernels:

* ``check_sampled`` compares, element by element, one row out of every
  ``row_block`` rows and one column out of every ``col_block`` columns with
  a float64 evaluation of the same rows and columns.  With the GEMM's
  128-row by 256-column CTA-pair tiles (``row_block=128``,
  ``col_block=256``), every tile, every K split and every cluster's tile
  sequence contributes a whole row and a whole column to the comparison.
* ``check_projection`` is Freivalds' identity ``C v = A (B v)`` over all
  elements for a few random vectors ``v``: with the elementwise tolerance
  ``|C - ref| <= rtol |ref| + atol``, the projected residual obeys
  ``|(C - ref) v| <= (rtol |ref| + atol) |v|``, checked with ``|ref|`` taken
  as ``|C|`` plus the residual bound itself.

Both report the largest error found, relative to the largest |reference|
value, for the test log.
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np

from conftest import assert_close


def tile_sample(n: int, block: int, rng) -> np.ndarray:
    """One random index inside every block of ``block`` consecutive indices,
    plus the last index."""
    starts = np.arange(0, n, block)
    ends = np.minimum(starts + block, n)
    idx = starts + (rng.random(len(starts)) * (ends - starts)).astype(np.int64)
    return np.unique(np.concatenate([idx, [n - 1]]))


def f64_rows(A: np.ndarray, rows: np.ndarray) -> np.ndarray:
    return np.asarray(A[rows], dtype=np.float64)


def matmul_cols(A: np.ndarray, Bc: np.ndarray, chunk: int = 8192) -> np.ndarray:
    """float64 ``A @ Bc`` for a tall float32 ``A`` and a narrow ``Bc``,
    converting ``A`` a block of rows at a time."""
    out = np.empty((A.shape[0], Bc.shape[1]), np.float64)
    for r in range(0, A.shape[0], chunk):
        out[r:r + chunk] = np.asarray(A[r:r + chunk], np.float64) @ Bc
    return out


def check_sampled(got: np.ndarray, ref_rows: Callable[[np.ndarray], np.ndarray],
                  ref_cols: Callable[[np.ndarray], np.ndarray], rtol: float, name: str,
                  row_block: int = 128, col_block: int = 256, seed: int = 0) -> float:
    """Compare sampled rows and columns of ``got`` with their float64 values.

    ``ref_rows(idx)`` returns the reference rows ``idx`` (shape
    ``[len(idx), N]``), ``ref_cols(idx)`` the reference columns (``[M,
    len(idx)]``).  atol is rtol times the largest |reference| value seen."""
    rng = np.random.default_rng(seed)
    M, N = got.shape
    rows = tile_sample(M, row_block, rng)
    cols = tile_sample(N, col_block, rng)
    rr = ref_rows(rows)
    rc = ref_cols(cols)
    scale = max(float(np.abs(rr).max()), float(np.abs(rc).max()), 1e-300)
    atol = rtol * scale
    assert_close(got[rows], rr, rtol, f"{name} rows", atol=atol)
    assert_close(got[:, cols], rc, rtol, f"{name} cols", atol=atol)
    err = max(float(np.abs(got[rows] - rr).max()), float(np.abs(got[:, cols] - rc).max()))
    return err / scale


def check_projection(got: np.ndarray, ref_apply: Callable[[np.ndarray], np.ndarray],
                     rtol: float, name: str, nvec: int = 3, seed: int = 1,
                     atol: Optional[float] = None) -> float:
    """Freivalds: ``got @ v`` against ``ref_apply(v)`` (the reference product
    applied to ``v`` without forming it) for ``nvec`` Gaussian vectors."""
    rng = np.random.default_rng(seed)
    N = got.shape[1]
    V = rng.standard_normal((N, nvec))
    gv = matmul_cols(got, V)
    rv = ref_apply(V)
    absC = np.abs(got)
    if atol is None:
        atol = rtol * float(absC.max())
    bound = matmul_cols(absC, np.abs(V)) * rtol + atol * np.abs(V).sum(axis=0)[None, :]
    res = np.abs(gv - rv)
    bad = res > bound * (1 + 2 * rtol)
    if bad.any():
        i = np.unravel_index(int(np.argmax(res - bound)), res.shape)
        raise AssertionError(f"{name}: projection residual {res[i]:.3e} > bound {bound[i]:.3e} "
                             f"at {i} ({int(bad.sum())} of {res.size})")
    return float((res / np.maximum(bound, 1e-300)).max()) * rtol
