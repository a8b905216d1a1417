"""tl_gemm_pair_prepare_colsum: the pair pre-pass that also writes the column
sums of its input (a linear layer's bias gradient, autograd.py:619-646).

The pair matrices must equal tl_gemm_pair_prepare's bit for bit (same
layouts, both lo orders); the sums must match float64 within rel 1e-6 of
max|sum| (they are summed in double and rounded once) and agree with
tl_reduce_cols(TL_RED_SUM) to within a float step.  Shapes cover one,
two and four column steps per thread (cols up to 8192), ragged rows and
columns, and each layout alone.
"""
import ctypes

import numpy as np
import pytest

from conftest import load_backend

pytestmark = pytest.mark.gpu

KMAJOR, MNMAJOR = 0, 1


def _bufs(rt, dev, L, rows, cols, layouts):
    out = {}
    for lay in layouts:
        nbytes = int(L.tl_gemm_pair_bytes(rows, cols, lay))
        out[lay] = (rt.DeviceBuffer(dev, ((nbytes + 3) // 4,)), rt.DeviceBuffer(dev, ((nbytes + 3) // 4,)))
    return out


@pytest.mark.parametrize("rows,cols,layouts,klo,mlo", [
    (65536, 4096, (KMAJOR, MNMAJOR), 0, 1),   # dY of the hidden layers at one GPU
    (8192, 4096, (KMAJOR, MNMAJOR), 0, 1),    # per rank at eight GPUs
    (8192, 4096, (MNMAJOR,), 0, 0),           # MN-major only (dh1's use)
    (3001, 1000, (KMAJOR, MNMAJOR), 1, 0),    # ragged rows and columns, one column step
    (5000, 8192, (KMAJOR,), 0, 0),            # four column steps
    (777, 33, (KMAJOR, MNMAJOR), 0, 1),       # narrow
])
def test_colsum_pairs_equal_plain_pairs_and_sums_match(rows, cols, layouts, klo, mlo):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    st = dev.stream
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) * rng.uniform(0.1, 10.0, cols)).astype(np.float32)
    X = rt.DeviceBuffer(dev, x.shape)
    X.upload(x)
    pairs = _bufs(rt, dev, L, rows, cols, layouts)
    plain = {lay: b[0] for lay, b in pairs.items()}
    fused = {lay: b[1] for lay, b in pairs.items()}
    ptr = lambda d, lay: d[lay].ptr if lay in d else None  # noqa: E731
    rt.check(L.tl_gemm_pair_prepare(X.ptr, cols, rows, cols, ptr(plain, KMAJOR), klo,
                                    ptr(plain, MNMAJOR), mlo, st))
    nscratch = int(L.tl_gemm_pair_colsum_scratch_bytes(rows, cols))
    assert nscratch > 0
    scratch = rt.DeviceBuffer(dev, ((nscratch + 3) // 4,))
    s1, s2, ref_sum = (rt.DeviceBuffer(dev, (cols,)) for _ in range(3))
    for out in (s1, s2):   # two calls in a row: the scratch's old contents do not leak in
        rt.check(L.tl_gemm_pair_prepare_colsum(X.ptr, cols, rows, cols, ptr(fused, KMAJOR), klo,
                                               ptr(fused, MNMAJOR), mlo, out.ptr, scratch.ptr,
                                               nscratch, st))
    red_bytes = int(L.tl_reduce_cols_scratch_bytes(rt.RED_SUM, rows, cols))
    red_scratch = rt.DeviceBuffer(dev, ((red_bytes + 3) // 4,), zero=True)
    rt.check(L.tl_reduce_cols(rt.RED_SUM, X.ptr, ref_sum.ptr, rows, cols, red_scratch.ptr, st))
    got = {lay: (plain[lay].download(), fused[lay].download()) for lay in layouts}
    a, b, r = s1.download(), s2.download(), ref_sum.download()
    for d in [X, scratch, s1, s2, ref_sum, red_scratch] + [v for p in pairs.values() for v in p]:
        d.free()
    for lay, (p_, f_) in got.items():
        np.testing.assert_array_equal(f_.view(np.uint32), p_.view(np.uint32),
                                      err_msg=f"pair layout {lay} differs")
    np.testing.assert_array_equal(a, b)
    exact = x.astype(np.float64).sum(axis=0)
    scale = np.abs(exact).max()
    assert np.abs(a - exact).max() <= 1e-6 * scale, "column sums vs float64"
    # double sums of the same values in another order, each rounded once: at
    # most a float step apart (two where a sum sits on a binade boundary)
    ulp = np.spacing(np.abs(r).astype(np.float32))
    assert np.all(np.abs(a - r) <= 2 * ulp), "column sums vs tl_reduce_cols"


def test_colsum_limits():
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    rows, cols = 256, 8200   # more than 8192 columns: refused
    X = rt.DeviceBuffer(dev, (rows, cols))
    k = rt.DeviceBuffer(dev, ((int(L.tl_gemm_pair_bytes(rows, cols, KMAJOR)) + 3) // 4,))
    s = rt.DeviceBuffer(dev, (cols,))
    n = int(L.tl_gemm_pair_colsum_scratch_bytes(rows, cols))
    scratch = rt.DeviceBuffer(dev, ((n + 3) // 4,))
    assert L.tl_gemm_pair_prepare_colsum(X.ptr, cols, rows, cols, k.ptr, 0, None, 0, s.ptr,
                                         scratch.ptr, n, dev.stream) == rt.TL_ERR_UNSUPPORTED
    # a scratch smaller than asked for: refused before any launch
    assert L.tl_gemm_pair_prepare_colsum(X.ptr, cols, rows, 4096, k.ptr, 0, None, 0, s.ptr,
                                         scratch.ptr, 64, dev.stream) == rt.TL_ERR_INVALID_ARG
    for d in (X, k, s, scratch):
        d.free()
    err = ctypes.c_int(0)
    rt.check(L.tl_device_error(ctypes.byref(err), 1))
    assert err.value == 0
