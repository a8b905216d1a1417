"""The allocation-free column reduction, checked against tl_reduce_cols.

``tl_reduce_cols_noalloc`` is for callers that cannot allocate device memory,
for example a plugin inside a host framework that owns every device
allocation, or a path with a fixed memory budget that must not allocate
while it runs.  It keeps its scratch in a 1 MiB array inside the library
instead of taking a scratch buffer.  This test calls it through the C ABI
twice in a row (the second call reuses the array the first one left behind)
and compares both results with the scratch-taking entry point: sums and means
within rel 1e-5 (chunking differs, so float64 partials round differently),
max/min/argmax/argmin exactly.  It also checks that a row too wide for the
array is rejected before anything runs.

The file name sorts last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest

from conftest import assert_close, load_backend

pytestmark = pytest.mark.gpu

OPS = {"sum": 0, "mean": 1, "max": 2, "min": 3, "argmax": 4, "argmin": 5}


@pytest.mark.parametrize("rows,cols", [(1000, 4096), (16384, 4096), (300, 257), (65536, 64),
                                       (3, 130560)])
@pytest.mark.parametrize("op", list(OPS))
def test_noalloc_matches_scratch_entry_point(rows, cols, op):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    code = OPS[op]
    if code >= 4 and cols > 65280:
        pytest.skip("argmax/argmin take at most 65280 columns")
    dev = rt.Device.get(0)
    rng = np.random.default_rng(rows + cols + code)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    if code >= 4:  # each column's extreme repeated in a later row: the first index must win
        x[rows // 2, :] = x.max(axis=0) if code == 4 else x.min(axis=0)
    dx = rt.DeviceBuffer(dev, (rows, cols))
    dx.upload(x)
    ref = rt.DeviceBuffer(dev, (cols,))
    scratch = rt.DeviceBuffer(dev, (L.tl_reduce_cols_scratch_bytes(code, rows, cols) // 4 + 1,), zero=True)
    rt.check(L.tl_reduce_cols(code, dx.ptr, ref.ptr, rows, cols, scratch.ptr, dev.stream))
    expect = ref.download()
    for call in range(2):
        out = rt.DeviceBuffer(dev, (cols,))
        out.zero()
        rt.check(L.tl_reduce_cols_noalloc(code, dx.ptr, out.ptr, rows, cols, dev.stream),
                 f"noalloc call {call}")
        got = out.download()
        if code in (0, 1):
            assert_close(got, expect, 1e-5, f"{op} call {call}")
        else:
            np.testing.assert_array_equal(got, expect, err_msg=f"{op} call {call}")
        out.free()
    for b in (dx, ref, scratch):
        b.free()


def test_noalloc_rejects_rows_wider_than_its_array():
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    buf = rt.DeviceBuffer(dev, (130564,))
    out = rt.DeviceBuffer(dev, (130564,))
    assert L.tl_reduce_cols_noalloc(0, buf.ptr, out.ptr, 1, 130561, dev.stream) == rt.TL_ERR_INVALID_ARG
    assert L.tl_reduce_cols_noalloc(4, buf.ptr, out.ptr, 1, 65281, dev.stream) == rt.TL_ERR_INVALID_ARG
    dev.sync()
    buf.free()
    out.free()
