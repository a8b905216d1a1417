"""The allocation-free column reduction, checked against tl_reduce_cols and
against NumPy in float64.

``tl_reduce_cols_noalloc`` is for callers that cannot allocate device memory,
for example a plugin inside a host framework that owns every device
allocation, or a path with a fixed memory budget that must not allocate
while it runs.  It keeps its scratch in a 1 MiB array inside the library
instead of taking a scratch buffer.  This test calls it through the C ABI
twice in a row (the second call reuses the array the first one left behind)
and compares both results

* with the scratch-taking entry point: sums and means within rel 1e-5
  (chunking differs, so float64 partials round differently),
  max/min/argmax/argmin exactly;
* with NumPy on the same float32 input: sums and means against the float64
  column sums within rel 1e-5, max/min exactly, argmax/argmin exactly with
  the first index winning ties.

Shapes cover the float4 path, the one-column-per-lane path at widths above
32768 columns (cols % 4 != 0, and an input that starts 4 bytes past a
16-byte boundary), and the widest rows the array takes.  Rows one column
too wide are rejected before anything runs.

The file name sorts last so that a run stopping at its first failure has
already run every other test.
"""
import numpy as np
import pytest

from conftest import assert_close, load_backend

pytestmark = pytest.mark.gpu

OPS = {"sum": 0, "mean": 1, "max": 2, "min": 3, "argmax": 4, "argmin": 5}
MAX_COLS = 129024      # (1 MiB - 16 KiB) / 8 bytes of partials per column
MAX_COLS_ARG = 64512   # / 16 bytes


def _numpy(op, x):
    x64 = x.astype(np.float64)
    return {"sum": lambda: x64.sum(axis=0), "mean": lambda: x64.mean(axis=0),
            "max": lambda: x.max(axis=0), "min": lambda: x.min(axis=0),
            "argmax": lambda: np.argmax(x, axis=0).astype(np.float32),
            "argmin": lambda: np.argmin(x, axis=0).astype(np.float32)}[op]()


@pytest.mark.parametrize("rows,cols,offset", [
    (1000, 4096, 0), (16384, 4096, 0), (300, 257, 0), (65536, 64, 0),
    (5, 40001, 0),            # one column per lane, 1251 column stripes
    (7, 40000, 1),            # cols % 4 == 0 but the input is not 16-byte aligned
    (3, MAX_COLS, 0), (4, MAX_COLS_ARG, 0)])
@pytest.mark.parametrize("op", list(OPS))
def test_noalloc_matches_scratch_entry_point_and_numpy(rows, cols, offset, op):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    code = OPS[op]
    if code >= 4 and cols > MAX_COLS_ARG:
        pytest.skip(f"argmax/argmin take at most {MAX_COLS_ARG} columns")
    dev = rt.Device.get(0)
    rng = np.random.default_rng(rows + cols + code)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    if code >= 4:  # each column's extreme repeated in a later row: the first index must win
        x[rows // 2, :] = x.max(axis=0) if code == 4 else x.min(axis=0)
    # ``offset`` floats of padding in front: the input pointer is the
    # allocation's base plus 4 * offset bytes
    buf = rt.DeviceBuffer(dev, (rows * cols + offset,))
    buf.upload(np.concatenate([np.zeros(offset, np.float32), x.reshape(-1)]))
    ptr = buf.ptr + 4 * offset
    ref = rt.DeviceBuffer(dev, (cols,))
    scratch = rt.DeviceBuffer(dev, (L.tl_reduce_cols_scratch_bytes(code, rows, cols) // 4 + 1,), zero=True)
    rt.check(L.tl_reduce_cols(code, ptr, ref.ptr, rows, cols, scratch.ptr, dev.stream))
    expect = ref.download()
    want = _numpy(op, x)
    for call in range(2):
        out = rt.DeviceBuffer(dev, (cols,))
        out.zero()
        rt.check(L.tl_reduce_cols_noalloc(code, ptr, out.ptr, rows, cols, dev.stream),
                 f"noalloc call {call}")
        got = out.download()
        out.free()
        if code in (0, 1):
            assert_close(got, expect, 1e-5, f"{op} call {call} vs tl_reduce_cols")
            assert_close(got, want, 1e-5, f"{op} call {call} vs numpy float64")
        else:
            np.testing.assert_array_equal(got, expect, err_msg=f"{op} call {call} vs tl_reduce_cols")
            np.testing.assert_array_equal(got, want, err_msg=f"{op} call {call} vs numpy")
    for b in (buf, ref, scratch):
        b.free()


def test_noalloc_rejects_rows_wider_than_its_array():
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    buf = rt.DeviceBuffer(dev, (MAX_COLS + 4,))
    out = rt.DeviceBuffer(dev, (MAX_COLS + 4,))
    assert L.tl_reduce_cols_noalloc(0, buf.ptr, out.ptr, 1, MAX_COLS + 1, dev.stream) == rt.TL_ERR_INVALID_ARG
    assert L.tl_reduce_cols_noalloc(4, buf.ptr, out.ptr, 1, MAX_COLS_ARG + 1, dev.stream) == rt.TL_ERR_INVALID_ARG
    dev.sync()
    buf.free()
    out.free()
