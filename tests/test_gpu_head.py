"""tl_head_ce (the fused classifier head) against the unfused calls it
replaces, bit for bit, and against float64.

Unfused: ``tl_gemm`` (z = A W + b), ``tl_softmax_rows``,
``tl_ce_softmax_backward`` (the cross_entropy VJP chained through the
softmax VJP) and ``tl_gemm_masked`` (dx = dz W^T masked by A > 0).  The fused
call must return the same z, p, dp, dz and dx to the last bit, for one-hot
and class-index targets, with and without a bias, for 3 to 16 classes, with
the row count a multiple of the kernel's row groups or not, and with the
two row-group sizes (2 and 4 rows a warp).  Against float64 (a sanity
check): rel 1e-5 for z, p and the gradients, atol rel * max|ref|.
"""
import numpy as np
import pytest

from conftest import assert_close, load_backend

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,onehot,bias", [
    (8192, 10, 4096, 1, True),     # the per-rank head at 8 GPUs (2 rows a warp)
    (65536, 10, 4096, 1, True),    # one GPU (4 rows a warp)
    (3001, 3, 1024, 0, False),     # 4 padded classes, class-index targets, ragged rows
    (1000, 16, 512, 1, True),      # 16 classes
    (5000, 7, 260, 0, True),       # 8 padded classes, K not a multiple of 32
])
def test_fused_head_equals_the_unfused_calls(M, N, K, onehot, bias):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    st = dev.stream
    rng = np.random.default_rng(M + N + K)
    A = np.maximum(rng.standard_normal((M, K)), 0).astype(np.float32)  # a relu output
    W = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    cls = rng.integers(0, N, M)
    T = np.eye(N, dtype=np.float32)[cls] if onehot else cls.astype(np.float32)
    divisor = float(M)
    buf = lambda a: (lambda d: (d.upload(a), d)[1])(rt.DeviceBuffer(dev, a.shape))  # noqa: E731
    dA, dW, db, dT = buf(A), buf(W), buf(b), buf(T)
    up = buf(np.ones(1, np.float32))
    out1 = {k: rt.DeviceBuffer(dev, s) for k, s in
            [("z", (M, N)), ("p", (M, N)), ("dp", (M, N)), ("dz", (M, N)), ("dx", (M, K))]}
    out2 = {k: rt.DeviceBuffer(dev, v.shape) for k, v in out1.items()}
    bp = db.ptr if bias else None
    assert L.tl_head_ce_ok(M, N, K, dA.ptr, K, out2["dx"].ptr, K) == 1
    rt.check(L.tl_gemm(0, 0, M, N, K, dA.ptr, K, dW.ptr, N, out1["z"].ptr, N, bp, 0, 0, st))
    rt.check(L.tl_softmax_rows(out1["z"].ptr, out1["p"].ptr, M, N, st))
    rt.check(L.tl_ce_softmax_backward(out1["p"].ptr, dT.ptr, onehot, up.ptr, divisor,
                                      out1["dp"].ptr, out1["dz"].ptr, M, N, 0, st))
    rt.check(L.tl_gemm_masked(0, 1, M, K, N, out1["dz"].ptr, N, dW.ptr, N, out1["dx"].ptr, K,
                              None, 0, 0, dA.ptr, K, st))
    rt.check(L.tl_head_ce(dA.ptr, K, dW.ptr, N, bp, dT.ptr, onehot, up.ptr, divisor,
                          out2["z"].ptr, out2["p"].ptr, out2["dp"].ptr, out2["dz"].ptr,
                          out2["dx"].ptr, K, dA.ptr, K, M, N, K, st))
    got = {k: (out1[k].download(), out2[k].download()) for k in out1}
    for d in [dA, dW, db, dT, up] + list(out1.values()) + list(out2.values()):
        d.free()
    for k, (u, f) in got.items():
        np.testing.assert_array_equal(f, u, err_msg=f"fused {k} differs from the unfused calls")
    # float64 sanity
    z = A.astype(np.float64) @ W.astype(np.float64) + (b if bias else 0)
    e = np.exp(z - z.max(axis=1, keepdims=True))
    p = e / e.sum(axis=1, keepdims=True)
    t = np.eye(N)[cls]
    g = (p - t) / divisor
    dz = p * (g - (g * p).sum(axis=1, keepdims=True))
    dx = (dz @ W.astype(np.float64).T) * (A > 0)
    for k, ref in [("z", z), ("p", p), ("dp", g), ("dz", dz), ("dx", dx)]:
        assert_close(got[k][1], ref, 1e-5 if k != "dx" else 1e-4, f"fused {k} vs float64")


def test_unsupported_shapes_are_refused():
    tl = load_backend()
    L = tl.runtime.lib()
    assert L.tl_head_ce_ok(8192, 10, 4094, 256, 4094, 256, 4094) == 0   # K not a multiple of 4
    assert L.tl_head_ce_ok(8192, 17, 4096, 256, 4096, 256, 4096) == 0   # more than 16 classes
    assert L.tl_head_ce_ok(64, 10, 256, 256, 256, 256, 256) == 0        # M * K < 65536
    assert L.tl_head_ce_ok(8192, 10, 4096, 260, 4096, 256, 4096) == 0   # A not 16-byte aligned
