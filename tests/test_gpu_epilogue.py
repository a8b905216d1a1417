"""GEMM epilogues on the GPU: the relu-mask epilogue (tl_gemm_masked) on every
GEMM path against a float64 product, and a training program whose relu and
relu-VJP passes were folded into GEMM epilogues and whose GEMM operand pairs
are prepared once per value (pairs.py) against the same program run unfused
-- bit-identical, since the folded ops round exactly as the region kernels do
and the prepared pairs equal the per-call ones.  Tolerance for the products: rel 1e-5 of max|C|."""
import ctypes

import numpy as np
import pytest

from conftest import assert_close, load_backend

pytestmark = pytest.mark.gpu


def _masked(ta, tb, M, N, K, bias=False, acc=False, relu=False, seed=0):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    rng = np.random.default_rng(seed + M + 3 * N + 7 * K)
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    bv = rng.standard_normal(N).astype(np.float32)
    mask = rng.standard_normal((M, N)).astype(np.float32)
    mask[rng.random((M, N)) < 0.1] = 0.0          # exact zeros are masked out
    mask[0, : min(N, 4)] = [np.nan, -0.0, np.inf, -np.inf][: min(N, 4)]
    bufs = [rt.DeviceBuffer(dev, a.shape) for a in (A, B, C0, bv, mask)]
    for b, a in zip(bufs, (A, B, C0, bv, mask)):
        b.upload(a)
    dA, dB, dC, db, dm = bufs
    rt.check(L.tl_gemm_masked(ta, tb, M, N, K, dA.ptr, A.shape[1], dB.ptr, B.shape[1], dC.ptr, N,
                              db.ptr if bias else None, 1 if acc else 0, 1 if relu else 0,
                              dm.ptr, N, dev.stream))
    out = dC.download()
    err = ctypes.c_int(0)
    rt.check(L.tl_device_error(ctypes.byref(err), 1))
    for b in bufs:
        b.free()
    Am = A.astype(np.float64).T if ta else A.astype(np.float64)
    Bm = B.astype(np.float64).T if tb else B.astype(np.float64)
    ref = Am @ Bm
    if bias:
        ref = ref + bv
    if relu:
        ref = np.maximum(ref, 0)
    ref = ref * (mask > 0)
    if acc:
        ref = ref + C0
    return out, ref, err.value


@pytest.mark.parametrize("ta,tb,M,N,K", [
    (0, 0, 300, 520, 200),     # tensor cores, CTA pair
    (0, 1, 1024, 512, 512),
    (1, 0, 640, 256, 300),
    (1, 1, 100, 300, 64),      # tensor cores, single CTA (M <= 128)
    (0, 0, 1000, 10, 4092),    # skinny nn
    (1, 0, 1024, 10, 40000),   # skinny tn
    (0, 1, 1000, 4096, 10),    # skinny nt (128-bit stores)
    (0, 1, 100, 1030, 10),     # skinny nt (scalar stores)
    (0, 0, 333, 1000, 777),    # CUDA-core tiles
])
@pytest.mark.parametrize("bias,acc,relu", [(False, False, False), (True, False, True), (True, True, False)])
def test_masked_gemm_paths(ta, tb, M, N, K, bias, acc, relu):
    out, ref, err = _masked(ta, tb, M, N, K, bias=bias, acc=acc, relu=relu)
    assert err == 0
    assert_close(out, ref, 1e-5, f"masked {ta}{tb} {M}x{N}x{K}")
    # masked-out entries are exact zeros (or the accumulated value)
    if not acc:
        assert np.all(out[ref == 0] == 0)


@pytest.mark.parametrize("B,I,H,epochs", [(512, 64, 384, 3),      # head kernel, 2 rows a warp
                                          (8192, 1024, 4096, 2),  # the per-rank step at 8 GPUs
                                          (65536, 1024, 4096, 1)])  # one GPU: 4 rows a warp
def test_folded_training_is_bit_identical(B, I, H, epochs):
    """The program with its relu / relu-VJP passes folded into GEMM epilogues,
    its operand pairs prepared once per value and its classifier head fused
    (head.py: forward product, softmax, the chained cross_entropy/softmax VJP
    and the masked dX in one kernel) equals the unfused program bit for bit.
    (The bias sums folded into the pair steps add in another order and are
    checked separately below.)"""
    tl = load_backend()
    pr = tl.programs
    ast = pr.mlp3_train(B=B, I=I, H=H, C=10, epochs=epochs)
    feeds = pr.mlp3_inputs(B=B, I=I, H=H, C=10, seed=3)
    fetch = ["loss", "W1", "b1", "W2", "b2", "W3", "b3"]
    fused = tl.Program(ast, None, feeds=feeds, fetch=fetch, fuse_colsum=False)
    a = fused.run()
    steps = fused._all_steps()
    fused.free()
    masked = [s for s in steps if getattr(s, "fname", "") in ("tl_gemm_masked", "tl_gemm_pairs")
              and s.args[14 if s.fname == "tl_gemm_masked" else 16][0] == "ptr"]
    assert len(masked) == 1  # h1's gradient; h2's comes from the fused head
    assert sum(getattr(s, "fname", "") == "tl_head_ce" for s in steps) == 1
    # operand pairs prepared once per value: x (hoisted), a1, h2's and h1's gradients
    assert sum(getattr(s, "fname", "") == "tl_gemm_pair_prepare" for s in steps) == 4
    b = tl.Program(ast, None, feeds=feeds, fetch=fetch, fuse_ops=False).run()
    for k in fetch:
        assert np.array_equal(np.asarray(a[k]), np.asarray(b[k])), k


@pytest.mark.parametrize("B,I,H,epochs", [(512, 64, 384, 3), (8192, 1024, 4096, 2),
                                          (65536, 1024, 4096, 1)])
def test_folded_bias_sums_match(B, I, H, epochs):
    """With the bias gradients' row sums folded into the pair steps of the
    same gradients (pairs.py fuse_bias_colsums; both sums are taken in double
    and rounded once, in different orders), the loss and every parameter
    match the program that keeps the separate sums: rel 1e-6 of max|value|
    (in practice equal, a float step at most where a double sum rounds the
    other way)."""
    tl = load_backend()
    pr = tl.programs
    ast = pr.mlp3_train(B=B, I=I, H=H, C=10, epochs=epochs)
    feeds = pr.mlp3_inputs(B=B, I=I, H=H, C=10, seed=3)
    fetch = ["loss", "W1", "b1", "W2", "b2", "W3", "b3"]
    P = tl.Program(ast, None, feeds=feeds, fetch=fetch)
    a = P.run()
    steps = P._all_steps()
    P.free()
    assert sum(getattr(s, "fname", "") == "tl_gemm_pair_prepare_colsum" for s in steps) == 2
    b = tl.Program(ast, None, feeds=feeds, fetch=fetch, fuse_colsum=False).run()
    for k in fetch:
        x, y = np.asarray(a[k], np.float64), np.asarray(b[k], np.float64)
        assert np.abs(x - y).max() <= 1e-6 * max(np.abs(y).max(), 1e-30), k


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(1024, 4096, 2048),   # 64 cluster tiles: K split 8 ways
                                   (4096, 4096, 512)])   # 256 cluster tiles: K split 2 ways
@pytest.mark.parametrize("bias,acc,relu", [(True, False, True), (False, True, False)])
def test_split_k_gemm(ta, tb, M, N, K, bias, acc, relu):
    """Products of a few waves of 256 x 256 tiles split K across CTA pairs and
    fold the partial sums in split order before the epilogue."""
    out, ref, err = _masked(ta, tb, M, N, K, bias=bias, acc=acc, relu=relu)
    assert err == 0
    assert_close(out, ref, 1e-5, f"split-K {ta}{tb} {M}x{N}x{K}")


class _StorePath:
    """Select the CTA-pair epilogue's store path for a with-block."""

    def __init__(self, tma):
        self.tma = tma

    def __enter__(self):
        self.L = load_backend().runtime.lib()
        self.prev = ctypes.c_int(-1)
        assert self.L.tl_gemm_set_store_path(self.tma, ctypes.byref(self.prev)) == 0
        return self

    def __exit__(self, *exc):
        self.L.tl_gemm_set_store_path(self.prev.value, None)
        return False


@pytest.mark.parametrize("ta,tb,M,N,K,bias,acc,relu,masked", [
    (0, 0, 4096, 4096, 1024, True, False, True, False),   # the first layer's shape, scaled
    (0, 1, 4096, 4096, 2048, False, False, False, True),  # dX with the relu-VJP mask
    (1, 0, 1024, 4096, 8192, False, False, False, False),  # dW: K split 8 (partials by TMA)
    (0, 0, 1000, 1000, 520, True, False, True, True),     # ragged rows and columns
    (1, 1, 336, 260, 4096, True, False, False, False),    # ragged, split K
    (0, 0, 600, 300, 256, True, True, True, False),       # accumulate: per-row stores
])
def test_tma_store_epilogue_is_bit_identical(ta, tb, M, N, K, bias, acc, relu, masked):
    """The CTA-pair epilogue's TMA stores (32 x 32 slabs staged in shared
    memory, clipped at the edges; split-K partials through a 3-D map) give the
    per-row stores' results bit for bit, with bias, relu, the relu-VJP mask
    and accumulate, on ragged shapes; both within rel 1e-5 of float64."""
    outs = []
    for tma in (0, 1):
        with _StorePath(tma):
            if masked:
                out, ref, err = _masked(ta, tb, M, N, K, bias=bias, acc=acc, relu=relu)
            else:
                from test_gpu_gemm import _run
                out, ref, path, err = _run(ta, tb, M, N, K, bias=bias, acc=acc, relu=relu)
                assert path == 0
        assert err == 0
        outs.append(out)
    np.testing.assert_array_equal(outs[1], outs[0])
    assert_close(outs[1], ref, 1e-5, f"TMA-store epilogue {ta}{tb} {M}x{N}x{K}")


def test_store_path_rejects_unknown():
    assert load_backend().runtime.lib().tl_gemm_set_store_path(2, None) != 0
