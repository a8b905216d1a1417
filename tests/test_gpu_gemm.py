"""tl_gemm on the GPU against a float64 product.

Covers every storage combination the executor uses (A as stored or
transposed, B as stored or transposed), ragged M/N/K (the tensor-core tiles
are 128x256x32, so partial tiles exercise TMA zero fill and masked stores;
K not a multiple of 32 exercises the zero columns of the bf16 pair
matrices), bias, relu and accumulate, under the default all-bf16 BF16X3
operand scheme, the TF32+bf16 scheme and the three-TF32 scheme, on 256 x 256
CTA-pair tiles (the default
for more than 128 rows; rows and columns past M and N exercise a pair whose
second CTA is wholly out of range) and on single-CTA tiles.  Tolerance: rel 1e-4 of max|C| (the GEMM bar);
the split products are expected near 1e-6 (split-TF32) to 5e-6 (BF16X3).  Also checks which path a
shape takes and that no kernel left a device error.
"""
import ctypes

import numpy as np
import pytest

from conftest import assert_close, load_backend

pytestmark = pytest.mark.gpu

SHAPES = [(64, 32, 32), (128, 256, 64), (200, 300, 100), (1024, 512, 512), (332, 1000, 780),
          (4096, 256, 4096), (256, 128, 16384)]


def _run(ta, tb, M, N, K, bias=False, acc=False, relu=False, seed=0):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    rng = np.random.default_rng(seed + M + N + K + 7 * ta + 3 * tb)
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    bv = rng.standard_normal(N).astype(np.float32)
    dA, dB, dC, db = (rt.DeviceBuffer(dev, a.shape) for a in (A, B, C0, bv))
    dA.upload(A)
    dB.upload(B)
    dC.upload(C0)
    db.upload(bv)
    lda, ldb = A.shape[1], B.shape[1]
    path = L.tl_gemm_path(ta, tb, M, N, K, dA.ptr, lda, dB.ptr, ldb, dC.ptr, N)
    rt.check(L.tl_gemm(ta, tb, M, N, K, dA.ptr, lda, dB.ptr, ldb, dC.ptr, N,
                       db.ptr if bias else None, 1 if acc else 0, 1 if relu else 0, dev.stream))
    out = dC.download()
    err = ctypes.c_int(0)
    rt.check(L.tl_device_error(ctypes.byref(err), 1))
    Am = A.astype(np.float64).T if ta else A.astype(np.float64)
    Bm = B.astype(np.float64).T if tb else B.astype(np.float64)
    ref = Am @ Bm
    if bias:
        ref = ref + bv
    if relu:
        ref = np.maximum(ref, 0)
    if acc:
        ref = ref + C0
    for b in (dA, dB, dC, db):
        b.free()
    return out, ref, path, err.value


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_layouts(ta, tb, M, N, K):
    out, ref, path, err = _run(ta, tb, M, N, K)
    assert err == 0
    assert path == 0, "this shape should run on the tensor cores"
    # the split product keeps near-fp32 accuracy: far inside the 1e-4 bar
    assert_close(out, ref, 1e-5, f"gemm ta={ta} tb={tb} {M}x{N}x{K}")


@pytest.mark.parametrize("bias,acc,relu", [(True, False, False), (False, True, False),
                                           (True, False, True), (True, True, False)])
def test_gemm_epilogues(bias, acc, relu):
    out, ref, path, err = _run(0, 0, 300, 520, 200, bias=bias, acc=acc, relu=relu)
    assert err == 0 and path == 0
    assert_close(out, ref, 1e-5, "epilogue")


@pytest.mark.parametrize("M,N,K", [(10, 64, 100), (7, 5, 3), (333, 1000, 777), (3, 6, 4)])
def test_gemm_cuda_core_shapes(M, N, K):
    # leading dimensions that are not a multiple of 4 floats (16 bytes), or
    # products too small or too narrow for 128x256 tiles, take the CUDA cores
    out, ref, path, err = _run(0, 0, M, N, K, bias=True)
    assert path == 1
    assert_close(out, ref, 1e-5, "cuda-core gemm")


@pytest.mark.parametrize("ta,tb,M,N,K", [(0, 0, 8192, 10, 4096), (1, 0, 2048, 10, 16384),
                                         (1, 0, 333, 7, 5000), (0, 1, 8192, 1024, 10),
                                         (0, 1, 70000, 40, 3), (0, 0, 16, 10, 4096),
                                         (0, 0, 1000, 10, 4092), (0, 0, 777, 24, 1000),
                                         (0, 0, 300, 10, 4095), (1, 0, 1024, 10, 40000),
                                         (1, 0, 516, 16, 3000), (1, 0, 4096, 24, 2000),
                                         (0, 1, 1000, 4096, 10), (0, 1, 65, 1028, 12),
                                         (0, 1, 100, 1030, 10)])
@pytest.mark.parametrize("bias,acc", [(True, False), (False, True)])
def test_gemm_skinny(ta, tb, M, N, K, bias, acc):
    """Classifier-head products (N or K of 10) on the bandwidth-bound kernels."""
    out, ref, path, err = _run(ta, tb, M, N, K, bias=bias, acc=acc)
    assert path == 1
    assert_close(out, ref, 1e-5, f"skinny {ta}{tb} {M}x{N}x{K}")


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(200, 300, 100), (332, 1000, 780), (256, 128, 16384)])
def test_gemm_three_tf32_scheme(ta, tb, M, N, K):
    """The three-TF32-MMA scheme (hi*hi + hi*lo + lo*hi) stays selectable."""
    tl = load_backend()
    L = tl.runtime.lib()
    prev = ctypes.c_int(-1)
    tl.runtime.check(L.tl_gemm_set_scheme(0, ctypes.byref(prev)))
    try:
        out, ref, path, err = _run(ta, tb, M, N, K, bias=True)
        assert err == 0 and path == 0
        assert_close(out, ref, 1e-5, f"3xTF32 {ta}{tb} {M}x{N}x{K}")
    finally:
        tl.runtime.check(L.tl_gemm_set_scheme(prev.value, None))
    assert prev.value == 2, "BF16X3 is the default scheme"


@pytest.mark.parametrize("scheme", [0, 1, 2])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(300, 520, 200), (1024, 512, 512)])
def test_gemm_single_cta_tiles(scheme, ta, tb, M, N, K):
    """128 x 256 single-CTA tiles (the CTA-pair tiles switched off)."""
    tl = load_backend()
    L = tl.runtime.lib()
    prev_pair, prev_scheme = ctypes.c_int(-1), ctypes.c_int(-1)
    tl.runtime.check(L.tl_gemm_set_cta_pair(0, ctypes.byref(prev_pair)))
    tl.runtime.check(L.tl_gemm_set_scheme(scheme, ctypes.byref(prev_scheme)))
    try:
        out, ref, path, err = _run(ta, tb, M, N, K, bias=True, relu=True)
        assert err == 0 and path == 0
        assert_close(out, ref, 1e-5, f"single-CTA {scheme} {ta}{tb} {M}x{N}x{K}")
    finally:
        tl.runtime.check(L.tl_gemm_set_cta_pair(prev_pair.value, None))
        tl.runtime.check(L.tl_gemm_set_scheme(prev_scheme.value, None))
    assert prev_pair.value == 1, "CTA-pair tiles are the default"


class _Scheme:
    """Select a GEMM operand scheme for the duration of a with-block."""

    def __init__(self, scheme):
        self.scheme = scheme

    def __enter__(self):
        tl = load_backend()
        self.L = tl.runtime.lib()
        self.prev = ctypes.c_int(-1)
        tl.runtime.check(self.L.tl_gemm_set_scheme(self.scheme, ctypes.byref(self.prev)))
        return self

    def __exit__(self, *exc):
        self.L.tl_gemm_set_scheme(self.prev.value, None)
        return False


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_tf32_bf16_scheme(ta, tb, M, N, K):
    """The split-TF32 scheme with bf16 corrections (hi*hi on TF32 plus one
    bf16 pair MMA) on CTA-pair tiles, split K included, within rel 1e-5."""
    with _Scheme(1):
        out, ref, path, err = _run(ta, tb, M, N, K, bias=True)
    assert err == 0 and path == 0
    assert_close(out, ref, 1e-5, f"tf32+bf16 {ta}{tb} {M}x{N}x{K}")


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_several_tiles_per_cluster(ta, tb):
    """A launch of many waves (74 x 16 CTA-pair tiles, ragged M, N and K on
    a 148-SM B200): each CTA pair computes two or more tiles in turn, the
    stage ring and accumulators running on across them."""
    M, N, K = 18900, 4056, 520
    out, ref, path, err = _run(ta, tb, M, N, K, bias=True, relu=True)
    assert err == 0 and path == 0
    assert_close(out, ref, 1e-5, f"tiles per cluster {ta}{tb} {M}x{N}x{K}")


def test_gemm_scheme_rejects_unknown():
    tl = load_backend()
    L = tl.runtime.lib()
    assert L.tl_gemm_set_scheme(7, None) != 0


def test_gemm_explicit_split_mode():
    tl = load_backend()
    L = tl.runtime.lib()
    L.tl_gemm_force_simt(2)
    try:
        for ta, tb in [(0, 0), (1, 1)]:
            out, ref, path, err = _run(ta, tb, 520, 264, 300)
            assert err == 0 and path == 0
            assert_close(out, ref, 1e-5, "explicit split")
    finally:
        L.tl_gemm_force_simt(0)


@pytest.mark.parametrize("scheme", [1, 2])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(300, 520, 200), (1000, 264, 1000)])
def test_prepared_pairs_match_per_call_pairs(scheme, ta, tb, M, N, K):
    """Pairs from tl_gemm_pair_prepare (both layouts from one read, ragged
    shapes: padding rows and columns) give the same product, bit for bit, as
    the pairs tl_gemm computes itself, under both pair schemes."""
    with _Scheme(scheme):
        _prepared_pairs_case(ta, tb, M, N, K)


def _prepared_pairs_case(ta, tb, M, N, K):
    tl = load_backend()
    rt = tl.runtime
    L = rt.lib()
    dev = rt.Device.get(0)
    rng = np.random.default_rng(M + N + K + ta + 2 * tb)
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    dA, dB = rt.DeviceBuffer(dev, A.shape), rt.DeviceBuffer(dev, B.shape)
    dA.upload(A)
    dB.upload(B)
    lda, ldb = A.shape[1], B.shape[1]
    assert L.tl_gemm_uses_pairs(ta, tb, M, N, K, lda, ldb) == 1
    # the layout each operand needs (include/tlb200.h), and both layouts of A
    a_layout, b_layout = (1 if ta else 0), (0 if tb else 1)
    pk = rt.DeviceBuffer(dev, (L.tl_gemm_pair_bytes(*A.shape, 0) // 4,))
    pm = rt.DeviceBuffer(dev, (L.tl_gemm_pair_bytes(*A.shape, 1) // 4,))
    pb = rt.DeviceBuffer(dev, (L.tl_gemm_pair_bytes(*B.shape, b_layout) // 4,))
    rt.check(L.tl_gemm_pair_prepare(dA.ptr, lda, A.shape[0], A.shape[1], pk.ptr, 0, pm.ptr, 0,
                                    dev.stream))
    rt.check(L.tl_gemm_pair_prepare(dB.ptr, ldb, B.shape[0], B.shape[1],
                                    pb.ptr if b_layout == 0 else None, 1,
                                    pb.ptr if b_layout == 1 else None, 1, dev.stream))
    pa = pm if a_layout == 1 else pk
    dC1, dC2 = rt.DeviceBuffer(dev, (M, N)), rt.DeviceBuffer(dev, (M, N))
    rt.check(L.tl_gemm(ta, tb, M, N, K, dA.ptr, lda, dB.ptr, ldb, dC1.ptr, N, None, 0, 0,
                       dev.stream))
    rt.check(L.tl_gemm_pairs(ta, tb, M, N, K, dA.ptr, lda, pa.ptr, dB.ptr, ldb, pb.ptr, dC2.ptr, N,
                             None, 0, 0, None, 0, dev.stream))
    c1, c2 = dC1.download(), dC2.download()
    for b in (dA, dB, pk, pm, pb, dC1, dC2):
        b.free()
    assert np.array_equal(c1, c2)
    ref = (A.astype(np.float64).T if ta else A.astype(np.float64)) @ \
        (B.astype(np.float64).T if tb else B.astype(np.float64))
    assert_close(c2, ref, 1e-5, f"prepared pairs {ta}{tb} {M}x{N}x{K}")


class _Schedule:
    """Select the CTA-pair tile schedule for the duration of a with-block."""

    def __init__(self, dynamic):
        self.dynamic = dynamic

    def __enter__(self):
        tl = load_backend()
        self.L = tl.runtime.lib()
        self.prev = ctypes.c_int(-1)
        tl.runtime.check(self.L.tl_gemm_set_tile_schedule(self.dynamic, ctypes.byref(self.prev)))
        return self

    def __exit__(self, *exc):
        self.L.tl_gemm_set_tile_schedule(self.prev.value, None)
        return False


@pytest.mark.parametrize("scheme", [0, 1, 2])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(200, 300, 100), (1024, 512, 512), (4096, 256, 4096),
                                   (256, 128, 16384), (18900, 4056, 520)])
def test_gemm_dynamic_tile_schedule(scheme, ta, tb, M, N, K):
    """Dynamic tile scheduling (cluster launch control: running CTA pairs
    take the tiles of clusters not launched yet) gives the static schedule's
    product bit for bit -- each tile's arithmetic is the same wherever it
    runs -- on ragged shapes, split K (256 x 128 x 16384) and launches of
    many waves, under every operand scheme, and within rel 1e-5 of float64."""
    with _Scheme(scheme):
        with _Schedule(0):
            static, ref, path, err = _run(ta, tb, M, N, K, bias=True, relu=True)
        assert err == 0 and path == 0
        with _Schedule(1):
            dyn, _, path, err = _run(ta, tb, M, N, K, bias=True, relu=True)
        assert err == 0 and path == 0
    np.testing.assert_array_equal(dyn, static)
    assert_close(dyn, ref, 1e-5, f"dynamic schedule {scheme} {ta}{tb} {M}x{N}x{K}")


def test_gemm_dynamic_schedule_accumulate_and_plan():
    tl = load_backend()
    L = tl.runtime.lib()
    with _Schedule(1):
        out, ref, path, err = _run(0, 1, 2048, 1024, 768, bias=True, acc=True)
        plan = (ctypes.c_int * 4)()
        tl.runtime.check(L.tl_gemm_tc_plan(65536, 4096, 4096, plan))
    assert err == 0 and path == 0
    assert_close(out, ref, 1e-5, "dynamic schedule, accumulate")
    assert plan[2] == 1 and plan[3] == 4096, "one tile per cluster launch"
