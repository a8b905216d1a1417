"""The tensor-core GEMM launch plan (tl_gemm_tc_plan), on the CPU: the K
splits and tiles-per-cluster decisions for the training step's shapes, and
their invariants over a sweep of shapes (148 SMs, 74 CTA pairs, when no GPU
is visible).

Rules under test (csrc/gemm_tc.cu): a launch of few cluster waves splits K
until the waves are >= 95% full, keeping >= 8 k-blocks per split; a launch of
many waves lets each CTA pair compute up to four tiles in turn while at least
four waves of clusters remain and the last wave is no emptier (within 1%)
than with one tile per cluster.  The automatic tile schedule is dynamic
(running CTA pairs take pending clusters' tiles) where that would leave one
tile per cluster, and for K <= 1024."""
import ctypes
import math

import pytest

from conftest import load_backend

SLOTS = 74  # CTA pairs on a 148-SM B200


def _plan(M, N, K):
    L = load_backend().runtime.lib()
    out = (ctypes.c_int * 4)()
    assert L.tl_gemm_tc_plan(M, N, K, out) == 0
    return tuple(out)


@pytest.mark.parametrize("M,N,K,plan", [
    (65536, 4096, 4096, (1, 1, 4, 1024)),   # hidden forward / dX: four tiles per pair
    (65536, 4096, 1024, (2, 1, 1, 4096)),   # first layer: short tiles, dynamic schedule
    (4096, 4096, 65536, (2, 2, 1, 512)),    # dW2: 256 tiles, K split in two, dynamic
    (1024, 4096, 65536, (2, 8, 1, 512)),    # dW1: 64 tiles, K split eight ways, dynamic
    (8192, 4096, 4096, (2, 1, 1, 512)),     # the 8-GPU per-rank forward: 6.9 waves, dynamic
    (64, 256, 256, (0, 1, 1, 1)),           # one row tile: single-CTA 128 x 256
])
def test_training_step_plans(M, N, K, plan):
    assert _plan(M, N, K) == plan


def _eff(clusters):
    return clusters / (math.ceil(clusters / SLOTS) * SLOTS)


@pytest.mark.parametrize("M", [256, 1000, 4096, 9472, 18944, 32768, 65536, 131072])
@pytest.mark.parametrize("N", [256, 1000, 4096, 8192])
@pytest.mark.parametrize("K", [32, 520, 4096, 65536])
def test_plan_invariants(M, N, K):
    pair, splits, tpc, launched = _plan(M, N, K)
    assert pair in (1, 2)
    # the automatic schedule: dynamic where static would leave one tile per
    # cluster, and for short tiles
    assert (pair == 2) == (tpc == 1 or K <= 1024) and (pair == 1 or tpc == 1)
    tiles = math.ceil(M / 256) * math.ceil(N / 256)
    work = tiles * splits
    nk = math.ceil(K / 32)
    assert 1 <= splits <= 8 and 1 <= tpc <= 4
    # every (tile, split) is computed exactly once and no cluster is empty
    assert launched == math.ceil(work / tpc) and (launched - 1) * tpc < work
    if splits > 1:
        assert tiles < 8 * SLOTS and nk // splits >= 8 and _eff(work) >= 0.95
        assert tpc == 1
    if tpc > 1:
        assert launched >= 4 * SLOTS and _eff(launched) >= _eff(work) - 0.01


def test_plan_follows_the_cta_pair_switch():
    L = load_backend().runtime.lib()
    prev = ctypes.c_int(-1)
    assert L.tl_gemm_set_cta_pair(0, ctypes.byref(prev)) == 0
    try:
        assert _plan(65536, 4096, 4096) == (0, 1, 1, 16 * 512)
    finally:
        L.tl_gemm_set_cta_pair(prev.value, None)
    assert _plan(65536, 4096, 4096)[0] == 1


def test_plan_rejects_empty_products():
    L = load_backend().runtime.lib()
    out = (ctypes.c_int * 4)()
    assert L.tl_gemm_tc_plan(0, 4096, 4096, out) != 0
    assert L.tl_gemm_tc_plan(64, 4096, 0, out) != 0


@pytest.mark.parametrize("M,N,K,plan", [
    (65536, 4096, 4096, (2, 1, 1, 4096)),   # one tile per cluster launch
    (4096, 4096, 65536, (2, 2, 1, 512)),    # the K splits are unchanged
    (8192, 4096, 4096, (2, 1, 1, 512)),
])
def test_plan_under_the_dynamic_schedule(M, N, K, plan):
    L = load_backend().runtime.lib()
    prev = ctypes.c_int(-1)
    assert L.tl_gemm_set_tile_schedule(1, ctypes.byref(prev)) == 0
    try:
        assert _plan(M, N, K) == plan
    finally:
        L.tl_gemm_set_tile_schedule(prev.value, None)
    assert prev.value == 2
    assert L.tl_gemm_set_tile_schedule(3, None) != 0
