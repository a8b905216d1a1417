"""Parity of the benchmark workloads on the GPU against the oracle.

Tolerances: elementwise, reductions, softmax, norms rel 1e-5; GEMM and
training rel 1e-4; comparison masks and argmax/argmin bit-exact.  Each with
atol = rtol * max|ref| of the tensor.  Full-size GEMMs are checked through a
size-independent projection identity instead of a float64 product.
"""
import numpy as np
import pytest

from conftest import assert_close, load_backend
from oracle import OracleProgram

pytestmark = pytest.mark.gpu


def _env(P):
    return {k: {"shape": v} for k, v in P.shapes.items()}


@pytest.mark.parametrize("N", [64, 1000, 2048, 8192])
def test_fused_chain(N):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.fused_chain(N), pr.fused_chain_inputs(N, seed=N)
    P = tl.Program(ast, None, feeds=feeds, fetch=["y", "m"])
    out = P.run()
    regions = [s for s in P._all_steps() if type(s).__name__ == "RegionStep"]
    assert len(regions) == 1, "mult/add/gelu/greater must fuse into one kernel"
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    assert_close(out["y"], ref["y"], 1e-5, "y")
    # the mask is exact for the operands the kernel computed ...
    np.testing.assert_array_equal(out["m"], (out["y"] > 0).astype(np.float32))
    # ... and for the reference's float32 evaluation order
    ref32 = OracleProgram(ast, _env(P), dtype=np.float32, feeds=feeds).run()
    np.testing.assert_array_equal(out["m"], ref32["m"])
    P.free()


@pytest.mark.parametrize("R,C", [(7, 5), (64, 10), (300, 257), (1024, 4096), (16384, 4096)])
def test_reductions_softmax_layer_norm(R, C):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.reductions(R, C), pr.reductions_inputs(R, C, seed=1)
    names = [n for n, _, _ in pr.REDUCTION_OPS] + ["sm", "ln"]
    P = tl.Program(ast, None, feeds=feeds, fetch=names)
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    for n in names:
        if n.startswith("arg"):
            np.testing.assert_array_equal(out[n], np.asarray(ref[n], np.float32), err_msg=n)
        else:
            assert_close(out[n], ref[n], 1e-5, n)
    P.free()


def test_mlp2_training_step():
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.mlp2_step(), pr.mlp2_inputs(seed=0)
    P = tl.Program(ast, None, feeds=feeds)
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    for k in ["h", "a", "z", "p", "loss", "W1_grad", "b1_grad", "W2_grad", "b2_grad",
              "W1_new", "b1_new", "W2_new", "b2_new", "z_grad", "p_grad", "h_grad", "a_grad"]:
        assert_close(out[k], ref[k], 1e-4, k)
    P.free()


@pytest.mark.parametrize("M,K,N", [(64, 32, 48), (520, 264, 136), (1024, 512, 256)])
def test_linear_layer_autograd(M, K, N):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.linear_layer(M, K, N), pr.linear_layer_inputs(M, K, N, seed=2)
    P = tl.Program(ast, None, feeds=feeds, fetch=["z", "y", "loss", "X_grad", "W_grad", "b_grad"])
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    for k in ["z", "y", "loss", "X_grad", "W_grad", "b_grad"]:
        assert_close(out[k], ref[k], 1e-4, k)
    P.free()


def test_mlp3_training_loop_small():
    tl = load_backend()
    pr = tl.programs
    kw = dict(B=512, I=64, H=128, C=10)
    ast = pr.mlp3_train(epochs=5, **kw)
    feeds = pr.mlp3_inputs(seed=3, **kw)
    fetch = ["W1", "b1", "W2", "b2", "W3", "b3", "loss"]
    P = tl.Program(ast, None, feeds=feeds, fetch=fetch)
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    for k in fetch:
        assert_close(out[k], ref[k], 1e-4, k)
    P.free()


def test_mlp3_graph_replay_matches_eager():
    tl = load_backend()
    pr = tl.programs
    kw = dict(B=256, I=32, H=64, C=10)
    ast = pr.mlp3_train(epochs=4, **kw)
    feeds = pr.mlp3_inputs(seed=4, **kw)
    fetch = ["W1", "W2", "W3", "b3"]
    a = tl.Program(ast, None, feeds=feeds, fetch=fetch, use_graphs=True).run()
    b = tl.Program(ast, None, feeds=feeds, fetch=fetch, use_graphs=False).run()
    for k in fetch:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)


def test_numpy_semantics_match_the_oracle():
    """semantics="numpy": the square broadcast reads B[j] and the softmax ->
    cross_entropy gradient is (p - t) / B, on the GPU as in the oracle."""
    tl = load_backend()
    pr = tl.programs
    N = 1000
    ast, feeds = pr.fused_chain(N), pr.fused_chain_inputs(N, seed=5)
    P = tl.Program(ast, None, feeds=feeds, fetch=["y", "m"], semantics="numpy")
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds, semantics="numpy").run()
    ref32 = OracleProgram(ast, _env(P), dtype=np.float32, feeds=feeds, semantics="numpy").run()
    P.free()
    assert_close(out["y"], ref["y"], 1e-5, "y")
    np.testing.assert_array_equal(out["m"], ref32["m"])
    ast, feeds = pr.mlp2_step(), pr.mlp2_inputs(seed=2)
    P = tl.Program(ast, None, feeds=feeds, semantics="numpy")
    out = P.run()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds, semantics="numpy").run()
    P.free()
    for k in ["loss", "z_grad", "p_grad", "W1_grad", "b1_grad", "W2_grad", "b2_grad",
              "W1_new", "b2_new"]:
        assert_close(out[k], ref[k], 1e-4, k)
