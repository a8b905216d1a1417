"""Movement ops fused into elementwise kernels as index maps, on the GPU.

slice (kernel_generator.py:1112-1240), transpose (:1949-1972), reshape
(:2067-2086) and concat along axis 0 (:2092-2132) have no arithmetic, so
their results are compared exactly with the float64 oracle's (relu, add and
a copy of float32 values round the same in both).  Each case also checks the
kernel count: a chain of views ending in elementwise ops is one region
kernel, and the views themselves are never written.
"""
import numpy as np
import pytest

from conftest import load_backend
from oracle import OracleProgram

pytestmark = pytest.mark.gpu

tl = load_backend()
from tensor_lang_b200.programs import _call, _fill, _let  # noqa: E402
from tensor_lang_b200.steps import RegionStep, ViewStep  # noqa: E402


def _v(name, expr):
    return {"type": "let", "name": name, "ty": None, "requires_grad": False, "expr": expr}


def _slice(t, r0, r1, c0, c1):
    return {"type": "slice", "tensor": t, "specs": [{"type": "slice", "start": r0, "end": r1},
                                                    {"type": "slice", "start": c0, "end": c1}]}


def _run(ast, feeds, fetch, n_regions):
    P = tl.Program(ast, None, feeds=feeds, fetch=fetch)
    out = P.run()
    steps = P._all_steps()
    P.free()
    assert not any(isinstance(s, ViewStep) for s in steps)
    assert sum(isinstance(s, RegionStep) for s in steps) == n_regions, [s.label for s in steps]
    env = {k: {"shape": v} for k, v in P.shapes.items()}
    ref = OracleProgram(ast, env, dtype=np.float64, feeds=feeds).run()
    for k in fetch:
        np.testing.assert_array_equal(out[k], np.asarray(ref[k], np.float32), err_msg=k)
    return out


@pytest.mark.parametrize("R,C,r0,r1,c0,c1", [
    (64, 48, 4, 36, 8, 40),          # float4 path on the slice, gather after the transpose
    (1000, 777, 3, 998, 5, 700),     # ragged
    (4096, 4096, 0, 4096, 0, 4096),  # whole tensor, larger than L2
])
def test_relu_of_transpose_of_slice(R, C, r0, r1, c0, c1):
    ast = [_let("x", _fill((R, C)), (R, C)),
           _v("s", _slice("x", r0, r1, c0, c1)),
           _v("t", {"type": "transpose", "tensor": "s"}),
           _let("y", _call("relu", "t"))]
    x = np.random.default_rng(R).standard_normal((R, C)).astype(np.float32)
    _run(ast, {"x": x}, ["y"], 1)


@pytest.mark.parametrize("r1,r2,C", [(7, 4, 9), (512, 256, 1024), (3, 5, 4)])
def test_add_of_concat_and_its_transpose(r1, r2, C):
    R = r1 + r2
    ast = [_let("a", _fill((r1, C)), (r1, C)),
           _let("b", _fill((r2, C)), (r2, C)),
           _let("w", _fill((R, C)), (R, C)),
           _v("c", {"type": "concat", "tensors": ["a", "b"], "axis": 0}),
           _let("y", _call("add", "c", "w")),
           _v("ct", {"type": "transpose", "tensor": "c"}),
           _v("cs", _slice("ct", 0, C, 1, R - 1)),
           _let("z", _call("relu", "cs"))]
    rng = np.random.default_rng(R * C)
    feeds = {"a": rng.standard_normal((r1, C)).astype(np.float32),
             "b": rng.standard_normal((r2, C)).astype(np.float32),
             "w": rng.standard_normal((R, C)).astype(np.float32)}
    # y and z have different shapes: two segments of one launch
    _run(ast, feeds, ["y", "z"], 1)


def test_reshape_feeds_a_broadcast_free_chain():
    ast = [_let("x", _fill((256, 64)), (256, 64)),
           _let("w", _fill((128, 128)), (128, 128)),
           _v("r", {"type": "reshape", "tensor": "x", "new_shape": [128, 128]}),
           _let("y", _call("mult", "r", "w")),
           _let("z", _call("relu", "y"))]
    rng = np.random.default_rng(3)
    feeds = {"x": rng.standard_normal((256, 64)).astype(np.float32),
             "w": rng.standard_normal((128, 128)).astype(np.float32)}
    _run(ast, feeds, ["z"], 1)


def test_fetched_view_is_written_and_equal():
    ast = [_let("x", _fill((300, 200)), (300, 200)),
           _v("t", {"type": "transpose", "tensor": "x"}),
           _let("y", _call("relu", "t"))]
    x = np.random.default_rng(4).standard_normal((300, 200)).astype(np.float32)
    out = _run(ast, {"x": x}, ["t", "y"], 1)
    np.testing.assert_array_equal(out["t"], x.T)
