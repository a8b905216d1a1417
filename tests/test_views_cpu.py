"""Index maps of the movement ops (``views.py``) and the decision to fold a
view into its readers or write it (``steps.resolve_views``), on the CPU.

Each map is evaluated here by gathering through its offsets and compared
with NumPy's slice / transpose / reshape / concatenate of the same arrays,
chained in every order the 2-D ops allow.
"""
import itertools

import numpy as np
import pytest

from conftest import load_backend

tl = load_backend()
from tensor_lang_b200 import views as V  # noqa: E402
from tensor_lang_b200.programs import _call, _fill, _let  # noqa: E402
from tensor_lang_b200.steps import EW, RegionStep, ViewStep  # noqa: E402


def gather(m, shape, arrays):
    """Evaluate map ``m`` over output ``shape``: out[k] = src.flat[offset(k)]."""
    out = np.empty(shape, np.float64)
    for k in itertools.product(*[range(d) for d in shape]):
        node = m
        while node[0] == "pw":
            node = node[3] if k[node[1]] < node[2] else node[4]
        _, src, base, strides = node
        out[k] = arrays[src].reshape(-1)[base + sum(a * b for a, b in zip(k, strides))]
    return out


def _slice(m, shp, r0, r1, c0, c1):
    out = (r1 - r0, c1 - c0)
    return V.View("slice", "o", out, ["i"], (r0, c0)).build([m], [shp]), out


def _transpose(m, shp):
    out = (shp[1], shp[0])
    return V.View("transpose", "o", out, ["i"], ()).build([m], [shp]), out


def test_single_ops_match_numpy():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 9))
    y = rng.standard_normal((4, 9))
    A = {"x": x, "y": y}
    mx = V.identity(x.shape, "x")
    m, s = _slice(mx, x.shape, 2, 6, 1, 8)
    np.testing.assert_array_equal(gather(m, s, A), x[2:6, 1:8])
    m, s = _transpose(mx, x.shape)
    np.testing.assert_array_equal(gather(m, s, A), x.T)
    m = V.View("reshape", "o", (3, 21), ["x"], ()).build([mx], [x.shape])
    np.testing.assert_array_equal(gather(m, (3, 21), A), x.reshape(3, 21))
    m = V.View("concat0", "o", (11, 9), ["x", "y"], ()).build(
        [mx, V.identity(y.shape, "y")], [x.shape, y.shape])
    np.testing.assert_array_equal(gather(m, (11, 9), A), np.concatenate([x, y]))


@pytest.mark.parametrize("r0,r1,c0,c1", [(0, 11, 0, 9), (2, 9, 3, 8), (7, 11, 0, 4),
                                         (0, 7, 2, 9), (6, 8, 1, 2)])
def test_compositions_match_numpy(r0, r1, c0, c1):
    rng = np.random.default_rng(r0 * 100 + c0)
    x = rng.standard_normal((7, 9))
    y = rng.standard_normal((4, 9))
    A = {"x": x, "y": y}
    cat = np.concatenate([x, y])
    m = V.View("concat0", "o", cat.shape, ["x", "y"], ()).build(
        [V.identity(x.shape, "x"), V.identity(y.shape, "y")], [x.shape, y.shape])
    # slice of a concat: the split moves or disappears
    ms, ss = _slice(m, cat.shape, r0, r1, c0, c1)
    np.testing.assert_array_equal(gather(ms, ss, A), cat[r0:r1, c0:c1])
    # transpose of that: the split moves to axis 1
    mt, st = _transpose(ms, ss)
    np.testing.assert_array_equal(gather(mt, st, A), cat[r0:r1, c0:c1].T)
    # slice of the transpose
    mts, sts = _slice(mt, st, 0, st[0], 0, max(1, st[1] - 1))
    np.testing.assert_array_equal(gather(mts, sts, A), cat[r0:r1, c0:c1].T[:, :max(1, st[1] - 1)])
    # a reshape composes only with a whole tensor in row-major order
    whole = V.View("reshape", "o", (9, 7), ["x"], ()).build([V.identity(x.shape, "x")], [x.shape])
    assert whole is not None
    assert V.View("reshape", "o", (ss[1], ss[0]), ["i"], ()).build([ms], [ss]) is None or \
        V.is_whole(ms, ss)


def test_vec4_rule():
    m = V.identity((8, 16), "x")
    assert V.vec4_ok(m, 2)
    t, _ = _transpose(m, (8, 16))
    assert not V.vec4_ok(t, 2)            # stride 16 along the last axis
    s, _ = _slice(m, (8, 16), 1, 5, 4, 12)
    assert V.vec4_ok(s, 2)                 # base 20, strides (16, 1)
    s, _ = _slice(m, (8, 16), 1, 5, 3, 11)
    assert not V.vec4_ok(s, 2)             # base 19: not 16-byte aligned


def _prog(stmts, fetch):
    return tl.Program(stmts, None, fetch=fetch)


def _slice_expr(t, r0, r1, c0, c1):
    return {"type": "slice", "tensor": t,
            "specs": [{"type": "slice", "start": r0, "end": r1},
                      {"type": "slice", "start": c0, "end": c1}]}


def _view_let(name, expr):
    return {"type": "let", "name": name, "ty": None, "requires_grad": False, "expr": expr}


def test_chain_is_one_region():
    ast = [_let("x", _fill((64, 48), 1.0), (64, 48)),
           _view_let("s", _slice_expr("x", 4, 36, 8, 40)),
           _view_let("t", {"type": "transpose", "tensor": "s"}),
           _let("y", _call("relu", "t"))]
    P = _prog(ast, ["y"])
    P._fuse_all()
    steps = [s for s in P._all_steps() if "y" in s.writes]
    assert len(steps) == 1 and isinstance(steps[0], RegionStep)
    assert not any(isinstance(s, ViewStep) for s in P._all_steps())
    assert "s" not in P.live and "t" not in P.live


def test_fetched_view_is_written():
    ast = [_let("x", _fill((64, 48), 1.0), (64, 48)),
           _view_let("t", {"type": "transpose", "tensor": "x"}),
           _let("y", _call("relu", "t"))]
    P = _prog(ast, ["y", "t"])
    P._fuse_all()
    writers = [s for s in P._all_steps() if "t" in s.writes]
    assert len(writers) == 1 and getattr(writers[0], "fname", "") == "tl_transpose2d"


def test_view_read_by_a_library_kernel_is_written():
    ast = [_let("x", _fill((64, 48), 1.0), (64, 48)),
           _view_let("t", {"type": "transpose", "tensor": "x"}),
           _let("s", {"type": "sum", "tensor": "t", "axis": 1})]
    P = _prog(ast, ["s"])
    P._fuse_all()
    assert any(getattr(s, "fname", "") == "tl_transpose2d" for s in P._all_steps())


def test_view_of_a_region_value_is_read_after_it_is_written():
    # square: relu(x) and the transpose's reader share one iteration shape
    ast = [_let("x", _fill((32, 32), 1.0), (32, 32)),
           _let("a", _call("relu", "x")),
           _view_let("t", {"type": "transpose", "tensor": "a"}),
           _let("y", _call("add", "t", "x"))]
    P = _prog(ast, ["y"])
    P._fuse_all()
    regions = [s for s in P._all_steps() if isinstance(s, RegionStep)]
    wa = [i for i, s in enumerate(regions) if "a" in s.writes]
    ry = [i for i, s in enumerate(regions) if "y" in s.writes]
    assert wa and ry and wa[0] < ry[0], "the transpose must read a from memory, after it is written"
