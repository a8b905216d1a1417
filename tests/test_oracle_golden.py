"""Pin the oracle: it must reproduce the reference's own results.

* every ``// @EXPECTED`` block of the reference's 106 test programs;
* every tensor the reference executor wrote for those programs
  (``tests/golden/ref_programs.json``, produced by ``make_golden.py``);
* gradients of the reference ``autograd.ComputationGraph`` on seeded graphs.
"""
import numpy as np
import pytest

from conftest import arr, golden
from oracle import OracleProgram
from oracle.tl_oracle import _Graph, _Node

PROGS = golden("ref_programs.json")
NAMES = sorted(k for k, v in PROGS.items() if v["typecheck_ok"])


def _run(rec, dt, mode="extended"):
    lf = {k: arr(v) for k, v in rec["load_files"].items()}
    return OracleProgram(rec["ast"], rec["env"], dtype=dt, load_files=lf, record=mode).run()


def test_golden_corpus_complete():
    assert len(PROGS) == 106
    assert all(v["expected"] for v in PROGS.values())
    # load_dynamic / load_inferred type-check only once basics.tl has saved its files
    assert len(NAMES) == 106


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("dt", [np.float64, np.float32], ids=["f64", "f32"])
def test_expected_block(name, dt):
    rec = PROGS[name]
    out = _run(rec, dt)
    for key, exp in rec["expected"].items():
        assert key in out, key
        got = np.asarray(out[key], dtype=np.float64)
        e = np.asarray(exp, dtype=np.float64)
        if e.size == 1 and got.size == 1:
            assert np.isclose(got.item(), e.item(), rtol=1e-5, atol=1e-8), (key, got, e)
        else:
            assert got.shape == e.shape, (key, got.shape, e.shape)
            assert np.allclose(got, e, rtol=1e-5, atol=1e-8), (key, got, e)


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("mode", ["reference", "extended"])
def test_every_reference_tensor(name, mode):
    rec = PROGS[name]
    out = _run(rec, np.float64, mode)
    for key, ref in rec["outputs"].items():
        r = arr(ref)
        got = np.asarray(out[key], dtype=np.float64)
        assert got.shape == r.shape, key
        assert np.allclose(got, r, rtol=1e-5, atol=1e-6), key


@pytest.mark.parametrize("case", golden("autograd_cases.json"), ids=lambda c: c["label"])
def test_autograd_matches_reference_graph(case):
    g = _Graph(np.float32)
    for k, v in case["tensors"].items():
        g.register(k, arr(v).astype(np.float32), k in case["requires_grad"])
    for op, out, ins, meta in case["nodes"]:
        g.nodes.append(_Node(op, out, ins, meta))
    g.backward(case["loss"])
    assert sorted(g.grads) == sorted(case["gradients"])
    for k, v in case["gradients"].items():
        # float32 restatement is bit-identical to the reference graph
        np.testing.assert_array_equal(g.grads[k], arr(v).astype(np.float32))
