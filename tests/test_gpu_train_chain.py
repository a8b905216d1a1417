"""Whole training runs of the 3-layer MLP (1024 -> 4096 -> 4096 -> 10) on the
GPU against the float64 oracle: 3 epochs on the full batch of 65536 rows,
and 100 epochs on a batch of 4096, from the same seeded data and weights.

The oracle's results come from ``tests/golden/train_chain.npz``, written by
``tests/golden/make_train_chain.py`` (a float64 full-batch step takes
minutes of CPU; the fixture keeps what the comparison needs).

What is compared, and why this way:

* the loss of the last epoch: rel 1e-4;
* the weights after the run: rel 1e-4, atol 1e-4 * max|ref| (exactly for
  the head, through the fixed projections ``W @ V`` for the two large
  weights; the biases start at zero, so their final values are their
  updates, compared next);
* each parameter's update ``D = P_final - P_initial`` (the parameters
  themselves hide it: the update is ~1e-3 of ``P``), in relative Frobenius
  norm ``||D_gpu - D_ref|| / ||D_ref||``, exactly for the biases and the
  head, estimated from ``D @ V`` for the large weights.  An elementwise rel
  1e-4 bound on an update is met by no float32 evaluation, the reference's
  own included: a relu whose pre-activation lies within rounding distance of
  0 takes either branch, and one such flip moves a whole row of ``h1_grad``
  into every column of ``W1_grad`` and a whole entry into ``b1_grad``.  The
  fixture records how far the float32 oracle -- the reference's own
  arithmetic -- lands from float64 on the same run (``dev32``, printed
  beside each GPU figure): up to 4.2e-3 (``W1`` after 3 full-batch epochs).
  Flips make the deviation chaotic rather than proportional to the
  products' error (the split-TF32 GEMMs, more accurate than BF16X3, moved
  ``b1`` farther over 100 epochs), so the bound is absolute: 1e-2 of the
  update's norm.  A wiring error in the loop (a stale operand, a lost
  update, a wrong divisor) moves an update by O(1).  Each kernel on this
  path is held to rel 1e-4 (GEMMs) or 1e-5 from its own inputs at
  these sizes in ``tests/test_gpu_full_size.py``.
"""
import importlib.util

import numpy as np
import pytest

from conftest import GOLDEN, assert_close, load_backend

pytestmark = pytest.mark.gpu

FIXTURE = GOLDEN / "train_chain.npz"
_spec = importlib.util.spec_from_file_location("make_train_chain", GOLDEN / "make_train_chain.py")
mk = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mk)


def _scheme(code):
    tl = load_backend()
    import ctypes
    prev = ctypes.c_int(-1)
    tl.runtime.check(tl.runtime.lib().tl_gemm_set_scheme(code, ctypes.byref(prev)))
    return prev.value


@pytest.mark.skipif(not FIXTURE.exists(), reason="train_chain.npz not generated")
@pytest.mark.parametrize("scheme", [2, 1], ids=["bf16x3", "tf32bf16"])
@pytest.mark.parametrize("run", ["full", "b4096"])
def test_training_run_matches_the_float64_oracle(run, scheme):
    tl = load_backend()
    fx = np.load(FIXTURE)
    if f"{run}/batch" not in fx.files:
        pytest.skip(f"train_chain.npz holds no {run!r} run")
    B, epochs = int(fx[f"{run}/batch"]), int(fx[f"{run}/epochs"])
    pr = tl.programs
    feeds = mk.batch_inputs(pr, B)
    ast = pr.mlp3_train(B=B, epochs=epochs, **mk.DIMS)
    prev = _scheme(scheme)
    try:
        P = tl.Program(ast, None, feeds=feeds, fetch=list(mk.PARAMS) + ["loss"])
        out = P.run()
        P.free()
    finally:
        _scheme(prev)
    assert_close(np.asarray(out["loss"]).reshape(1), np.asarray(fx[f"{run}/loss64"]).reshape(1),
                 1e-4, f"{run} loss")
    bad = []
    for p in mk.PARAMS:
        D = out[p].astype(np.float64) - feeds[p].astype(np.float64)
        norm = float(fx[f"{run}/{p}/norm"])
        if p in mk.PROJECTED:
            V = mk.proj_matrix(p, D.shape[1])
            err = np.linalg.norm(D @ V - fx[f"{run}/{p}/proj"]) / np.sqrt(mk.NPROJ)
            ref = feeds[p].astype(np.float64) @ V + fx[f"{run}/{p}/proj"]
            got = out[p].astype(np.float64) @ V
        else:
            err = np.linalg.norm(D - fx[f"{run}/{p}/delta"])
            ref = feeds[p].astype(np.float64) + fx[f"{run}/{p}/delta"]
            got = out[p].astype(np.float64)
        # the weights themselves (projected for the large ones): rel 1e-4; a
        # bias starts at zero, so its final value is its update, checked below
        if p.startswith("W"):
            assert_close(got, ref, 1e-4, f"{run} {p}")
        dev = err / norm
        dev32 = float(fx[f"{run}/{p}/dev32"])
        print(f"{run} scheme {scheme} {p}: update deviation {dev:.2e} (float32 oracle {dev32:.2e})")
        if dev > 1e-2:
            bad.append(f"{p}: {dev:.3e} (float32 oracle {dev32:.3e})")
    assert not bad, f"{run}: " + "; ".join(bad)
