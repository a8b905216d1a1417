"""Generate ``train_chain.npz``: float64 oracle results of the 3-layer MLP
training loop (1024 -> 4096 -> 4096 -> 10, relu, softmax -> cross_entropy,
SGD lr 0.01) that the GPU tests compare whole training runs against.

    python tests/golden/make_train_chain.py [--out tests/golden/train_chain.npz]

Runs only the oracle (``oracle/tl_oracle.py``) on the CPU; about 45 minutes
on 8 cores, most of it the float64 full-batch steps.  Two runs, both from
``programs.mlp3_inputs(seed=0)``:

* ``full``: the full batch of 65536 rows, 3 epochs;
* ``b4096``: the first 4096 rows of the same generator's batch (a batch of
  4096 drawn with seed 0), 100 epochs.

Each run is computed by the float64 oracle (the correctness reference) and
by the float32 oracle (the reference's own arithmetic).  A 4096 x 4096
parameter update is too large to commit, so the fixture keeps, per
parameter ``P`` with update ``D = P_final - P_initial``:

* ``<run>/<P>/delta`` -- ``D`` itself for the biases and the 4096 x 10 head;
* ``<run>/<P>/proj`` -- ``D @ V`` for the two large weights, ``V`` four
  standard-normal columns from ``default_rng(<seed of P>)``; for a Gaussian
  ``V``, ``||E @ V||_F^2 / 4`` estimates ``||E||_F^2`` of an error ``E``;
* ``<run>/<P>/norm`` -- ``||D||_F``;
* ``<run>/<P>/dev32`` -- ``||D32 - D64||_F / ||D64||_F``: how far the
  float32 oracle's update is from the float64 one (exact, not projected);
* ``<run>/loss64``, ``<run>/loss32`` -- the loss of the last epoch.

The float32 deviation is printed beside the GPU's by the test: a relu whose
pre-activation sits within rounding distance of 0 can take either branch in
any float32 evaluation, and one such flip moves a whole row or column of a
weight gradient, so no float32 run matches a float64 update elementwise
(see ``tests/test_gpu_train_chain.py``).
"""
from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import OracleProgram  # noqa: E402

PARAMS = ("W1", "b1", "W2", "b2", "W3", "b3")
PROJECTED = ("W1", "W2")
NPROJ = 4
RUNS = {"full": (65536, 3), "b4096": (4096, 100)}
DIMS = dict(I=1024, H=4096, C=10)


def _programs():
    from __graft_entry__ import load_package
    return load_package().programs


def shape_env(ast):
    from __graft_entry__ import load_package
    return {k: {"shape": v} for k, v in load_package().shapes.complete_env(ast, {}).items()}


def proj_matrix(name: str, cols: int) -> np.ndarray:
    """The fixed projection ``V`` of a parameter (also used by the test)."""
    seed = 1000 + PARAMS.index(name)
    return np.random.default_rng(seed).standard_normal((cols, NPROJ))


def batch_inputs(pr, B: int) -> dict:
    """The run's inputs: the parameters of ``mlp3_inputs(seed=0)`` and the
    first ``B`` rows of its 65536-row batch."""
    full = pr.mlp3_inputs(B=65536, seed=0, **DIMS)
    if B == 65536:
        return full
    out = dict(full)
    out["x"] = np.ascontiguousarray(full["x"][:B])
    out["t"] = np.ascontiguousarray(full["t"][:B])
    return out


def run_oracle(pr, B: int, epochs: int, dtype):
    ast = pr.mlp3_train(B=B, epochs=epochs, **DIMS)
    feeds = batch_inputs(pr, B)
    t0 = time.time()
    out = OracleProgram(ast, shape_env(ast), dtype=dtype, feeds=feeds).run()
    dt = time.time() - t0
    res = {p: np.asarray(out[p], np.float64) - feeds[p].astype(np.float64) for p in PARAMS}
    return res, float(np.asarray(out["loss"]).reshape(-1)[0]), dt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "train_chain.npz"))
    ap.add_argument("--runs", default=",".join(RUNS))
    args = ap.parse_args()
    pr = _programs()
    data = {}
    out = Path(args.out)
    if out.exists():
        with np.load(out) as old:
            data.update({k: old[k] for k in old.files})
    for run in args.runs.split(","):
        B, epochs = RUNS[run]
        d64, loss64, t64 = run_oracle(pr, B, epochs, np.float64)
        print(f"{run}: float64 oracle {t64:.0f} s, loss {loss64!r}", flush=True)
        d32, loss32, t32 = run_oracle(pr, B, epochs, np.float32)
        print(f"{run}: float32 oracle {t32:.0f} s, loss {loss32!r}", flush=True)
        data[f"{run}/loss64"] = np.float64(loss64)
        data[f"{run}/loss32"] = np.float64(loss32)
        data[f"{run}/batch"] = np.int64(B)
        data[f"{run}/epochs"] = np.int64(epochs)
        for p in PARAMS:
            D = d64[p]
            data[f"{run}/{p}/norm"] = np.float64(np.linalg.norm(D))
            data[f"{run}/{p}/dev32"] = np.float64(np.linalg.norm(d32[p] - D) / np.linalg.norm(D))
            if p in PROJECTED:
                data[f"{run}/{p}/proj"] = D @ proj_matrix(p, D.shape[1])
            else:
                data[f"{run}/{p}/delta"] = D
            print(f"  {p}: |D| {np.linalg.norm(D):.4e}, float32 deviation "
                  f"{float(data[f'{run}/{p}/dev32']):.3e}", flush=True)
        np.savez(out, **data)
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
