"""Data-parallel training on 2 GPUs equals single-GPU training.

Runs ``tests/dp_worker.py`` under ``torch.distributed.run`` (one process per
GPU, NCCL over NVLink), then the same program on one GPU, and compares the
parameters after 4 epochs (rel 1e-4: the all-reduced gradient sums the
shards in a different order than one GPU sums the whole batch).  The hidden
biases start at +-0.5 so that no relu decision sits at float32 rounding
distance from 0 (dp_worker.margin_biases).  Skipped when fewer than 2 GPUs
are visible.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO, assert_close, load_backend
from dp_worker import margin_biases
from oracle import OracleProgram

pytestmark = pytest.mark.gpu


def _ngpus():
    tl = load_backend()
    n = ctypes.c_int(0)
    tl.runtime.lib().tl_device_count(ctypes.byref(n))
    return n.value


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_dp2_matches_single_gpu(tmp_path):
    out = tmp_path / "dp.npz"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NCCL_DEBUG="WARN")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29547", str(REPO / "tests" / "dp_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    got = np.load(out)

    tl = load_backend()
    kw = dict(B=512, I=64, H=128, C=10)
    ast = tl.programs.mlp3_train(epochs=4, **kw)
    feeds = margin_biases(tl.programs.mlp3_inputs(seed=5, **kw))
    P = tl.Program(ast, None, feeds=feeds, fetch=list(got.files))
    single = P.run()
    P.free()
    env_shapes = {k: {"shape": v} for k, v in P.shapes.items()}
    ref = OracleProgram(ast, env_shapes, dtype=np.float64, feeds=feeds).run()
    for k in got.files:
        assert_close(got[k], single[k], 1e-4, f"{k} dp2 vs 1 GPU")
        assert_close(got[k], ref[k], 1e-4, f"{k} dp2 vs oracle")
