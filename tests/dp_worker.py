"""One rank of the data-parallel training check (launched by test_gpu_dp.py).

Trains the small 3-layer MLP for a few epochs with the batch split over the
ranks and writes the final parameters (rank 0) to the .npz given as argv[1].
"""
import os
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
from __graft_entry__ import load_package  # noqa: E402


def margin_biases(feeds: dict) -> dict:
    """Hidden-layer biases of +-0.5 (alternating units) instead of zero.

    With zero biases some pre-activations of the 512 x 128 layers sit within
    float32 rounding of 0, where a float32 run and the float64 oracle may take
    different relu branches; one flipped unit moves a whole gradient entry in
    or out of the bias gradient's column sum.  A 0.5 offset keeps every
    pre-activation about 3 standard deviations from the branch point while
    half the units stay active and half inactive."""
    out = dict(feeds)
    for name in ("b1", "b2"):
        n = out[name].shape[0]
        out[name] = np.where(np.arange(n) % 2 == 0, 0.5, -0.5).astype(np.float32)
    return out


def main(out_path: str, epochs: int = 4):
    tl = load_package()
    from tensor_lang_b200 import dp
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    kw = dict(B=512, I=64, H=128, C=10)
    B = kw["B"]
    b = B // world
    tl.runtime.Device.get(local)
    port = int(os.environ["MASTER_PORT"]) + 17
    rdv = dp.Rendezvous(rank, world, os.environ.get("MASTER_ADDR", "127.0.0.1"), port, timeout=60)
    comm = dp.Communicator(rdv, timeout_ms=60000)
    feeds = margin_biases(tl.programs.mlp3_inputs(seed=5, rows=(rank * b, (rank + 1) * b), **kw))
    ast = tl.programs.mlp3_train(epochs=epochs, **kw)
    D = dp.DataParallelProgram(ast, None, comm, device=local, feeds=feeds,
                               fetch=["W1", "b1", "W2", "b2", "W3", "b3"])
    out = D.run()
    comm.wait(D.program.stream)
    if rank == 0:
        np.savez(out_path, **out)
    D.program.free()
    comm.destroy()
    rdv.close()


if __name__ == "__main__":
    main(sys.argv[1])
