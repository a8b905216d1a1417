"""The classifier-head fusion pass (head.py) on the CPU: where it applies and
what it leaves alone.

The fused call replaces the head's forward product, softmax, the chained
cross_entropy/softmax VJP and the masked dX product, runs where the VJP ran
(after the loss seed), and is followed by the loss kernel; dW and db of the
head keep their kernels.  Its GPU results are checked bit for bit against the
unfused program in tests/test_gpu_epilogue.py.
"""
import pytest

from conftest import load_backend

tl = load_backend()
pr = tl.programs


def _plan(B=512, I=64, H=384, C=10, fetch=("loss", "W3"), program=None):
    ast = program or pr.mlp3_train(B=B, I=I, H=H, C=C, epochs=1)
    P = tl.Program(ast, None, fetch=list(fetch))
    P._fuse_all()
    return P, P._all_steps()


def _names(steps):
    return [getattr(s, "fname", type(s).__name__) for s in steps]


def test_head_of_the_training_step_is_one_call():
    P, steps = _plan()
    names = _names(steps)
    assert names.count("tl_head_ce") == 1
    assert "tl_softmax_rows" not in names and "tl_ce_softmax_backward" not in names
    head = names.index("tl_head_ce")
    # the loss seed before it, the loss kernel after it; dW3 and db3 stay
    assert any("loss_grad" in s.writes for s in steps[:head])
    assert names.index("tl_cross_entropy") > head
    masked = [s for s in steps if getattr(s, "fname", "") == "tl_gemm_masked"]
    assert not masked, "the head's masked dX product is part of the fused call"
    fused = steps[head]
    args = dict(zip(["A", "lda", "W", "ldw", "bias", "t", "onehot", "up", "div", "z", "p", "dp",
                     "dz", "dx", "lddx", "mask", "ldm", "M", "N", "K"], fused.args))
    assert args["A"] == ("ptr", "a2") and args["W"] == ("ptr", "W3") and args["mask"] == ("ptr", "a2")
    assert args["onehot"] == ("int", 1) and args["div"] == ("float", 512.0)
    assert args["z"] == ("null",)            # z is read by nothing else: not written
    assert args["dz"] == ("ptr", "z_grad") and args["dx"] == ("ptr", "h2_grad")
    assert (args["M"], args["N"], args["K"]) == (("int", 512), ("int", 10), ("int", 384))


def test_fetched_logits_are_written():
    P, steps = _plan(fetch=("loss", "z", "p", "z_grad", "h2_grad"))
    fused = next(s for s in steps if getattr(s, "fname", "") == "tl_head_ce")
    assert fused.args[9] == ("ptr", "z") and "z" in fused.writes


def test_too_small_products_keep_the_unfused_kernels():
    # M * K < 65536: tl_gemm keeps its tiled kernel there, so no fused call
    P, steps = _plan(B=64, I=32, H=64)
    names = _names(steps)
    assert "tl_head_ce" not in names and "tl_softmax_rows" in names


def test_logits_read_elsewhere_block_the_fusion():
    ast = pr.mlp3_train(B=512, I=64, H=384, C=10, epochs=1)
    body = ast[-1]["body"]
    i = next(j for j, n in enumerate(body) if n.get("name") == "p")
    body.insert(i + 1, {"type": "let", "name": "zr", "ty": None, "requires_grad": False,
                        "expr": {"type": "relu", "args": ["z"]}})
    P, steps = _plan(program=ast, fetch=("loss", "zr"))
    assert "tl_head_ce" not in _names(steps)


def test_data_parallel_divisor_is_the_global_batch():
    from tensor_lang_b200 import dp

    class _Comm:
        world, rank, handle, stream = 2, 0, None, None
    kw = dict(B=1024, I=64, H=384, C=10)
    D = dp.DataParallelProgram(pr.mlp3_train(epochs=1, **kw), None, _Comm(), device=0,
                               feeds=pr.mlp3_inputs(rows=(0, 512), **kw), fetch=["loss", "W3"])
    D.program._fuse_all()
    fused = next(s for s in D.program._all_steps() if getattr(s, "fname", "") == "tl_head_ce")
    assert fused.args[8] == ("float", 1024.0) and fused.args[17] == ("int", 512)
