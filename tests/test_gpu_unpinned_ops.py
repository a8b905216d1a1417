"""GPU parity of the ops whose semantics no reference test pins.

The reference has grammar and type rules for gelu and swish but no kernel
(tensorlang.lark:175-176, type_checker.py:274), a layer_norm VJP that no
program can reach because layer_norm is never recorded (autograd.py:649-674),
and batch_norm / instance_norm only in 2x3 test programs.  Here each is run
on the GPU at sizes of the benchmark workloads and compared with the float64
oracle on the same seeded inputs.

Tolerances (atol = rtol * max|ref| of each tensor, as everywhere):
* forward activations and normalisations: rel 1e-5;
* VJPs (the mse seed 2(y-T)/N times the activation's or layer_norm's
  derivative): rel 1e-4.
"""
import numpy as np
import pytest

from conftest import assert_close, load_backend
from oracle import OracleProgram

pytestmark = pytest.mark.gpu


def _env(P):
    return {k: {"shape": v} for k, v in P.shapes.items()}


@pytest.mark.parametrize("op", ["gelu", "swish", "relu", "sigmoid", "tanh"])
@pytest.mark.parametrize("R,C", [(300, 257), (4096, 4096)])
def test_activation_forward_and_vjp(op, R, C):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.unary_vjp(op, R, C), pr.unary_vjp_inputs(R, C, seed=R + C)
    P = tl.Program(ast, None, feeds=feeds, fetch=["y", "loss", "x_grad"])
    out = P.run()
    P.free()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    assert_close(out["y"], ref["y"], 1e-5, f"{op} y")
    assert_close(out["loss"], ref["loss"], 1e-5, f"{op} loss")
    assert_close(out["x_grad"], ref["x_grad"], 1e-4, f"{op} x_grad")


@pytest.mark.parametrize("R,C", [(7, 5), (300, 257), (1024, 4096), (16384, 4096), (64, 6000)])
def test_layer_norm_vjp(R, C):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.layer_norm_vjp(R, C), pr.layer_norm_vjp_inputs(R, C, seed=R)
    P = tl.Program(ast, None, feeds=feeds, fetch=["y", "loss", "x_grad"])
    out = P.run()
    P.free()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    assert_close(out["y"], ref["y"], 1e-5, "layer_norm y")
    assert_close(out["loss"], ref["loss"], 1e-5, "loss")
    assert_close(out["x_grad"], ref["x_grad"], 1e-4, "layer_norm x_grad")
    # the VJP of a normalisation sums to zero along each row
    rows = np.abs(out["x_grad"].astype(np.float64).sum(axis=1))
    assert rows.max() <= 1e-4 * np.abs(ref["x_grad"]).max() * np.sqrt(C)


@pytest.mark.parametrize("R,C", [(7, 5), (300, 257), (16384, 4096)])
def test_batch_norm_and_instance_norm(R, C):
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.norms(R, C), pr.norms_inputs(R, C, seed=C)
    P = tl.Program(ast, None, feeds=feeds, fetch=["bn", "inn"])
    out = P.run()
    P.free()
    ref = OracleProgram(ast, _env(P), dtype=np.float64, feeds=feeds).run()
    assert_close(out["bn"], ref["bn"], 1e-5, "batch_norm")
    assert_close(out["inn"], ref["inn"], 1e-5, "instance_norm")
