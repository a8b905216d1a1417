"""The ``semantics="numpy"`` switch, on the CPU: the oracle's two textbook
rules against plain NumPy, the lowering the switch selects, and that the
default stays reference-literal.

Reference rules replaced by the switch:
* a 2-D op 1-D broadcast reads ``B[i]`` whenever the row counts match
  (kernel_generator.py:303-348), so a square ``x[n,n] * s[n]`` scales rows;
  NumPy scales columns (``B[j]``);
* cross_entropy's VJP ``(p - t) / B`` (autograd.py:691-704) is taken as the
  gradient of p and the softmax VJP (autograd.py:563-580) is chained after
  it; the textbook gradient of the logits is ``(p - t) / B`` itself.

The GPU side of the switch is checked against the oracle in
test_gpu_configs.py."""
import numpy as np
import pytest

from conftest import load_backend
from oracle import OracleProgram

load_backend()  # registers the package as tensor_lang_b200


def _env(P):
    return {k: {"shape": v} for k, v in P.shapes.items()}


def _chain(N=6, seed=0):
    tl = load_backend()
    pr = tl.programs
    return tl, pr.fused_chain(N), pr.fused_chain_inputs(N, seed=seed)


def _gelu(v):
    from scipy.special import erf
    return 0.5 * v * (1.0 + erf(v / np.sqrt(2.0)))


def test_oracle_square_broadcast_rule():
    tl, ast, feeds = _chain()
    env = {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}
    x, s, b = (feeds[k].astype(np.float64) for k in ("x", "s", "b"))
    lit = OracleProgram(ast, env, feeds=feeds).run()
    num = OracleProgram(ast, env, feeds=feeds, semantics="numpy").run()
    np.testing.assert_allclose(lit["y"], _gelu(x * s[:, None] + b), rtol=1e-12)   # B[i]
    np.testing.assert_allclose(num["y"], _gelu(x * s[None, :] + b), rtol=1e-12)   # B[j]
    assert not np.allclose(lit["y"], num["y"])


def test_oracle_textbook_softmax_cross_entropy_gradient():
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.mlp2_step(), pr.mlp2_inputs(seed=1)
    env = {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}
    lit = OracleProgram(ast, env, feeds=feeds).run()
    num = OracleProgram(ast, env, feeds=feeds, semantics="numpy").run()
    p, t = num["p"], feeds["t"].astype(np.float64)
    B = p.shape[0]
    np.testing.assert_allclose(num["z_grad"], (p - t) / B, rtol=1e-12, atol=0)
    assert not np.any(num["p_grad"])  # the textbook path gives p nothing
    # the reference chains the softmax VJP after (p - t) / B
    g = (p - t) / B
    np.testing.assert_allclose(lit["z_grad"], p * (g - np.sum(g * p, axis=1, keepdims=True)),
                               rtol=1e-10, atol=1e-15)
    assert not np.allclose(lit["z_grad"], num["z_grad"])


def test_generator_square_broadcast_kernel():
    from tensor_lang_b200.kernel_generator import KernelGenerator
    ref, npy = KernelGenerator(), KernelGenerator(numpy_broadcast=True)
    args = ("mult", "mult", "y", "x", "s")
    assert ref.binary_broadcast(*args, (8, 8), (8,), (8, 8))[1][0] == "mult_broadcast_rows"
    assert npy.binary_broadcast(*args, (8, 8), (8,), (8, 8))[1][0] == "mult_broadcast"
    # NumPy has no rule for [8,4] op [8]: the per-row rule stays
    assert npy.binary_broadcast(*args, (8, 4), (8,), (8, 4))[1][0] == "mult_broadcast_rows"
    assert npy.binary_broadcast(*args, (4, 8), (8,), (4, 8))[1][0] == "mult_broadcast"


def _bw_fnames(P):
    return [getattr(s, "fname", None) for s in P.phase_bw]


def test_program_backward_follows_the_switch():
    tl = load_backend()
    pr = tl.programs
    ast, feeds = pr.mlp2_step(), pr.mlp2_inputs(seed=0)
    lit = tl.Program(ast, None, feeds=feeds)
    num = tl.Program(ast, None, feeds=feeds, semantics="numpy")
    assert "tl_ce_softmax_backward" in _bw_fnames(lit)
    assert "tl_ce_softmax_backward" not in _bw_fnames(num)
    with pytest.raises(ValueError):
        tl.Program(ast, None, feeds=feeds, semantics="torch")
