"""The arithmetic of the tensor-core operand schemes, restated in NumPy on
the CPU: how each scheme splits an fp32 operand, which products it keeps,
and the error that leaves against an fp64 product.  Products and sums are
exact here, so the figures are the split error alone: 1.3-1.5e-6 for
TF32+bf16 and 4.6-5.1e-6 for BF16X3 (max error rel to max|C|, N(0,1) data,
K = 256 and 4096).  The GPU measures 1.3-2.0e-6 and 4.2-4.6e-6: the split,
not its fp32 accumulation, sets the error.

Scheme definitions (csrc/gemm_tc.cu):
* TF32+bf16: hi = x with the low 13 mantissa bits dropped (the tensor core's
  reading of an fp32 operand as TF32), lo = x - hi (exact); products
  hi*hi + bf16(x)*bf16(lo_b) + bf16(lo_a)*bf16(x_b);
* BF16X3: a0 = bf16(x) (round to nearest even), a1 = bf16(x - a0); products
  a0*b0 + a0*b1 + a1*b0.
"""
import numpy as np
import pytest


def bf16(x):
    """Round float32 to bfloat16 (nearest, ties to even), returned as float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


def trunc_tf32(x):
    u = np.asarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)
    return u.view(np.float32)


def tf32_bf16_product(A, B):
    f = np.float64
    ha, hb = trunc_tf32(A), trunc_tf32(B)
    la, lb = A - ha, B - hb  # exact in fp32
    return (ha.astype(f) @ hb.astype(f) + bf16(A).astype(f) @ bf16(lb).astype(f)
            + bf16(la).astype(f) @ bf16(B).astype(f))


def bf16x3_product(A, B):
    f = np.float64
    a0, b0 = bf16(A), bf16(B)
    a1, b1 = bf16(A - a0), bf16(B - b0)
    return a0.astype(f) @ b0.astype(f) + a0.astype(f) @ b1.astype(f) + a1.astype(f) @ b0.astype(f)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -9, -2.5, 3.0e38],
                 np.float32)
    got = bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa -> 1
    np.testing.assert_array_equal(got[:2], [1.0, 1.0])
    assert got[2] == np.float32(1.0 + 2 ** -6)     # tie -> even (1 + 4 * 2^-8)
    assert got[3] == 1.0 and got[4] == -2.5
    assert np.isfinite(got[5])


def test_split_parts_are_exact_and_small():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(1 << 16).astype(np.float32)
    hi = trunc_tf32(x)
    assert np.all(np.abs(x - hi) <= np.abs(x) * 2.0 ** -10)
    a0 = bf16(x)
    r = (x.astype(np.float64) - a0.astype(np.float64))
    assert np.array_equal(r.astype(np.float32).astype(np.float64), r)  # x - a0 exact in fp32
    assert np.all(np.abs(r) <= np.abs(x) * 2.0 ** -8)
    a1 = bf16(x - a0)
    resid = x.astype(np.float64) - a0 - a1
    assert np.all(np.abs(resid) <= np.abs(x) * 2.0 ** -16)


@pytest.mark.parametrize("K", [256, 4096])
def test_split_errors_against_fp64(K):
    rng = np.random.default_rng(K)
    A = rng.standard_normal((64, K)).astype(np.float32)
    B = rng.standard_normal((K, 96)).astype(np.float32)
    ref = A.astype(np.float64) @ B.astype(np.float64)
    scale = np.abs(ref).max()
    e_tb = np.abs(tf32_bf16_product(A, B) - ref).max() / scale
    e_x3 = np.abs(bf16x3_product(A, B) - ref).max() / scale
    # both far inside the GEMM tolerance (1e-4); BF16X3 drops a1*b1 and
    # rounds a1, b1 (~2^-16 per product), TF32+bf16 rounds the lows (~2^-19)
    assert e_tb < 3e-6 and e_x3 < 1e-5
    assert e_tb < e_x3
