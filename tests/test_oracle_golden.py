"""Pin the CPU oracle to the reference's own kernels (CPU only).

The fixtures in tests/golden/ were produced by the reference's Triton kernels
run under Triton's CPU interpreter (tests/golden/make_golden.py).  In the
interpreter's arithmetic mode (truncating bf16 cast, no FMA contraction,
rsqrt = 1/sqrt) the oracle must reproduce them bit for bit; the product mode
differs from that mode only in those three switches, which the remaining tests
check against independent float64 / int64 restatements.
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


@pytest.mark.parametrize("name", ["gemm_small", "gemm_bigacc"])
def test_gemm_matches_reference_kernel(name):
    d = load(name)
    y = oracle.int8_mm_scaled(d["xq"], d["w"], d["xs"], d["ws"], final_round=oracle.TRUNC)
    np.testing.assert_array_equal(y, d["out"])


@pytest.mark.parametrize("name", ["norm_d1024", "norm_d5120_adv", "norm_d1000_tail"])
def test_norm_kernels_match_reference_kernels(name):
    d = load(name)
    mode = dict(fma=False, rsqrt_mode=oracle.RSQRT_RECIP, final_round=oracle.TRUNC)
    eps = float(d["eps"])
    # s1 = bf16(1.0 + scale): the reference evaluates it with PyTorch (RNE), h3_fuse_patch.py:113,116
    np.testing.assert_array_equal(oracle.one_plus(d["scale"], oracle.RNE), d["s1"])
    h, _ = oracle.norm_mod(d["x"], d["w"], eps, d["ridx"], d["s1"], d["shift"], **mode)
    np.testing.assert_array_equal(h, d["h_norm_mod"])
    xn, h2, _ = oracle.gate_norm_mod_(d["x"], d["o"], d["gate"], d["w"], eps, d["ridx"], d["s1"], d["shift"], **mode)
    np.testing.assert_array_equal(xn, d["x_gate_norm_mod"])
    np.testing.assert_array_equal(h2, d["h_gate_norm_mod"])
    xg = oracle.gate_(d["x"], d["o"], d["gate"], d["ridx"], final_round=oracle.TRUNC)
    np.testing.assert_array_equal(xg, d["x_gate"])


def test_product_mode_differs_only_in_final_rounding():
    """Product-mode GEMM == interpreter-mode GEMM except for the last cast."""
    d = load("gemm_bigacc")
    y, acc = oracle.int8_mm_scaled(d["xq"], d["w"], d["xs"], d["ws"], want_acc=True)
    exact = d["xq"].astype(np.int64) @ d["w"].astype(np.int64).T
    np.testing.assert_array_equal(acc.astype(np.int64), exact)
    assert np.abs(exact).max() > 2 ** 24  # float(acc) rounds in this case
    f = (acc.astype(np.float32) * d["xs"][:, None]) * d["ws"][None, :]
    np.testing.assert_array_equal(y, oracle.f32_to_bf16(f, oracle.RNE))
    np.testing.assert_array_equal(oracle.f32_to_bf16(f, oracle.TRUNC), d["out"])


def test_f32_to_bf16_matches_torch():
    g = torch.Generator().manual_seed(5)
    v = torch.randn(100000, generator=g) * torch.logspace(-30, 30, 100000)
    v[:5] = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 1.0 + 2 ** -8])
    ours = oracle.f32_to_bf16(v.numpy())
    ref = v.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
