"""CPU checks of the ConvRot restatement (oracle.rotate_groups / quant_rowwise_convrot).

The rotation is the normalised Walsh-Hadamard transform per group of columns,
computed as the fast transform in binary32.  Checked against float64 matrix
products with scipy's Sylvester-ordered Hadamard matrix: exact for small
integer inputs (every partial sum is exact in binary32), within binary32
rounding otherwise; rotating twice gives the input back (H is symmetric and
orthogonal after normalisation).
"""
import numpy as np
import pytest
import scipy.linalg as sl
import torch

import oracle


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("group", [64, 256])
def test_rotation_is_normalised_hadamard(group):
    g = torch.Generator().manual_seed(group)
    H = sl.hadamard(group).astype(np.float64) / np.sqrt(group)
    # small integers: every partial sum is exact in binary32, so the result is exact
    xi = torch.randint(-8, 9, (6, 4 * group), generator=g).to(torch.bfloat16)
    y = oracle.rotate_groups(_bits(xi), group)
    ref = np.concatenate([xi.double().numpy()[:, i:i + group] @ H for i in range(0, 4 * group, group)], axis=1)
    np.testing.assert_array_equal(y, ref.astype(np.float32))
    # N(0,1): within binary32 rounding of the exact transform
    x = torch.randn(6, 4 * group, generator=g).to(torch.bfloat16)
    y = oracle.rotate_groups(_bits(x), group)
    ref = np.concatenate([x.double().numpy()[:, i:i + group] @ H for i in range(0, 4 * group, group)], axis=1)
    assert np.abs(y - ref).max() <= 4 * np.finfo(np.float32).eps * np.abs(x.double().numpy()).max()


def test_rotation_wide_range_within_rounding_and_involutive():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(4, 512, generator=g) * torch.logspace(-6, 6, 512)).to(torch.bfloat16)
    y = oracle.rotate_groups(_bits(x), 256)
    H = sl.hadamard(256).astype(np.float64) / 16
    xd = x.double().numpy()
    ref = np.concatenate([xd[:, :256] @ H, xd[:, 256:] @ H], axis=1)
    scale = np.abs(xd).max()
    assert np.abs(y - ref).max() <= 8 * np.finfo(np.float32).eps * scale
    back = np.concatenate([y[:, :256].astype(np.float64) @ H, y[:, 256:].astype(np.float64) @ H], axis=1)
    assert np.abs(back - xd).max() <= 16 * np.finfo(np.float32).eps * scale


def test_convrot_quant_is_quant_of_rotated_rows():
    """Codes and scales equal the plain absmax quantisation of the rotated fp32 rows."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(16, 1024, generator=g).to(torch.bfloat16)
    x[0] = 0
    q, s = oracle.quant_rowwise_convrot(_bits(x), 256)
    y = oracle.rotate_groups(_bits(x), 256)
    amax = np.abs(y).max(axis=1)
    s_ref = (amax / np.float32(127)).astype(np.float32)
    np.testing.assert_array_equal(s, s_ref)
    assert (q[0] == 0).all() and s[0] == 0
    ref = np.clip(np.rint(y[1:] / s_ref[1:, None]), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(q[1:], ref)
