"""The eager PyTorch restatement (oracle/torch_path.py) agrees with the C oracle on CPU."""
import numpy as np
import torch

import oracle
from oracle import torch_path as tp


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_quant_matches_oracle():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(512, 5120, generator=g).to(torch.bfloat16)
    x[3] = 0
    q, s = tp.quant_rowwise(x)
    qo, so = oracle.quant_rowwise(_bits(x))
    np.testing.assert_array_equal(q.numpy(), qo)
    np.testing.assert_array_equal(s.reshape(-1).numpy(), so)


def test_linear_matches_oracle():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(64, 1024, generator=g).to(torch.bfloat16)
    w = torch.randint(-127, 128, (256, 1024), generator=g, dtype=torch.int8)
    ws = torch.rand(256, generator=g) * 1e-3
    b = (torch.randn(256, generator=g) * 0.02).to(torch.bfloat16)
    y = tp.linear(x, w, ws, b)
    qo, so = oracle.quant_rowwise(_bits(x))
    yo = oracle.int8_mm_scaled(qo, w.numpy(), so, ws.numpy(), bias=_bits(b))
    np.testing.assert_array_equal(_bits(y), yo)


def test_gate_matches_oracle():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(32, 512, generator=g).to(torch.bfloat16)
    o = torch.randn(32, 512, generator=g).to(torch.bfloat16)
    gt = (0.1 * torch.randn(2, 512, generator=g)).to(torch.bfloat16)
    ridx = torch.randint(0, 2, (32,), generator=g, dtype=torch.int32)
    ref = oracle.gate_(_bits(x), _bits(o), _bits(gt), ridx.numpy())
    np.testing.assert_array_equal(_bits(tp.gate_(x.clone(), o, gt, ridx)), ref)
