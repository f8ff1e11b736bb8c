"""Host-side routing of the patched int8_linear (CPU only, no device work).

The reference's fast path accepts only some calls and sends the rest back to
comfy-kitchen (h3_linear_fast_patch.py:64-80); h3b.int8_linear signals the calls
it does not cover with NotImplementedError before touching any tensor on a
device, so an installer can do the same fallback.  Covered calls that are given
CPU tensors raise TypeError (there is no CPU path)."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))

import h3b  # noqa: E402

X = torch.zeros(4, 256, dtype=torch.bfloat16)
W = torch.zeros(8, 256, dtype=torch.int8)
WS = torch.ones(8)


@pytest.mark.parametrize("kw", [dict(residual=torch.zeros(4, 8)), dict(input_act="gelu"),
                                dict(input_act="swiglu", convrot=False),
                                dict(input_act="swiglu", convrot=True, input_act_weight=torch.ones(1)),
                                dict(convrot=True, convrot_groupsize=128), dict(out_dtype=torch.float16)])
def test_uncovered_variants_raise_not_implemented(kw):
    with pytest.raises(NotImplementedError):
        h3b.int8_linear(X, W, WS, **kw)


@pytest.mark.parametrize("kw", [dict(), dict(convrot=True, convrot_groupsize=256), dict(bias=torch.zeros(8).bfloat16())])
def test_covered_variants_need_cuda_tensors(kw):
    with pytest.raises(TypeError):
        h3b.int8_linear(X, W, WS, **kw)


def test_swiglu_input_is_twice_as_wide():
    with pytest.raises(TypeError):  # covered (ConvRot + SwiGLU), CPU tensor
        h3b.int8_linear(torch.zeros(4, 512, dtype=torch.bfloat16), W, WS, convrot=True, input_act="swiglu")
