"""The installed fused DiTBlock.forward on the GPU (h3_fuse_patch.py:76-150).

install_fuse replaces DiTBlock.forward of a stand-in for ComfyUI's block
(tests/fake_comfy.py: the attributes the fused forward reads and an eager
forward in the reference's documented order).  On CUDA bf16 input the fused
forward runs h3b's norm_mod / gate_norm_mod_ / gate_ kernels around the
block's own attention and mlp and must give the eager forward's bytes; calls it
does not cover (grad enabled, segments that leave a gap) go to the original.
"""
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")
from h3b import install  # noqa: E402

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import fake_comfy  # noqa: E402

DEV = torch.device("cuda", 0)


def test_installed_fused_forward_matches_the_original(monkeypatch):
    monkeypatch.setenv("H3_FUSE", "1")
    mm = fake_comfy.module()
    orig = mm.DiTBlock.forward
    assert install.install_fuse(mm)
    try:
        D, S = 5120, 3000
        blk = mm.DiTBlock(D, 3, DEV, 7)
        x = torch.randn(S, D, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).to(DEV)
        rows = torch.randint(0, 3, (500,), generator=torch.Generator().manual_seed(9))
        segs = [(1000, 1500, rows), (0, 1000, 0), (1500, S, 2)]  # unsorted, one per-row tensor segment
        with torch.no_grad():
            for _ in range(2):  # the second call reuses the cached row index
                y = mm.DiTBlock.forward(blk, x.clone(), None, segs, None)
                y_ref = orig(blk, x.clone(), None, segs, None)
                torch.cuda.synchronize()
                assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
        assert install.fuse_counters() == (2, 0)
        # not covered: grad enabled, and segments with a gap -> the original forward
        y_g = mm.DiTBlock.forward(blk, x.clone(), None, segs, None)
        with torch.no_grad():
            y_gap = mm.DiTBlock.forward(blk, x.clone(), None, [(0, 1000, 0), (1200, S, 1)], None)
        assert install.fuse_counters() == (2, 2)
        assert y_g.shape == x.shape and y_gap.shape == x.shape
        assert h3b.status() == 0
    finally:
        install.uninstall_fuse()
    assert mm.DiTBlock.forward is orig
