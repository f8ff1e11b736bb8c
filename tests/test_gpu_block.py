"""The whole fused DiT block on h3b kernels vs the reference's eager PyTorch path, on one GPU.

Both sides run the same block (h3b.model.block_forward vs
oracle.torch_path.block_forward) on identical weights and inputs, with the same
SDPA call in the middle.  Every h3b kernel is bit-exact against the eager op
it replaces, so the block output must be bit-exact too.
"""
import pytest
import torch

from gpu_util import randn_bf16

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")
from h3b import model as hm  # noqa: E402
from oracle import torch_path as tp  # noqa: E402

DEV = torch.device("cuda", 0)


def _run(cfg, S, R, seed, text_len=0):
    p = hm.make_params(cfg, 0, seed, DEV, R=R)
    x = randn_bf16((S, cfg.dim), seed).to(DEV)
    ridx = torch.zeros(S, dtype=torch.int32, device=DEV)
    ridx[S // 3:] = R - 1
    text = randn_bf16((text_len, cfg.dim), seed + 1).to(DEV) if text_len else None
    y = hm.block_forward(cfg, p, x.clone(), ridx, None, text)
    y_ref = tp.block_forward(cfg, p, x.clone(), ridx, None, text)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    n_bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
    assert n_bad == 0, f"{n_bad} of {y.numel()} elements differ from the eager reference block"
    assert h3b.status() == 0


def test_block_small():
    _run(hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816), S=1000, R=2, seed=3)


def test_block_full_width_one_frame():
    _run(hm.DiTConfig(), S=4128, R=2, seed=4)


def test_block_with_text_cross_attention():
    _run(hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816, text_len=64), S=777, R=1, seed=5, text_len=64)


def test_block_fused_producers_path():
    """The block with the fused norm->quant and GELU->quant producers is bit-exact too."""
    cfg = hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816)
    p = hm.make_params(cfg, 0, 9, DEV, R=2)
    x = randn_bf16((900, cfg.dim), 9).to(DEV)
    ridx = torch.zeros(900, dtype=torch.int32, device=DEV)
    ridx[450:] = 1
    y = hm.block_forward(cfg, p, x.clone(), ridx, fused_producers=True)
    y2 = hm.block_forward(cfg, p, x.clone(), ridx, fused_producers=False)
    y_ref = tp.block_forward(cfg, p, x.clone(), ridx)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert torch.equal(y2.view(torch.int16), y_ref.view(torch.int16))


def test_host_pipeline_matches_serial_steps():
    """HostPipeline (copies on side streams, three slots in flight) returns, for
    every submitted step, the same bytes as a plain copy-in / forward / copy-out."""
    cfg = hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816, n_blocks=2)
    S = 1500
    dit = hm.SynthDiT(cfg, DEV, seed=9)
    ridx = torch.zeros(S, dtype=torch.int32, device=DEV)
    xs = [randn_bf16((S, cfg.dim), 40 + k).pin_memory() for k in range(5)]
    outs = [torch.empty(S, cfg.dim, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    pipe = hm.HostPipeline(dit, S, ridx, depth=3)
    for k in range(5):
        pipe.submit(xs[k], outs[k])
    pipe.flush()
    torch.cuda.synchronize()
    for k in range(5):
        ref = dit.forward(xs[k].to(DEV), ridx).cpu()
        assert torch.equal(outs[k].view(torch.int16), ref.view(torch.int16)), f"step {k} differs"


def test_host_pipeline_with_per_step_conditioning():
    """Per-step adaLN conditioning through HostPipeline's input copy stream
    (cond_host -> the slot's device copies -> `before`): each step's output
    equals a serial forward with that step's conditioning loaded first."""
    cfg = hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816, n_blocks=2)
    S = 1200
    dit = hm.SynthDiT(cfg, DEV, seed=10)
    ridx = torch.zeros(S, dtype=torch.int32, device=DEV)
    xs = [randn_bf16((S, cfg.dim), 60 + k).pin_memory() for k in range(4)]
    es = [[randn_bf16(tuple(p.e.shape), 70 + 10 * k + b, 0.1).pin_memory() for b, p in enumerate(dit.params)]
          for k in range(4)]
    outs = [torch.empty(S, cfg.dim, dtype=torch.bfloat16).pin_memory() for _ in range(4)]

    def load(cond):
        for p, e in zip(dit.params, cond):
            p.e.copy_(e, non_blocking=True)
            p.tables = h3b.modulation_tables(*(p.e[:, i] for i in range(6)))
    pipe = hm.HostPipeline(dit, S, ridx, depth=3)
    for k in range(4):
        pipe.submit(xs[k], outs[k], before=load, cond_host=es[k])
    pipe.flush()
    torch.cuda.synchronize()
    for k in range(4):
        load([e.to(DEV) for e in es[k]])
        ref = dit.forward(xs[k].to(DEV), ridx).cpu()
        assert torch.equal(outs[k].view(torch.int16), ref.view(torch.int16)), f"step {k} differs"


def test_block_with_qk_norm():
    """The block with the per-head q/k RMSNorm (rms_norm kernel on the unfused path)."""
    _run(hm.DiTConfig(dim=1024, heads=8, head_dim=128, ffn=2816, qk_norm=True), S=1000, R=2, seed=6)


def test_step_two_blocks_with_text_full_width():
    """Configuration 4's structure at full width: two blocks of the step model
    (D=5120, 40 heads, FFN 13824, 512 text tokens for the cross-attention), one
    latent frame of rows, bit-exact against the eager block loop
    (sp_forward.py:556-561 runs the blocks in order the same way)."""
    cfg = hm.DiTConfig(n_blocks=2, text_len=512)
    S = 4128
    dit = hm.SynthDiT(cfg, DEV, seed=21)
    x = randn_bf16((S, cfg.dim), 21).to(DEV)
    text = randn_bf16((512, cfg.dim), 22).to(DEV)
    ridx = torch.zeros(S, dtype=torch.int32, device=DEV)
    y = dit.forward(x.clone(), ridx, None, text)
    y_ref = x.clone()
    for p in dit.params:
        y_ref = tp.block_forward(cfg, p, y_ref, ridx, None, text)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    n_bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
    assert n_bad == 0, f"{n_bad} of {y.numel()} elements differ after 2 blocks"
    assert h3b.status() == 0


def test_block_full_size_s128000():
    """Configuration 3 at its full size: one block over S=128000 tokens on one
    GPU (the benchmark's block) against the eager block, bit for bit."""
    cfg = hm.DiTConfig()
    S = 128000
    p = hm.make_params(cfg, 0, 1, DEV)
    x = randn_bf16((S, cfg.dim), 31).to(DEV)
    ridx = torch.zeros(S, dtype=torch.int32, device=DEV)
    y = hm.block_forward(cfg, p, x.clone(), ridx)
    y_ref = tp.block_forward(cfg, p, x, ridx)  # in place on x: the input is not needed again
    torch.cuda.synchronize()
    n_bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
    assert n_bad == 0, f"{n_bad} of {y.numel()} elements differ at S=128000"
    assert torch.isfinite(y.float()).all()
    assert h3b.status() == 0
    del y, y_ref, x
    torch.cuda.empty_cache()
