"""The installers put h3b behind the reference's hooks and take it out again
(CPU only: fake hook targets, no device work).  Mirrors the reference's
install()/uninstall() of h3_linear_fast_patch.py:43-124: env-gated, ineligible
calls go to the original function, uninstall restores it."""
import os
import sys
import types

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))

from h3b import install, sp  # noqa: E402


def _fake_ckc():
    calls = []

    def orig(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256,
             input_act=None, input_act_weight=None, input_act_eps=0.0, residual=None, residual_scale=None):
        calls.append((tuple(x.shape), convrot, input_act, residual is not None))
        return "orig"

    return types.SimpleNamespace(int8_linear=orig), calls, orig


def test_linear_install_is_env_gated(monkeypatch):
    ckc, _, orig = _fake_ckc()
    monkeypatch.delenv("H3_LINEAR_FAST", raising=False)
    assert install.install_linear(ckc) is False
    assert ckc.int8_linear is orig


def test_linear_install_routes_and_uninstalls(monkeypatch):
    ckc, calls, orig = _fake_ckc()
    monkeypatch.setenv("H3_LINEAR_FAST", "1")
    assert install.install_linear(ckc) is True
    try:
        assert ckc.int8_linear is not orig
        x = torch.zeros(4, 256, dtype=torch.bfloat16)
        w = torch.zeros(8, 256, dtype=torch.int8)
        assert ckc.int8_linear(x, w, torch.ones(8)) == "orig"  # CPU tensor: the original runs
        assert ckc.int8_linear(x, w, torch.ones(8), residual=torch.zeros(4, 8)) == "orig"
        assert len(calls) == 2 and calls[1][3] is True
        assert install.linear_counters() == (0, 2)
    finally:
        install.uninstall_linear()
    assert ckc.int8_linear is orig


def test_sp_install_replaces_and_restores():
    def a(t, ctx):
        return "ref-a"

    def b(t, ctx):
        return "ref-b"

    mod = types.SimpleNamespace(a2a_gather_seq_scatter_heads=a, a2a_scatter_seq_gather_heads=b)
    install.install_sp(mod)
    try:
        assert mod.a2a_gather_seq_scatter_heads is sp.a2a_gather_seq_scatter_heads
        assert mod.a2a_scatter_seq_gather_heads is sp.a2a_scatter_seq_gather_heads
    finally:
        install.uninstall_sp()
    assert mod.a2a_gather_seq_scatter_heads is a and mod.a2a_scatter_seq_gather_heads is b


def test_reference_context_selects_nccl():
    """A context without exchange / peer attributes (the reference's SPContext)
    takes the NCCL back end."""
    ref_ctx = types.SimpleNamespace(rank=0, world=2, group=None, seq_len=10, splits=[5, 5], start=0, stop=5,
                                    local=5)
    assert sp._p2p(ref_ctx) is None
    with pytest.raises(TypeError):  # NCCL path: the pack kernel needs a CUDA tensor
        sp.a2a_gather_seq_scatter_heads(torch.zeros(5, 4, 8, dtype=torch.bfloat16), ref_ctx)
