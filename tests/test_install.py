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


# ---------------------------------------------------------------------------
# fused DiTBlock.forward installer (h3_fuse_patch.py:76-150), CPU side

def test_fuse_install_is_env_gated_and_falls_back_on_cpu(monkeypatch):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import fake_comfy
    mm = fake_comfy.module()
    orig = mm.DiTBlock.forward
    monkeypatch.delenv("H3_FUSE", raising=False)
    assert install.install_fuse(mm) is False and mm.DiTBlock.forward is orig
    monkeypatch.setenv("H3_FUSE", "1")
    assert install.install_fuse(mm) is True
    try:
        assert mm.DiTBlock.forward is not orig
        blk = mm.DiTBlock(64, 2, torch.device("cpu"), 1)
        x = torch.randn(10, 64).to(torch.bfloat16)
        segs = [(0, 4, 0), (4, 10, 1)]
        with torch.no_grad():
            y = mm.DiTBlock.forward(blk, x.clone(), None, segs, None)
            y_ref = orig(blk, x.clone(), None, segs, None)
        # CPU tensors are not covered: the original forward ran and gave its own result
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
        assert install.fuse_counters() == (0, 1)
    finally:
        install.uninstall_fuse()
    assert mm.DiTBlock.forward is orig


# ---------------------------------------------------------------------------
# after-import hooks for worker processes (h3_fuse_patch.py:152-183, boot/sitecustomize.py:26-44)

def _fake_tree(tmp_path):
    """comfy_kitchen/backends/cuda.py and minimax_sp/sp_forward.py under tmp_path."""
    ck = tmp_path / "comfy_kitchen" / "backends"
    ck.mkdir(parents=True)
    (tmp_path / "comfy_kitchen" / "__init__.py").write_text("")
    (ck / "__init__.py").write_text("")
    (ck / "cuda.py").write_text("def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False,"
                                " convrot_groupsize=256, input_act=None, input_act_weight=None, input_act_eps=0.0,"
                                " residual=None, residual_scale=None):\n    return 'orig'\n")
    sp_dir = tmp_path / "minimax_sp"
    sp_dir.mkdir()
    (sp_dir / "__init__.py").write_text("")
    (sp_dir / "sp_forward.py").write_text("def a2a_gather_seq_scatter_heads(t, ctx):\n    return 'orig'\n"
                                          "def a2a_scatter_seq_gather_heads(t, ctx):\n    return 'orig'\n")
    return tmp_path


def test_after_import_runs_once_after_the_module_executes(tmp_path, monkeypatch):
    (tmp_path / "h3b_fake_target.py").write_text("VALUE = 41\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    seen = []
    finder = install.after_import("h3b_fake_target", lambda m: seen.append(m.VALUE + 1))
    try:
        assert finder in sys.meta_path and not seen
        import h3b_fake_target  # noqa: F401
        assert seen == [42] and finder not in sys.meta_path
        # already imported: a new hook runs at once
        assert install.after_import("h3b_fake_target", lambda m: seen.append(0)) is None and seen == [42, 0]
    finally:
        if finder in sys.meta_path:
            sys.meta_path.remove(finder)
        sys.modules.pop("h3b_fake_target", None)


def test_boot_sitecustomize_patches_worker_imports(tmp_path):
    """A worker started with h3b/boot on PYTHONPATH and H3_LINEAR_FAST=1 / H3B_SP=1
    gets the h3b functions in place once it imports the target modules."""
    import subprocess
    tree = _fake_tree(tmp_path)
    boot = os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200", "h3b", "boot")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([boot, str(tree)]), H3_LINEAR_FAST="1", H3B_SP="1")
    code = ("import comfy_kitchen.backends.cuda as c, minimax_sp.sp_forward as s\n"
            "print(c.int8_linear.__module__, s.a2a_gather_seq_scatter_heads.__module__)\n")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.split() == ["h3b.install", "h3b.sp"], r.stdout
    # without the variables nothing is patched and h3b is not imported
    env0 = dict(os.environ, PYTHONPATH=os.pathsep.join([boot, str(tree)]))
    env0.pop("H3_LINEAR_FAST", None)
    env0.pop("H3B_SP", None)
    env0.pop("H3_FUSE", None)
    r0 = subprocess.run([sys.executable, "-c", code + "import sys; print('h3b' in sys.modules)"], env=env0,
                        capture_output=True, text=True, timeout=300)
    assert r0.returncode == 0, r0.stderr[-2000:]
    assert r0.stdout.split() == ["comfy_kitchen.backends.cuda", "minimax_sp.sp_forward", "False"], r0.stdout
