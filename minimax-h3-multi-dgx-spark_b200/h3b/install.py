"""Installers that put h3b behind the reference's own hooks, as the reference does.

  install_linear(ckc)   comfyui_nodes/h3-linear-fast/h3_linear_fast_patch.py:43-117
      env-gated (H3_LINEAR_FAST=1): replaces ckc.int8_linear (the module
      comfy_kitchen.backends.cuda unless another object is given) with a
      function that runs h3b.int8_linear for the calls it covers and calls the
      original for the rest -- CPU tensors, variants h3b does not cover
      (NotImplementedError) -- and, after a library error, for every later call
      (the reference disables its fast path the same way, :100-106).
  uninstall_linear()    :119-124, puts the original back.
  install_sp(mod)       replaces mod.a2a_gather_seq_scatter_heads and
      mod.a2a_scatter_seq_gather_heads (minimax_sp.sp_forward, sp_forward.py:179-198)
      with h3b's; they accept the reference's SPContext (NCCL back end) or an
      h3b.SPContext.  uninstall_sp() restores them.
  install_fuse(mm)      comfyui_nodes/h3-fuse-graph/h3_fuse_patch.py:76-150
      env-gated (H3_FUSE=1): replaces mm.DiTBlock.forward (the module
      comfy.ldm.minimax.model unless another object is given) with the fused
      forward -- norm_mod, attention, gate_norm_mod_, mlp, gate_ on h3b's
      kernels, same order and values -- and calls the original forward for
      the calls it does not cover (not bf16 / 2-D / contiguous / CUDA, grad
      enabled, mod_segments that do not tile the rows, a norm weight that is
      not bf16).  uninstall_fuse() restores it.
  fuse_kernels()        the module to import as `fk` in place of h3_fuse_kernels
      (h3_fuse_patch.py:81): h3b.fuse, with the same norm_mod / gate_norm_mod_ /
      gate_ signatures.
  after_import(match, fn)   h3_fuse_patch.py:152-183: a sys.meta_path finder that
      calls fn(module) right after the first module whose name matches is
      executed (worker processes import ComfyUI's modules without loading the
      custom nodes, so the hooks wait for the import).
  install_worker_hooks()    boot/sitecustomize.py:26-44 and
      boot/h3_fuse_launch.py:20-32: registers those after-import hooks from the
      environment (H3_LINEAR_FAST, H3_FUSE, H3B_SP); h3b/boot/sitecustomize.py
      calls it at interpreter start when its folder is on PYTHONPATH.
"""
import functools
import importlib.abc
import importlib.machinery
import logging
import os
import sys

import torch

from . import fuse, linear, sp
from ._lib import H3BError

log = logging.getLogger("h3b")
_linear_state = {"target": None, "orig": None, "disabled": False, "fast_calls": 0, "fallback_calls": 0}
_sp_state = {"target": None, "orig": None}
_fuse_state = {"target": None, "orig": None, "fused": 0, "fallback": 0, "ridx_key": None, "ridx": None}


def install_linear(ckc=None):
    """Patch ckc.int8_linear when H3_LINEAR_FAST=1; returns whether it patched."""
    if _linear_state["target"] is not None:
        return True
    if os.environ.get("H3_LINEAR_FAST", "0") != "1":
        return False
    if ckc is None:
        from comfy_kitchen.backends import cuda as ckc
    orig = ckc.int8_linear
    st = _linear_state

    def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256,
                    input_act=None, input_act_weight=None, input_act_eps=0.0, residual=None, residual_scale=None):
        if not st["disabled"] and x.is_cuda:
            try:
                y = linear.int8_linear(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize,
                                       input_act, input_act_weight, input_act_eps, residual, residual_scale)
                st["fast_calls"] += 1
                return y
            except NotImplementedError:
                pass
            except H3BError as e:
                st["disabled"] = True
                log.warning("h3b int8_linear failed, using the original from now on: %s", e)
        st["fallback_calls"] += 1
        return orig(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize, input_act,
                    input_act_weight, input_act_eps, residual, residual_scale)

    ckc.int8_linear = int8_linear
    st.update(target=ckc, orig=orig, disabled=False, fast_calls=0, fallback_calls=0)
    return True


def uninstall_linear():
    st = _linear_state
    if st["target"] is not None:
        st["target"].int8_linear = st["orig"]
        st.update(target=None, orig=None)


def linear_counters():
    """(calls run by h3b, calls sent to the original) since install_linear."""
    return _linear_state["fast_calls"], _linear_state["fallback_calls"]


_SP_NAMES = ("a2a_gather_seq_scatter_heads", "a2a_scatter_seq_gather_heads")


def install_sp(mod):
    """Replace the exchange functions of the module `mod` (minimax_sp.sp_forward)."""
    if _sp_state["target"] is not None:
        return True
    _sp_state.update(target=mod, orig={n: getattr(mod, n) for n in _SP_NAMES})
    for n in _SP_NAMES:
        setattr(mod, n, getattr(sp, n))
    return True


def uninstall_sp():
    if _sp_state["target"] is not None:
        for n, f in _sp_state["orig"].items():
            setattr(_sp_state["target"], n, f)
        _sp_state.update(target=None, orig=None)


def fuse_kernels():
    return fuse


# ---------------------------------------------------------------------------
# fused DiTBlock.forward (h3_fuse_patch.py:76-150)

class _PlainWeight:
    def __init__(self, w):
        self.w = w

    def __enter__(self):
        return self.w, None

    def __exit__(self, *exc):
        return False


def _norm_weight(norm, x):
    """The norm's weight the way ComfyUI's RMSNorm.forward takes it
    (h3_fuse_patch.py:59-64): through cast_weight when the layer casts or
    patches its weights, else the parameter itself; a context giving (w, b)."""
    if getattr(norm, "comfy_cast_weights", False) or len(getattr(norm, "weight_function", ()) or ()) > 0 \
            or len(getattr(norm, "bias_function", ()) or ()) > 0:
        return norm.cast_weight(x)
    return _PlainWeight(norm.weight)


def _cached_row_index(mod_segments, s, device):
    """row_index, remembered for the last (mod_segments object, s, device): the
    blocks of one forward share the list (h3_fuse_patch.py:35-37,55)."""
    st = _fuse_state
    key = st["ridx_key"]
    if key is not None and key[0] is mod_segments and key[1] == s and key[2] == device:
        return st["ridx"]
    r = fuse.row_index(mod_segments, s, device)
    if r is not None:
        st["ridx_key"], st["ridx"] = (mod_segments, s, device), r
    return r


def _fuse_fallback(reason):
    _fuse_state["fallback"] += 1
    if _fuse_state["fallback"] <= 5:
        log.warning("h3b fused DiTBlock.forward: original forward for this call (%s)", reason)


def install_fuse(mm=None):
    """Patch mm.DiTBlock.forward with the fused forward when H3_FUSE=1; returns whether it patched."""
    st = _fuse_state
    if st["target"] is not None:
        return True
    if os.environ.get("H3_FUSE", "0") != "1":
        return False
    if mm is None:
        import comfy.ldm.minimax.model as mm
    orig = mm.DiTBlock.forward
    bf16 = torch.bfloat16

    @functools.wraps(orig)
    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}, attention=None):  # noqa: B006
        def original(reason):
            _fuse_fallback(reason)
            return orig(self, x, t_emb, mod_segments, rope_freqs, transformer_options=transformer_options,
                        attention=attention)

        n1, n2 = self.norm1, self.norm2
        ok = (x.dim() == 2 and x.is_cuda and x.dtype == bf16 and x.is_contiguous() and x.data_ptr() % 16 == 0
              and x.shape[1] % 4 == 0 and n1.eps is not None and n2.eps is not None
              and tuple(n1.normalized_shape) == (x.shape[1],) and tuple(n2.normalized_shape) == (x.shape[1],)
              and not torch.is_grad_enabled())
        if not ok:
            return original(f"x={tuple(x.shape)} {x.dtype} cuda={x.is_cuda} contiguous={x.is_contiguous()} "
                            f"grad={torch.is_grad_enabled()}")
        s, D = x.shape
        ridx = _cached_row_index(mod_segments, s, x.device)
        if ridx is None:
            return original("mod_segments do not tile the rows")
        attn = self.attn if attention is None else attention
        vecs = [v.reshape(-1, D) for v in self.adaln_proj(t_emb)]
        s1a, sha, ga, s1m, shm, gm = fuse.modulation_tables(*vecs)
        run_every_op = getattr(sys.modules.get("comfy.ops"), "run_every_op", None)
        if run_every_op is not None:
            run_every_op()
        with _norm_weight(n1, x) as (w1, _):
            if w1 is None or w1.dtype != bf16 or not w1.is_contiguous():
                return original(f"norm1 weight {None if w1 is None else w1.dtype}")
            h = fuse.norm_mod(x, w1, float(n1.eps), ridx, s1a, sha)
        o = attn(h, rope_freqs=rope_freqs, transformer_options=transformer_options)
        del h
        o = o.contiguous()
        if run_every_op is not None:
            run_every_op()
        with _norm_weight(n2, x) as (w2, _):
            h = fuse.gate_norm_mod_(x, o, ga, w2, float(n2.eps), ridx, s1m, shm)
        del o
        o = self.mlp(h).contiguous()
        del h
        fuse.gate_(x, o, gm, ridx)
        st["fused"] += 1
        return x

    forward._h3b_orig = orig
    mm.DiTBlock.forward = forward
    st.update(target=mm, orig=orig, fused=0, fallback=0, ridx_key=None, ridx=None)
    return True


def uninstall_fuse():
    st = _fuse_state
    if st["target"] is not None:
        st["target"].DiTBlock.forward = st["orig"]
        st.update(target=None, orig=None, ridx_key=None, ridx=None)


def fuse_counters():
    """(forwards run fused, forwards sent to the original) since install_fuse."""
    return _fuse_state["fused"], _fuse_state["fallback"]


# ---------------------------------------------------------------------------
# after-import hooks for worker processes (h3_fuse_patch.py:152-183, boot/sitecustomize.py:26-44)

class _AfterImport(importlib.abc.MetaPathFinder):
    """Calls fn(module) right after the first module whose name satisfies
    match(name) has been executed, then leaves sys.meta_path."""

    def __init__(self, match, fn):
        self.match, self.fn = match, fn

    def find_spec(self, name, path=None, target=None):
        if not self.match(name):
            return None
        sys.meta_path.remove(self)  # let the normal finders locate the module
        try:
            spec = importlib.machinery.PathFinder.find_spec(name, path)
        finally:
            sys.meta_path.insert(0, self)
        if spec is None or spec.loader is None:
            return spec
        loader_exec = spec.loader.exec_module
        fn, me = self.fn, self

        def exec_module(module):
            loader_exec(module)
            if me in sys.meta_path:
                sys.meta_path.remove(me)
            fn(module)

        spec.loader.exec_module = exec_module
        return spec


def after_import(match, fn):
    """Run fn(module) after the module `match` selects is imported (match: a
    module name or a predicate on names).  A module already imported gets fn
    at once.  Returns the finder (None when fn already ran)."""
    pred = (lambda n: n == match) if isinstance(match, str) else match
    for name, mod in list(sys.modules.items()):
        if mod is not None and pred(name):
            fn(mod)
            return None
    finder = _AfterImport(pred, fn)
    sys.meta_path.insert(0, finder)
    return finder


def install_worker_hooks():
    """Register the env-gated installers as after-import hooks:
    H3_LINEAR_FAST=1 -> install_linear after comfy_kitchen.backends.cuda,
    H3_FUSE=1 -> install_fuse after comfy.ldm.minimax.model,
    H3B_SP=1 -> install_sp after *.minimax_sp.sp_forward.
    Returns the names of the hooks registered (or run at once)."""
    hooks = []
    if os.environ.get("H3_LINEAR_FAST", "0") == "1":
        after_import("comfy_kitchen.backends.cuda", install_linear)
        hooks.append("linear")
    if os.environ.get("H3_FUSE", "0") == "1":
        after_import("comfy.ldm.minimax.model", install_fuse)
        hooks.append("fuse")
    if os.environ.get("H3B_SP", "0") == "1":
        after_import(lambda n: n == "minimax_sp.sp_forward" or n.endswith(".minimax_sp.sp_forward"), install_sp)
        hooks.append("sp")
    return hooks
