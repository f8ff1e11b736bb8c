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
  fuse_kernels()        the module to import as `fk` in place of h3_fuse_kernels
      (h3_fuse_patch.py:81): h3b.fuse, with the same norm_mod / gate_norm_mod_ /
      gate_ signatures.
"""
import logging
import os

from . import fuse, linear, sp
from ._lib import H3BError

log = logging.getLogger("h3b")
_linear_state = {"target": None, "orig": None, "disabled": False, "fast_calls": 0, "fallback_calls": 0}
_sp_state = {"target": None, "orig": None}


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
