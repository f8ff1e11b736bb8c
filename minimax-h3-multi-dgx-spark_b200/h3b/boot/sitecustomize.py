"""Interpreter-start hook for worker processes (the reference's
comfyui_nodes/h3-linear-fast/boot/sitecustomize.py:1-44 counterpart).

Worker ranks run sp_worker.py, which imports ComfyUI's model and
comfy_kitchen without loading the custom nodes, so the h3b installers cannot
run from a custom node's __init__ there.  Start a worker with this folder on
PYTHONPATH and any of H3_LINEAR_FAST=1 / H3_FUSE=1 / H3B_SP=1 set: the
original sitecustomize (the first other one on sys.path, if any) runs first,
then h3b.install.install_worker_hooks() registers after-import hooks that
install h3b once the target modules are imported.  With none of the
variables set, nothing of h3b is imported.
"""
import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
for _p in sys.path:
    _cand = os.path.join(_p, "sitecustomize.py") if _p else ""
    if _p and os.path.abspath(_p) != _here and os.path.exists(_cand):
        try:
            with open(_cand, encoding="utf-8") as _f:
                exec(compile(_f.read(), _cand, "exec"), {"__name__": "sitecustomize_orig", "__file__": _cand})
        except Exception:  # noqa: BLE001 -- the original hook's failure must not stop the worker
            pass
        break

if any(os.environ.get(v, "0") == "1" for v in ("H3_LINEAR_FAST", "H3_FUSE", "H3B_SP")):
    _pkg_parent = os.path.dirname(os.path.dirname(_here))
    if _pkg_parent not in sys.path:
        sys.path.insert(0, _pkg_parent)
    from h3b.install import install_worker_hooks

    install_worker_hooks()
