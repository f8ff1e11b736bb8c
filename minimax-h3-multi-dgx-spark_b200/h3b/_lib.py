"""ctypes binding of libh3b.so (the C ABI in include/h3b.h).

Importing this module loads the library and fails loudly if it is missing:
the package has no CPU or PyTorch fallback for any op.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libh3b.so")

H3B_OK = 0
STATUS_OK, STATUS_MBAR_TIMEOUT, STATUS_PEER_TIMEOUT, STATUS_BAD_INDEX = 0, 1, 2, 3
STATUS_NAMES = {0: "ok", 1: "GEMM pipeline wait timed out", 2: "peer barrier timed out",
                3: "modulation row index out of range"}

# (name, restype, argtypes)
_P, _I64, _F32, _I32, _U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_uint32
_PP = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = [
    ("h3b_abi_version", _I32, []),
    ("h3b_last_error", ctypes.c_char_p, []),
    ("h3b_status_get", _I32, [ctypes.POINTER(ctypes.c_int), _P]),
    ("h3b_status_clear", _I32, [_P]),
    ("h3b_quant_rowwise", _I32, [_P, _I64, _I64, _I64, _P, _P, _P]),
    ("h3b_quant_rowwise_convrot", _I32, [_P, _I64, _I64, _I64, _I64, _P, _P, _P]),
    ("h3b_swiglu_quant_convrot", _I32, [_P, _I64, _I64, _I64, _I64, _P, _P, _P]),
    ("h3b_int8_mm_scaled", _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_int8_mm_scaled_gelu", _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_int8_mm_i32", _I32, [_P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_int8_mm_scaled_a2a", _I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _PP, _I64, _I64, _I64, _I64, _I32, _P]),
    ("h3b_int8_mm_scaled_a2a_qknorm", _I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _PP, _I64, _I64, _I64, _I64, _I32,
                                             _P, _I64, ctypes.c_float, _P]),
    ("h3b_int8_linear", _I32, [_P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _P, _P]),
    ("h3b_int8_linear_noalloc", _I32, [_P, _I64, _I64, _P, _P, _P, _I64, _P, _P]),
    ("h3b_norm_mod", _I32, [_P, _P, _F32, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_rms_norm", _I32, [_P, _P, ctypes.c_float, _P, _I64, _I64, _P]),
    ("h3b_gate_norm_mod_", _I32, [_P, _P, _P, _P, _F32, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_gate_", _I32, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_norm_mod_quant", _I32, [_P, _P, _F32, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_gate_norm_mod_quant_", _I32, [_P, _P, _P, _P, _F32, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("h3b_gelu_quant", _I32, [_P, _I64, _I64, _I64, _P, _P, _P]),
    ("h3b_gelu_tanh", _I32, [_P, _P, _I64, _P]),
    ("h3b_a2a_pack", _I32, [_P, _I64, _P, _I64, _I64, _I64, _I32, _P]),
    ("h3b_a2a_unpack", _I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _P]),
    ("h3b_ipc_handle", _I32, [_P, _P, ctypes.POINTER(ctypes.c_int64)]),
    ("h3b_ipc_open", _I32, [_P, _I64, _PP, _PP]),
    ("h3b_ipc_close", _I32, [_P]),
    ("h3b_peer_barrier", _I32, [_PP, _I32, _I32, _U32, _I64, _P]),
    ("h3b_a2a_fwd_p2p", _I32, [_I32, _PP, _I64, _PP, _I64, _I64, _I64, _I64, _I64, _I32, _P]),
    ("h3b_a2a_inv_quant", _I32, [_PP, _I64, _I64, _I64, _I64, _I32, _P, _P, _P]),
    ("h3b_a2a_inv_p2p", _I32, [_P, _I64, _PP, ctypes.POINTER(ctypes.c_int64), _I64, _I64, _I64, _I32, _P]),
]


class H3BError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libh3b.so is not built ({LIB_PATH}); run "
                          "`python minimax-h3-multi-dgx-spark_b200/build.py` (needs nvcc for sm_100a)")
    L = ctypes.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    if L.h3b_abi_version() != 2:
        raise ImportError("libh3b.so ABI version mismatch; rebuild it")
    return L


lib = _load()


def check(rc, what):
    if rc != H3B_OK:
        msg = lib.h3b_last_error().decode(errors="replace")
        raise H3BError(f"{what} failed ({rc}): {msg}")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def ptr_array(values):
    arr = (ctypes.c_void_p * len(values))(*[ctypes.c_void_p(int(v)) for v in values])
    return ctypes.cast(arr, _PP), arr


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise TypeError("h3b ops run on CUDA tensors only (there is no CPU path); got a tensor on " + str(t.device))


def status(device=None, raise_on_error=False):
    """Synchronise the current stream and read the device status word."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        v = ctypes.c_int(0)
        check(lib.h3b_status_get(ctypes.byref(v), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
              "h3b_status_get")
    if raise_on_error and v.value != STATUS_OK:
        raise H3BError(f"device status {v.value}: {STATUS_NAMES.get(v.value, 'unknown')}")
    return v.value


def clear_status(device=None):
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check(lib.h3b_status_clear(ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)), "h3b_status_clear")
