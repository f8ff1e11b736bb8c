"""CPU oracle for the H3 DiT hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this package, and only as the checker (or the timed CPU baseline).  The product
(minimax-h3-multi-dgx-spark_b200/h3b) never imports it and has no CPU path.

Contents
  * ctypes wrappers over h3_oracle.c (quantiser, INT8 GEMM + dequant epilogue,
    the three fused norm/modulation/gate kernels) taking numpy arrays;
  * sp_layout: the Ulysses all-to-all layout restated with numpy reshapes
    (comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:140-198);
  * seeded input generators shared by tests and benches (torch.Generator on
    CPU, so every machine draws the same values).

bf16 tensors are passed as uint16 numpy arrays holding the raw bit patterns.
"""
import ctypes
import os

import numpy as np

from .build import LIB, build_oracle

RNE, TRUNC = 0, 1
RSQRT_EXACT, RSQRT_RECIP = 0, 1

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build_oracle()
        L = ctypes.CDLL(LIB)
        p, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.h3o_quant_rowwise.argtypes = [p, i64, i64, p, p]
        L.h3o_quant_rowwise.restype = None
        L.h3o_quant_rowwise_convrot.argtypes = [p, i64, i64, i64, p, p, p]
        L.h3o_quant_rowwise_convrot.restype = None
        L.h3o_rotate_groups.argtypes = [p, i64, i64, p]
        L.h3o_rotate_groups.restype = None
        L.h3o_int8_mm_scaled.argtypes = [p, p, p, p, p, i64, i64, i64, p, p, i32]
        L.h3o_int8_mm_scaled.restype = None
        L.h3o_row_sumsq.argtypes = [p, i64, i32]
        L.h3o_row_sumsq.restype = f32
        L.h3o_rstd.argtypes = [f32, i64, f32, i32]
        L.h3o_rstd.restype = f32
        L.h3o_norm_mod.argtypes = [p, p, f32, p, p, p, p, i64, i64, p, p, i32, i32, i32, p]
        L.h3o_norm_mod.restype = None
        L.h3o_gate_norm_mod_.argtypes = [p, p, p, p, f32, p, p, p, p, i64, i64, p, p, i32, i32, i32, p]
        L.h3o_gate_norm_mod_.restype = None
        L.h3o_gate_.argtypes = [p, p, p, p, i64, i64, i32]
        L.h3o_gate_.restype = None
        L.h3o_one_plus.argtypes = [p, p, i64, i32]
        L.h3o_one_plus.restype = None
        L.h3o_f32_to_bf16.argtypes = [f32, i32]
        L.h3o_f32_to_bf16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    a = np.ascontiguousarray(a)
    if a.dtype != dtype:
        raise TypeError(f"expected {dtype}, got {a.dtype}")
    return a


# ---------------------------------------------------------------------------
# bf16 helpers (numpy)

def f32_to_bf16(a, mode=RNE):
    """float32 array -> uint16 bf16 bits (RNE like the GPU, or truncation)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    if mode == TRUNC:
        return (u >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) & 0x8000 | 0x7FC0).astype(np.uint16)
    return r


def bf16_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# a1 .. a7

def quant_rowwise(x_bf16):
    """x [M,K] bf16 bits -> (q [M,K] int8, s [M] float32)."""
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    lib().h3o_quant_rowwise(_ptr(x), M, K, _ptr(q), _ptr(s))
    return q, s


def rotate_groups(x_bf16, group=256):
    """x [M,K] bf16 bits -> fp32 [M,K]: each group of `group` columns rotated by
    the normalised Walsh-Hadamard transform (h3o_rotate_groups)."""
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    y = np.empty((M, K), np.float32)
    for m in range(M):
        lib().h3o_rotate_groups(_ptr(x[m]), K, group, _ptr(y[m]))
    return y


def quant_rowwise_convrot(x_bf16, group=256):
    """x [M,K] bf16 bits -> (q [M,K] int8, s [M] float32) of the ConvRot-rotated rows."""
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    work = np.empty(K, np.float32)
    lib().h3o_quant_rowwise_convrot(_ptr(x), M, K, group, _ptr(q), _ptr(s), _ptr(work))
    return q, s


def int8_mm_scaled(xq, w, xs, ws, bias=None, final_round=RNE, want_acc=False):
    """xq [M,K] int8, w [N,K] int8, xs [M] f32, ws [N] f32, bias [N] bf16 bits or None
    -> y [M,N] bf16 bits (and acc [M,N] int32 when want_acc)."""
    xq, w = _c(xq, np.int8), _c(w, np.int8)
    xs, ws = _c(np.reshape(xs, -1), np.float32), _c(ws, np.float32)
    M, K = xq.shape
    N = w.shape[0]
    assert w.shape[1] == K and xs.shape[0] == M and ws.shape[0] == N
    b = None if bias is None else _c(bias, np.uint16)
    y = np.empty((M, N), np.uint16)
    acc = np.empty((M, N), np.int32) if want_acc else None
    lib().h3o_int8_mm_scaled(_ptr(xq), _ptr(w), _ptr(xs), _ptr(ws), _ptr(b), M, N, K, _ptr(y), _ptr(acc),
                             final_round)
    return (y, acc) if want_acc else y


def row_sumsq(row_f32, fma=True):
    r = _c(row_f32, np.float32)
    return float(lib().h3o_row_sumsq(_ptr(r), r.shape[0], int(fma)))


def rstd_of(tot, D, eps, rsqrt_mode=RSQRT_EXACT):
    return np.float32(lib().h3o_rstd(np.float32(tot), D, np.float32(eps), rsqrt_mode))


def norm_mod(x, w, eps, ridx, s1, sh, rstd_override=None, fma=True, rsqrt_mode=RSQRT_EXACT, final_round=RNE):
    """Returns (h, rstd) -- h [S,D] bf16 bits, rstd [S] float32 actually used."""
    x, w = _c(x, np.uint16), _c(w, np.uint16)
    ridx = _c(ridx, np.int32)
    s1, sh = _c(s1, np.uint16), _c(sh, np.uint16)
    S, D = x.shape
    h = np.empty((S, D), np.uint16)
    rstd = np.empty(S, np.float32)
    ov = None if rstd_override is None else _c(rstd_override, np.float32)
    buf = np.empty(D, np.float32)
    lib().h3o_norm_mod(_ptr(x), _ptr(w), np.float32(eps), _ptr(ridx), _ptr(s1), _ptr(sh), _ptr(h), S, D,
                       _ptr(ov), _ptr(rstd), int(fma), rsqrt_mode, final_round, _ptr(buf))
    return h, rstd


def gate_norm_mod_(x, o, g, w, eps, ridx, s1, sh, rstd_override=None, fma=True, rsqrt_mode=RSQRT_EXACT,
                   final_round=RNE):
    """Returns (x_new, h, rstd); the input x is not modified."""
    xn = np.array(_c(x, np.uint16), copy=True)
    o, g, w = _c(o, np.uint16), _c(g, np.uint16), _c(w, np.uint16)
    ridx = _c(ridx, np.int32)
    s1, sh = _c(s1, np.uint16), _c(sh, np.uint16)
    S, D = xn.shape
    h = np.empty((S, D), np.uint16)
    rstd = np.empty(S, np.float32)
    ov = None if rstd_override is None else _c(rstd_override, np.float32)
    buf = np.empty(D, np.float32)
    lib().h3o_gate_norm_mod_(_ptr(xn), _ptr(o), _ptr(g), _ptr(w), np.float32(eps), _ptr(ridx), _ptr(s1),
                             _ptr(sh), _ptr(h), S, D, _ptr(ov), _ptr(rstd), int(fma), rsqrt_mode, final_round,
                             _ptr(buf))
    return xn, h, rstd


def gate_(x, o, g, ridx, final_round=RNE):
    """Returns the new x; the input is not modified."""
    xn = np.array(_c(x, np.uint16), copy=True)
    o, g = _c(o, np.uint16), _c(g, np.uint16)
    ridx = _c(ridx, np.int32)
    S, D = xn.shape
    lib().h3o_gate_(_ptr(xn), _ptr(o), _ptr(g), _ptr(ridx), S, D, final_round)
    return xn


def one_plus(scale, final_round=RNE):
    sc = _c(scale, np.uint16)
    out = np.empty_like(sc)
    lib().h3o_one_plus(_ptr(sc), _ptr(out), sc.size, final_round)
    return out
