"""Fused RMSNorm / adaLN modulation / gate / residual ops over libh3b.

Kernel-level API of comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py:174-192:
  norm_mod(x, w, eps, ridx, s1, sh) -> h
  gate_norm_mod_(x, o, g, w, eps, ridx, s1, sh) -> h     (x updated in place)
  gate_(x, o, g, ridx) -> x                               (in place)
plus the per-forward helpers of comfyui_nodes/h3-fuse-graph/h3_fuse_patch.py:
  row_index(mod_segments, s, device)   :32-56
  modulation_tables(vecs)              :111-118
the producers that also quantise their output for the INT8 linear they feed
(norm_mod_quant, gate_norm_mod_quant_), and the plain RMSNorm of the per-head
q/k norm (rms_norm, comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:296-298).
"""
import torch

from ._lib import check, lib, ptr, require_cuda, stream_of
from .trace import span

BF16 = torch.bfloat16


def _check(x, w, ridx, s1, sh):
    require_cuda(x, w, ridx, s1, sh)
    if x.dim() != 2 or x.dtype != BF16 or not x.is_contiguous():
        raise ValueError(f"fused norm: x must be a contiguous 2-D bf16 tensor, got {x.dtype} {tuple(x.shape)}")
    S, D = x.shape
    if w.dtype != BF16 or w.numel() != D or not w.is_contiguous():
        raise ValueError("fused norm: w must be a contiguous bf16 [D] tensor")
    if ridx.dtype != torch.int32 or ridx.numel() != S or not ridx.is_contiguous():
        raise ValueError("fused norm: ridx must be a contiguous int32 [S] tensor")
    for t in (s1, sh):
        if t.dtype != BF16 or t.dim() != 2 or t.shape[1] != D or not t.is_contiguous():
            raise ValueError("fused norm: modulation tables must be contiguous bf16 [R, D]")
    if s1.shape[0] != sh.shape[0]:
        raise ValueError("fused norm: s1 and sh must have the same number of rows")
    return S, D, s1.shape[0]


def norm_mod(x, w, eps, ridx, s1, sh):
    """h = bf16(rbf16(rbf16(w * (rstd * x)) * s1[r]) + sh[r]) per row (x bf16 [S,D])."""
    S, D, R = _check(x, w, ridx, s1, sh)
    h = torch.empty_like(x)
    with span("norm_mod", 4 * S * D):
        check(lib.h3b_norm_mod(ptr(x), ptr(w), float(eps), ptr(ridx), ptr(s1), ptr(sh), ptr(h), S, D, R, stream_of(x)),
              "h3b_norm_mod")
    return h


def rms_norm(x, w, eps):
    """F.rms_norm(x, (D,), w, eps) over the last dimension, bit for bit (bf16 in and out):
    the per-head q/k norm of sp_attention without RoPE (sp_forward.py:296-298)."""
    require_cuda(x, w)
    D = x.shape[-1]
    if x.dtype != BF16 or w.dtype != BF16 or w.numel() != D or not x.is_contiguous():
        raise ValueError("rms_norm: x must be contiguous bf16 [..., D] and w bf16 [D]")
    x2 = x.view(-1, D)
    h = torch.empty_like(x)
    with span("rms_norm", 4 * x.numel()):
        check(lib.h3b_rms_norm(ptr(x2), ptr(w.contiguous()), float(eps), ptr(h), x2.shape[0], D, stream_of(x)),
              "h3b_rms_norm")
    return h


def gate_norm_mod_(x, o, g, w, eps, ridx, s1, sh):
    """x <- bf16(x + o * g[r]) in place; returns h = norm_mod(x)."""
    S, D, R = _check(x, w, ridx, s1, sh)
    require_cuda(o, g)
    if o.shape != x.shape or o.dtype != BF16 or not o.is_contiguous():
        raise ValueError("gate_norm_mod_: o must match x")
    if g.dtype != BF16 or tuple(g.shape) != (R, D) or not g.is_contiguous():
        raise ValueError("gate_norm_mod_: g must be a contiguous bf16 [R, D] table")
    h = torch.empty_like(x)
    with span("gate_norm_mod_", 8 * S * D):
        check(lib.h3b_gate_norm_mod_(ptr(x), ptr(o), ptr(g), ptr(w), float(eps), ptr(ridx), ptr(s1), ptr(sh), ptr(h),
                                     S, D, R, stream_of(x)), "h3b_gate_norm_mod_")
    return h


def norm_mod_quant(x, w, eps, ridx, s1, sh):
    """quant_rowwise(norm_mod(x, w, eps, ridx, s1, sh)) in one pass: (xq int8 [S,D], xs fp32 [S,1])."""
    S, D, R = _check(x, w, ridx, s1, sh)
    xq = torch.empty((S, D), dtype=torch.int8, device=x.device)
    xs = torch.empty((S, 1), dtype=torch.float32, device=x.device)
    with span("norm_mod_quant", 3 * S * D + 4 * S):
        check(lib.h3b_norm_mod_quant(ptr(x), ptr(w), float(eps), ptr(ridx), ptr(s1), ptr(sh), ptr(xq), ptr(xs),
                                     S, D, R, stream_of(x)), "h3b_norm_mod_quant")
    return xq, xs


def gate_norm_mod_quant_(x, o, g, w, eps, ridx, s1, sh):
    """x <- bf16(x + o*g[r]) in place; returns quant_rowwise(norm_mod(x)) as (xq, xs)."""
    S, D, R = _check(x, w, ridx, s1, sh)
    require_cuda(o, g)
    if o.shape != x.shape or o.dtype != BF16 or not o.is_contiguous():
        raise ValueError("gate_norm_mod_quant_: o must match x")
    if g.dtype != BF16 or tuple(g.shape) != (R, D) or not g.is_contiguous():
        raise ValueError("gate_norm_mod_quant_: g must be a contiguous bf16 [R, D] table")
    xq = torch.empty((S, D), dtype=torch.int8, device=x.device)
    xs = torch.empty((S, 1), dtype=torch.float32, device=x.device)
    with span("gate_norm_mod_quant_", 7 * S * D + 4 * S):
        check(lib.h3b_gate_norm_mod_quant_(ptr(x), ptr(o), ptr(g), ptr(w), float(eps), ptr(ridx), ptr(s1), ptr(sh),
                                           ptr(xq), ptr(xs), S, D, R, stream_of(x)), "h3b_gate_norm_mod_quant_")
    return xq, xs


def gate_(x, o, g, ridx):
    """x <- bf16(x + o * g[r]) in place; returns x."""
    require_cuda(x, o, g, ridx)
    if x.dim() != 2 or x.dtype != BF16 or not x.is_contiguous():
        raise ValueError("gate_: x must be a contiguous 2-D bf16 tensor")
    S, D = x.shape
    if o.shape != x.shape or o.dtype != BF16 or not o.is_contiguous():
        raise ValueError("gate_: o must match x")
    if g.dtype != BF16 or g.dim() != 2 or g.shape[1] != D or not g.is_contiguous():
        raise ValueError("gate_: g must be a contiguous bf16 [R, D] table")
    if ridx.dtype != torch.int32 or ridx.numel() != S:
        raise ValueError("gate_: ridx must be int32 [S]")
    with span("gate_", 6 * S * D):
        check(lib.h3b_gate_(ptr(x), ptr(o), ptr(g), ptr(ridx), S, D, g.shape[0], stream_of(x)), "h3b_gate_")
    return x


def row_index(mod_segments, s, device):
    """(start, stop, row) triples -> int32 [s] table-row index, or None if the
    segments do not tile 0..s exactly (h3_fuse_patch.py:32-56).  `row` is an
    int or a per-row integer tensor."""
    segs = sorted(((a, b, row) for a, b, row in mod_segments), key=lambda t: t[0])
    pos = 0
    for a, b, row in segs:
        if a != pos or b < a:
            return None
        if torch.is_tensor(row) and row.numel() != b - a:
            return None
        pos = b
    if pos != s:
        return None
    r = torch.empty(s, dtype=torch.int32, device=device)
    for a, b, row in segs:
        if torch.is_tensor(row):
            r[a:b] = row.to(device=device, dtype=torch.int32)
        else:
            r[a:b] = int(row)
    return r


def modulation_tables(shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp):
    """adaLN vectors -> contiguous bf16 tables (s1a, sha, ga, s1m, shm, gm) with
    s1 = bf16(1.0 + bf16(scale)) (h3_fuse_patch.py:111-118)."""
    bf = lambda t: t.to(BF16)  # noqa: E731
    s1a = (1.0 + bf(scale_msa)).contiguous()
    s1m = (1.0 + bf(scale_mlp)).contiguous()
    return s1a, bf(shift_msa).contiguous(), bf(gate_msa).contiguous(), s1m, bf(shift_mlp).contiguous(), \
        bf(gate_mlp).contiguous()
