"""INT8 linear ops (activation quantiser, GEMM + dequant, patched Linear) over libh3b.

Mirrors the reference's operator surface:
  quant_rowwise / quant_rowwise_convrot      the quantiser called at h3_linear_fast_patch.py:89-95
  int8_mm_scaled(xq, w, xs, ws, out=None)    comfyui_nodes/h3-linear-fast/int8_gemm_triton.py:74-83
  supported(K)                               int8_gemm_triton.py:86-87
  int8_linear(x, weight, weight_scale, ...)  the patched comfy_kitchen int8_linear,
                                             comfyui_nodes/h3-linear-fast/h3_linear_fast_patch.py:60-110
Outputs are allocated with PyTorch's caching allocator on the input's device,
kernels run on the current CUDA stream, shape/dtype violations raise.
"""
import torch

from ._lib import check, lib, ptr, ptr_array, require_cuda, stream_of
from .trace import span


def supported(K):
    """K the GEMM accepts: a multiple of the 128-byte k-block (the reference needs K % 128 == 0 too)."""
    return K % 128 == 0


def quant_rowwise(x, xq=None, xs=None):
    """Per-token absmax quantisation: x bf16 [M,K] -> (xq int8 [M,K], xs fp32 [M,1]).

    xs = absmax/127, xq = clamp(round_half_even(x/xs), -127, 127); zero rows give 0/0.
    The [M,1] scale shape follows the reference's x_s (h3_linear_fast_patch.py:91)."""
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError(f"quant_rowwise: x must be a 2-D bf16 tensor with unit column stride, got {x.dtype} {tuple(x.shape)}")
    M, K = x.shape
    if xq is None:
        xq = torch.empty((M, K), dtype=torch.int8, device=x.device)
    if xs is None:
        xs = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    with span("quant", 3 * M * K + 4 * M):
        check(lib.h3b_quant_rowwise(ptr(x), x.stride(0), M, K, ptr(xq), ptr(xs), stream_of(x)), "h3b_quant_rowwise")
    return xq, xs


def quant_rowwise_convrot(x, group=256, xq=None, xs=None):
    """quant_rowwise of the ConvRot-rotated rows: each group of `group` (64 or 256)
    columns rotated by the normalised Walsh-Hadamard transform first
    (h3b_quant_rowwise_convrot; the quantiser of the reference's fast path,
    h3_linear_fast_patch.py:89-95)."""
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("quant_rowwise_convrot: x must be a 2-D bf16 tensor with unit column stride")
    M, K = x.shape
    if xq is None:
        xq = torch.empty((M, K), dtype=torch.int8, device=x.device)
    if xs is None:
        xs = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    with span("quant_convrot", 3 * M * K + 4 * M):
        check(lib.h3b_quant_rowwise_convrot(ptr(x), x.stride(0), M, K, group, ptr(xq), ptr(xs), stream_of(x)),
              "h3b_quant_rowwise_convrot")
    return xq, xs


def swiglu_quant_convrot(x, group=256, xq=None, xs=None):
    """quant_rowwise_convrot(bf16(silu(x[:, :K]) * x[:, K:])) for x bf16 [M, 2K]
    without materialising the activation (h3b_swiglu_quant_convrot; the
    reference fast path's input_act="swiglu", h3_linear_fast_patch.py:63,93-95)."""
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1 or x.shape[1] % 2:
        raise ValueError("swiglu_quant_convrot: x must be a 2-D bf16 [M, 2K] tensor with unit column stride")
    M, K = x.shape[0], x.shape[1] // 2
    if xq is None:
        xq = torch.empty((M, K), dtype=torch.int8, device=x.device)
    if xs is None:
        xs = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    with span("swiglu_quant_convrot", 5 * M * K + 4 * M):
        check(lib.h3b_swiglu_quant_convrot(ptr(x), x.stride(0), M, K, group, ptr(xq), ptr(xs), stream_of(x)),
              "h3b_swiglu_quant_convrot")
    return xq, xs


def gelu_quant(u, xq=None, xs=None):
    """quant_rowwise(F.gelu(u, approximate="tanh")) without materialising the GELU output."""
    require_cuda(u)
    if u.dtype != torch.bfloat16 or u.dim() != 2 or u.stride(1) != 1:
        raise ValueError("gelu_quant: u must be a 2-D bf16 tensor with unit column stride")
    M, K = u.shape
    if xq is None:
        xq = torch.empty((M, K), dtype=torch.int8, device=u.device)
    if xs is None:
        xs = torch.empty((M, 1), dtype=torch.float32, device=u.device)
    with span("gelu_quant", 3 * M * K + 4 * M):
        check(lib.h3b_gelu_quant(ptr(u), u.stride(0), M, K, ptr(xq), ptr(xs), stream_of(u)), "h3b_gelu_quant")
    return xq, xs


def gelu_tanh(u, out=None):
    """F.gelu(u, approximate="tanh") for bf16 u (any shape, contiguous), bit for bit."""
    require_cuda(u)
    if u.dtype != torch.bfloat16 or not u.is_contiguous() or u.numel() % 2:
        raise ValueError("gelu_tanh: u must be a contiguous bf16 tensor with an even number of elements")
    if out is None:
        out = torch.empty_like(u)
    with span("gelu", 4 * u.numel()):
        check(lib.h3b_gelu_tanh(ptr(u), ptr(out), u.numel(), stream_of(u)), "h3b_gelu_tanh")
    return out


def _gemm_checks(xq, w):
    require_cuda(xq, w)
    if xq.dtype != torch.int8 or w.dtype != torch.int8 or xq.dim() != 2 or w.dim() != 2:
        raise ValueError("int8 GEMM: xq and w must be 2-D int8 tensors")
    M, K = xq.shape
    N = w.shape[0]
    assert w.shape[1] == K and xq.is_contiguous() and w.is_contiguous()
    return M, N, K


def int8_mm_scaled(xq, w, xs, ws, out=None, bias=None, act=None):
    """xq [M,K] int8, w [N,K] int8, xs [M,1] fp32, ws [N] fp32 -> [M,N] bf16.

    out = bf16((float(xq @ w.T) * xs) * ws [+ bias]) with one rounding; with
    act="gelu", F.gelu(out, approximate="tanh") computed in the epilogue."""
    M, N, K = _gemm_checks(xq, w)
    xs = xs.reshape(-1)
    if xs.dtype != torch.float32 or ws.dtype != torch.float32 or xs.numel() != M or ws.numel() != N:
        raise ValueError("int8_mm_scaled: xs must be fp32 [M] / [M,1] and ws fp32 [N]")
    xs, ws = xs.contiguous(), ws.contiguous()
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != N:
            raise ValueError("int8_mm_scaled: bias must be bf16 [N]")
        bias = bias.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=xq.device)
    if act not in (None, "gelu"):
        raise ValueError(f"int8_mm_scaled: unknown act {act!r}")
    fn = lib.h3b_int8_mm_scaled_gelu if act == "gelu" else lib.h3b_int8_mm_scaled
    with span("gemm", 2 * M * N * K):
        check(fn(ptr(xq), ptr(w), ptr(xs), ptr(ws), ptr(bias), ptr(out), M, N, K, stream_of(xq)),
              "h3b_int8_mm_scaled_gelu" if act else "h3b_int8_mm_scaled")
    return out


def int8_mm_scaled_a2a(xq, w, xs, ws, bias, dst_ptrs, row_start, seg, head_dim, heads_per_rank, world, norm_w=None,
                       norm_eps=1e-6):
    """int8_mm_scaled whose epilogue stores column n of the [M,N] product into
    the receive buffer of the rank owning its head (h3b_int8_mm_scaled_a2a):
    dst_ptrs = device addresses [segment * world + rank] of bf16 buffers with
    rows of heads_per_rank*head_dim elements and at least row_start + M rows
    (the caller guarantees their size).  norm_w (bf16 [n, 128]): the first n
    segments (q, k) get a per-head RMSNorm with these weights in the epilogue
    (h3b_int8_mm_scaled_a2a_qknorm).  Returns nothing; the receivers see the
    rows after a peer barrier."""
    M, N, K = _gemm_checks(xq, w)
    xs = xs.reshape(-1)
    if xs.dtype != torch.float32 or ws.dtype != torch.float32 or xs.numel() != M or ws.numel() != N:
        raise ValueError("int8_mm_scaled_a2a: xs must be fp32 [M] / [M,1] and ws fp32 [N]")
    xs, ws = xs.contiguous(), ws.contiguous()
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != N:
            raise ValueError("int8_mm_scaled_a2a: bias must be bf16 [N]")
        bias = bias.contiguous()
    if len(dst_ptrs) != (N // seg) * world:
        raise ValueError("int8_mm_scaled_a2a: one destination per segment and rank")
    arr, keep = ptr_array(dst_ptrs)
    if norm_w is not None:
        if norm_w.dtype != torch.bfloat16 or norm_w.dim() != 2 or norm_w.shape[1] != head_dim:
            raise ValueError("int8_mm_scaled_a2a: norm_w must be bf16 [segments, head_dim]")
        norm_w = norm_w.contiguous()
        with span("gemm_a2a", 2 * M * N * K):
            check(lib.h3b_int8_mm_scaled_a2a_qknorm(ptr(xq), ptr(w), ptr(xs), ptr(ws), ptr(bias), M, N, K, arr,
                                                    row_start, seg, head_dim, heads_per_rank, world, ptr(norm_w),
                                                    norm_w.shape[0], float(norm_eps), stream_of(xq)),
                  "h3b_int8_mm_scaled_a2a_qknorm")
    else:
        with span("gemm_a2a", 2 * M * N * K):
            check(lib.h3b_int8_mm_scaled_a2a(ptr(xq), ptr(w), ptr(xs), ptr(ws), ptr(bias), M, N, K, arr, row_start,
                                             seg, head_dim, heads_per_rank, world, stream_of(xq)),
                  "h3b_int8_mm_scaled_a2a")
    del keep


def int8_mm_i32(xq, w, out=None):
    """Raw int32 accumulators xq @ w.T (for bit-exact checks of the tensor-core path)."""
    M, N, K = _gemm_checks(xq, w)
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32, device=xq.device)
    with span("gemm_i32", 2 * M * N * K):
        check(lib.h3b_int8_mm_i32(ptr(xq), ptr(w), ptr(out), M, N, K, stream_of(xq)), "h3b_int8_mm_i32")
    return out


def linear(x, w, ws, bias=None, convrot_group=0, swiglu=False):
    """The INT8 linear on a [*, K] bf16 activation: per-token quant + GEMM + dequant(+bias).
    convrot_group (64 / 256): the ConvRot quantiser, for weights stored rotated;
    swiglu (with convrot_group): x is [*, 2K] and the quantised row is
    bf16(silu(x[..., :K]) * x[..., K:])."""
    kin = x.shape[-1]
    x2d = x.reshape(-1, kin)
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    if swiglu:
        if not convrot_group:
            raise NotImplementedError("h3b linear: the SwiGLU input is covered with the ConvRot quantiser only")
        xq, xs = swiglu_quant_convrot(x2d, convrot_group)
    else:
        xq, xs = quant_rowwise_convrot(x2d, convrot_group) if convrot_group else quant_rowwise(x2d)
    out = int8_mm_scaled(xq, w, xs, ws, bias=bias)
    return out if x.dim() == 2 else out.reshape(*x.shape[:-1], w.shape[0])


def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256,
                input_act=None, input_act_weight=None, input_act_eps=0.0, residual=None, residual_scale=None):
    """Signature of comfy_kitchen.backends.cuda.int8_linear (h3_linear_fast_patch.py:60-61).

    Covers the plain per-token quantiser (convrot=False) and the ConvRot one
    (convrot=True, convrot_groupsize 64 or 256 -- the reference's fast path
    takes 256 only, :64), the latter also with the SwiGLU input activation
    (input_act="swiglu", x [*, 2K]), bias optional, no residual -- every call
    the reference's fast path accepts (:64-76); anything else raises
    NotImplementedError so that an installer can route the call to
    the original implementation, as the reference does for ineligible calls
    (h3_linear_fast_patch.py:64-80)."""
    if input_act not in (None, "none", "swiglu") or residual is not None:
        raise NotImplementedError("h3b int8_linear: this input_act / residual variant is not covered")
    if input_act == "swiglu" and (not convrot or input_act_weight is not None or input_act_eps):
        raise NotImplementedError("h3b int8_linear: SwiGLU is covered with ConvRot and no activation weight")
    if convrot and convrot_groupsize not in (64, 256):
        raise NotImplementedError(f"h3b int8_linear: ConvRot group {convrot_groupsize} (64 or 256 covered)")
    if (out_dtype or x.dtype) != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise NotImplementedError("h3b int8_linear: bf16 in/out only")
    n = weight.shape[0]
    ws = weight_scale.reshape(-1).to(torch.float32)
    if ws.numel() != n:
        ws = ws.expand(n).contiguous()
    return linear(x, weight.contiguous(), ws, bias, convrot_group=convrot_groupsize if convrot else 0,
                  swiglu=input_act == "swiglu")
