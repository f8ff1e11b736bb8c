"""The reference's eager PyTorch path for the H3 block hot path -- TEST INFRASTRUCTURE.

Used only by tests (as the checker of the h3b block on the GPU) and by
bench.py's CPU-baseline legs (timed on the host's cores).  Device-agnostic:
the same code runs on CPU or CUDA tensors.

What it restates (reference paths):
  * the eager DiTBlock sequence the fused kernels replace
    (comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py:3-7): F.rms_norm, then
    h.mul_(1 + scale).add_(shift), x.addcmul_(branch, gate);
  * the INT8 linear: per-token absmax quantisation (the formula of the
    benchmark configuration; comfy-kitchen's ConvRot quantiser is not in the
    reference), torch._int_mm, and the epilogue of
    comfyui_nodes/h3-linear-fast/int8_gemm_triton.py:2,61-66 plus bias;
  * the Ulysses all-to-all of comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:158-198
    (reshape/transpose + all_to_all_single);
  * sp_attention (sp_forward.py:276-318) with PyTorch SDPA.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F

BF16 = torch.bfloat16


def quant_rowwise(x):
    """scale = absmax / 127 as an IEEE division.  The divisor is a tensor on
    purpose: PyTorch's CUDA kernel turns division by a Python scalar into a
    multiplication by its rounded reciprocal, which changes the last bit of
    about 3% of the scales."""
    xf = x.float()
    amax = xf.abs().amax(dim=-1, keepdim=True)
    s = amax / torch.full_like(amax, 127.0)
    q = torch.where(s > 0, torch.round(xf / torch.where(s > 0, s, torch.ones_like(s))), torch.zeros_like(xf))
    return q.clamp_(-127, 127).to(torch.int8), s


def int8_mm_scaled(xq, w, xs, ws, bias=None):
    acc = torch._int_mm(xq, w.t())
    y = (acc.float() * xs.reshape(-1, 1)) * ws
    if bias is not None:
        y = y + bias.float()
    return y.to(BF16)


def linear(x, w, ws, bias=None):
    x2 = x.reshape(-1, x.shape[-1])
    q, s = quant_rowwise(x2)
    y = int8_mm_scaled(q, w, s, ws, bias)
    return y.reshape(*x.shape[:-1], w.shape[0])


def norm_mod(x, w, eps, ridx, s1, sh):
    r = ridx.long()
    return (F.rms_norm(x, (x.shape[-1],), w, eps) * s1[r]) + sh[r]


def gate_(x, o, g, ridx):
    return x.addcmul_(o, g[ridx.long()])


def gate_norm_mod_(x, o, g, w, eps, ridx, s1, sh):
    gate_(x, o, g, ridx)
    return norm_mod(x, w, eps, ridx, s1, sh)


def modulation_tables(shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp):
    """adaLN vectors -> bf16 tables (s1a, sha, ga, s1m, shm, gm), s1 = bf16(1.0 + bf16(scale))
    (h3_fuse_patch.py:111-118, evaluated with PyTorch as the reference does)."""
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    return (1.0 + bf(scale_msa)), bf(shift_msa), bf(gate_msa), (1.0 + bf(scale_mlp)), bf(shift_mlp), bf(gate_mlp)


def a2a_gather_seq_scatter_heads(t, ctx):
    s_local, heads, dim = t.shape
    p = ctx.world
    hp = heads // p
    chunk = hp * dim
    send = t.reshape(s_local, p, chunk).transpose(0, 1).contiguous().view(-1)
    out = torch.empty(ctx.seq_len * chunk, dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, send, output_split_sizes=[n * chunk for n in ctx.splits],
                           input_split_sizes=[ctx.local * chunk] * p, group=ctx.group)
    return out.view(ctx.seq_len, hp, dim)


def a2a_scatter_seq_gather_heads(t, ctx):
    chunk = t.shape[1]
    p = ctx.world
    out = torch.empty(p * ctx.local * chunk, dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous().view(-1), output_split_sizes=[ctx.local * chunk] * p,
                           input_split_sizes=[n * chunk for n in ctx.splits], group=ctx.group)
    return out.view(p, ctx.local, chunk).transpose(0, 1).reshape(ctx.local, p * chunk)


def sdpa_heads(q, k, v):
    o = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0),
                                       v.transpose(0, 1).unsqueeze(0))
    sq, h, dh = q.shape
    return o.squeeze(0).transpose(0, 1).reshape(sq, h * dh)


def block_forward(cfg, p, x, ridx, ctx=None, text=None):
    """Same block as h3b.model.block_forward, in eager PyTorch ops (x updated in place)."""
    s1a, sha, ga, s1m, shm, gm = p.tables
    D, H, Dh = cfg.dim, cfg.heads, cfg.head_dim
    s = x.shape[0]
    h = norm_mod(x, p.n1w, cfg.eps, ridx, s1a, sha)
    qkv = linear(h, p.qkv.w, p.qkv.ws, p.qkv.b)
    q, k, v = qkv[:, :D].view(s, H, Dh), qkv[:, D:2 * D].view(s, H, Dh), qkv[:, 2 * D:].view(s, H, Dh)
    if getattr(cfg, "qk_norm", False):  # attn.q_norm / k_norm without RoPE, sp_forward.py:296-298
        q = F.rms_norm(q, (Dh,), p.qkn[0], cfg.eps)
        k = F.rms_norm(k, (Dh,), p.qkn[1], cfg.eps)
    if ctx is not None and ctx.world > 1:
        q, k, v = (a2a_gather_seq_scatter_heads(t, ctx) for t in (q, k, v))
        o = a2a_scatter_seq_gather_heads(sdpa_heads(q, k, v), ctx)
    else:
        o = sdpa_heads(q, k, v)
    o = linear(o, p.out.w, p.out.ws, p.out.b)
    if text is not None:
        qc = linear(h, p.cq.w, p.cq.ws, p.cq.b).view(s, H, Dh)
        kv = linear(text, p.ckv.w, p.ckv.ws, p.ckv.b)
        t = text.shape[0]
        oc = sdpa_heads(qc, kv[:, :D].view(t, H, Dh), kv[:, D:].view(t, H, Dh))
        o = o + linear(oc, p.cout.w, p.cout.ws, p.cout.b)
    h = gate_norm_mod_(x, o, ga, p.n2w, cfg.eps, ridx, s1m, shm)
    u = linear(h, p.up.w, p.up.ws, p.up.b)
    m = linear(F.gelu(u, approximate="tanh"), p.down.w, p.down.ws, p.down.b)
    gate_(x, m, gm, ridx)
    return x
