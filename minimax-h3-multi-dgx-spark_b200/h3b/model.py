"""Synthetic H3-style DiT block/step driving the hot path (the benchmark caller).

ComfyUI's MiniMax H3 model is not part of this project, so the benchmark
configurations use a random-init stand-in with the same block structure:

  fused DiTBlock.forward   comfyui_nodes/h3-fuse-graph/h3_fuse_patch.py:96-143
      h = norm_mod(x, w1, eps, ridx, s1a, sha)
      o = attention(h)                      sp_attention, sp_forward.py:276-318
      h = gate_norm_mod_(x, o, ga, w2, eps, ridx, s1m, shm)
      o = mlp(h)                            up INT8 linear -> GELU(tanh) -> down INT8 linear
      gate_(x, o, gm, ridx)
  (with FUSED_NORM_QUANT the norm kernels also quantise their output for the
  INT8 linear they feed; with FUSED_GELU_QUANT the GELU runs inside the down
  projection's quantiser)
  sp_attention: qkv INT8 linear -> Ulysses forward all-to-all (q, k, v) ->
      SDPA over [1, H/P, S, Dh] -> inverse all-to-all -> out INT8 linear.

Optional text cross-attention (the 40-block step configuration): a second,
row-local attention branch from the same modulated h to a replicated text
context (q / kv / out INT8 linears); its output is added to the self-attention
output before the gated residual, so the fused norm chain is unchanged and no
exchange is needed for it.  The reference model has no such branch in this
file set; the layout is this harness's choice.

HostPipeline runs host-resident latents through the model with the input and
output copies on their own streams, overlapping the previous and next steps'
copies with each step's compute.

Weights are int8 with per-output-channel fp32 scales and bf16 biases, drawn
from a seeded generator on the target device.  Attention stays PyTorch's
scaled_dot_product_attention, as in the reference.
"""
import os
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import fuse, sp
from .linear import gelu_quant as _gelu_quant
from .linear import gelu_tanh as _gelu
from .linear import int8_mm_scaled as _mm8
from .linear import linear as _linear8
from .linear import quant_rowwise as _quant
from .trace import span

BF16 = torch.bfloat16


@dataclass
class Linear8:
    w: torch.Tensor  # int8 [N, K]
    ws: torch.Tensor  # fp32 [N]
    b: torch.Tensor  # bf16 [N]

    @staticmethod
    def random(n, k, gen, device):
        w = torch.randint(-127, 128, (n, k), generator=gen, device=device, dtype=torch.int8)
        # per-channel scales sized so a unit-variance input gives an O(1) output
        ws = (torch.rand(n, generator=gen, device=device) + 0.5) / (127.0 * k ** 0.5)
        b = (torch.randn(n, generator=gen, device=device) * 0.02).to(BF16)
        return Linear8(w, ws, b)


@dataclass
class BlockParams:
    n1w: torch.Tensor
    n2w: torch.Tensor
    qkv: Linear8
    out: Linear8
    up: Linear8
    down: Linear8
    e: torch.Tensor  # bf16 [R, 6, D] adaLN conditioning (shift/scale/gate x 2)
    cq: Linear8 = None
    ckv: Linear8 = None
    cout: Linear8 = None
    qkn: torch.Tensor = None  # bf16 [2, head_dim]: q and k RMSNorm weights (qk_norm only)
    tables: tuple = field(default=None, repr=False)


@dataclass
class DiTConfig:
    dim: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    eps: float = 1e-6
    n_blocks: int = 1
    text_len: int = 0  # > 0 enables the cross-attention branch
    qk_norm: bool = False  # per-head RMSNorm of q and k (attn.q_norm / k_norm), no RoPE


def make_params(cfg, block_index, seed, device, R=1):
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + block_index)
    D = cfg.dim
    p = BlockParams(
        n1w=(1 + 0.02 * torch.randn(D, generator=g, device=device)).to(BF16),
        n2w=(1 + 0.02 * torch.randn(D, generator=g, device=device)).to(BF16),
        qkv=Linear8.random(3 * D, D, g, device),
        out=Linear8.random(D, D, g, device),
        up=Linear8.random(cfg.ffn, D, g, device),
        down=Linear8.random(D, cfg.ffn, g, device),
        e=(0.1 * torch.randn(R, 6, D, generator=g, device=device)).to(BF16),
    )
    if cfg.text_len:
        p.cq = Linear8.random(D, D, g, device)
        p.ckv = Linear8.random(2 * D, D, g, device)
        p.cout = Linear8.random(D, D, g, device)
    if cfg.qk_norm:
        p.qkn = (1 + 0.02 * torch.randn(2, cfg.head_dim, generator=g, device=device)).to(BF16)
    p.tables = fuse.modulation_tables(*(p.e[:, i] for i in range(6)))
    return p


def _lin(x, l):
    return _linear8(x, l.w, l.ws, l.b)


def _lin_q(q, l):
    """INT8 linear on already-quantised activations (codes, scales)."""
    xq, xs = q
    return _mm8(xq, l.w, xs, l.ws, bias=l.b)


def sdpa(q, k, v):
    """q [Sq, h, Dh], k/v [Sk, h, Dh] (any row strides) -> [Sq, h, Dh] (a strided view of
    SDPA's [1, h, Sq, Dh] output) via SDPA on [1, h, S, Dh] views (PyTorch's own
    kernel, as in the reference; traced as "sdpa" with its 4*Sq*Sk*h*Dh flops)."""
    sq, h, dh = q.shape
    with span("sdpa", 4.0 * sq * k.shape[0] * h * dh, launches=0):
        o = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0),
                                           v.transpose(0, 1).unsqueeze(0))
    return o.squeeze(0).transpose(0, 1)


def sdpa_heads(q, k, v):
    """q [Sq, h, Dh], k/v [Sk, h, Dh] (any row strides) -> [Sq, h*Dh] via SDPA on [1, h, S, Dh] views."""
    sq, h, dh = q.shape
    return sdpa(q, k, v).reshape(sq, h * dh)


def self_attention(cfg, p, hq, ctx, overlap_groups=None):
    """hq: the quantised block input (codes, scales) of the modulated h.

    overlap_groups: head groups of the exchange/attention overlap
    (sp.sp_attention_overlap, sp_forward.py:299-306); None reads the
    environment (sp.overlap_groups), 0 or 1 disables it."""
    s = hq[0].shape[0]
    D, H, Dh = cfg.dim, cfg.heads, cfg.head_dim
    sharded = ctx is not None and ctx.world > 1
    hp = H // ctx.world if sharded else H
    n = (sp.overlap_groups(hp, ctx.world) if overlap_groups is None else overlap_groups) if sharded else 0
    overlap = n > 1 and hp % n == 0
    if sharded and not overlap and sp._p2p(ctx) is not None and FUSED_EXCHANGE:
        # the qkv GEMM's epilogue (with the q/k norms when the block has them)
        # stores q, k, v straight into the owners' buffers; the out projection's
        # quantiser gathers its rows from every rank's output
        q, k, v = ctx.peer.gemm_fwd(hq[0], hq[1], p.qkv.w, p.qkv.ws, p.qkv.b, ctx,
                                    norm_w=p.qkn if cfg.qk_norm else None, norm_eps=cfg.eps)
        return _lin_q(ctx.peer.inv_quant(sdpa(q, k, v), ctx), p.out)
    qkv = _lin_q(hq, p.qkv)  # [s, 3D]
    q = qkv[:, :D].view(s, H, Dh)
    k = qkv[:, D:2 * D].view(s, H, Dh)
    v = qkv[:, 2 * D:].view(s, H, Dh)
    if cfg.qk_norm:
        q = fuse.rms_norm(q.contiguous(), p.qkn[0], cfg.eps)
        k = fuse.rms_norm(k.contiguous(), p.qkn[1], cfg.eps)
    if not sharded:
        return _lin(sdpa_heads(q, k, v), p.out)
    if overlap:
        return _lin(sp.sp_attention_overlap(q, k, v, ctx, sdpa_heads, n), p.out)
    q, k, v = sp.a2a_gather_qkv(q, k, v, ctx)  # [S, H/P, Dh] each
    o = sdpa_heads(q, k, v)  # [S, (H/P)*Dh]
    o = sp.a2a_scatter_seq_gather_heads(o, ctx)  # [s_local, D]
    return _lin(o, p.out)


def cross_attention(cfg, p, hq, text):
    s = hq[0].shape[0]
    D, H, Dh = cfg.dim, cfg.heads, cfg.head_dim
    q = _lin_q(hq, p.cq).view(s, H, Dh)
    kv = _lin(text, p.ckv)
    t = text.shape[0]
    k = kv[:, :D].view(t, H, Dh)
    v = kv[:, D:].view(t, H, Dh)
    return _lin(sdpa_heads(q, k, v), p.cout)


# With the peer-memory exchange the qkv projection's epilogue writes q, k and v
# straight into the receive buffers of the ranks owning their heads
# (PeerExchange.gemm_fwd) and the out projection's quantiser reads its rows
# from every rank's attention output (PeerExchange.inv_quant), so neither
# exchange needs a copy kernel.  H3B_FUSED_EXCHANGE=0 selects the separate
# exchange kernels.
FUSED_EXCHANGE = os.environ.get("H3B_FUSED_EXCHANGE", "1") != "0"

# The modulated activations feed only INT8 linears, so the norm kernels can emit
# their int8 codes and scales directly (norm_mod_quant / gate_norm_mod_quant_)
# and the GELU can run inside the down projection's quantiser (gelu_quant);
# results equal the unfused sequence bit for bit.  Each is switchable
# (H3B_FUSED_NORM_QUANT, H3B_FUSED_GELU_QUANT = 0 / 1); the defaults are the
# faster form as measured in the block.
FUSED_NORM_QUANT = os.environ.get("H3B_FUSED_NORM_QUANT", "0") == "1"
FUSED_GELU_QUANT = os.environ.get("H3B_FUSED_GELU_QUANT", "1") == "1"
# The GELU can instead run in the up projection's epilogue (the GEMM writes
# gelu(u), the plain quantiser follows); H3B_GELU_EPILOGUE=1 selects it and it
# takes precedence over FUSED_GELU_QUANT.
GELU_EPILOGUE = os.environ.get("H3B_GELU_EPILOGUE", "0") == "1"


def block_forward(cfg, p, x, ridx, ctx=None, text=None, fused_producers=None, overlap_groups=None):
    """One fused DiT block on the rank's rows x [s_local, D] (updated in place and returned)."""
    fused = FUSED_NORM_QUANT if fused_producers is None else fused_producers
    fused_gelu = FUSED_GELU_QUANT if fused_producers is None else fused_producers
    s1a, sha, ga, s1m, shm, gm = p.tables
    if fused:
        hq = fuse.norm_mod_quant(x, p.n1w, cfg.eps, ridx, s1a, sha)
    else:
        hq = _quant(fuse.norm_mod(x, p.n1w, cfg.eps, ridx, s1a, sha))
    o = self_attention(cfg, p, hq, ctx, overlap_groups)
    if text is not None:
        o = o + cross_attention(cfg, p, hq, text)
    del hq
    if fused:
        hq = fuse.gate_norm_mod_quant_(x, o, ga, p.n2w, cfg.eps, ridx, s1m, shm)
    else:
        hq = _quant(fuse.gate_norm_mod_(x, o, ga, p.n2w, cfg.eps, ridx, s1m, shm))
    del o
    if GELU_EPILOGUE and fused_producers is None:
        aq = _quant(_mm8(hq[0], p.up.w, hq[1], p.up.ws, bias=p.up.b, act="gelu"))
        del hq
    else:
        u = _lin_q(hq, p.up)
        del hq
        aq = _gelu_quant(u) if fused_gelu else _quant(_gelu(u))
        del u
    m = _lin_q(aq, p.down)
    del aq
    fuse.gate_(x, m, gm, ridx)
    return x


class SynthDiT:
    """n_blocks random-init blocks; forward runs them in order on the rank's rows."""

    def __init__(self, cfg, device, seed=0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.params = [make_params(cfg, i, seed, self.device) for i in range(cfg.n_blocks)]

    def forward(self, x, ridx, ctx=None, text=None):
        for p in self.params:
            x = block_forward(self.cfg, p, x, ridx, ctx, text)
        return x


class HostPipeline:
    """Host-resident latents through a model, with the copies off the compute stream.

    submit(x_host, out_host) runs one step: the rows x_host [rows, D] (pinned
    bf16) are copied to the device on an input copy stream, `model.forward`
    runs on the current stream, and the result is copied into out_host (pinned)
    on an output copy stream.  Up to `depth` steps are in flight on `depth`
    device slots, so the input copy of step k+1 and the output copy of step
    k-1 run during step k's compute; a slot is refilled only after its previous
    output copy has finished.  flush() makes the current stream wait for every
    copy issued so far: out_host of a submitted step is valid once the current
    stream has passed that point (e.g. after flush() and a synchronize).
    `before` (optional) is called on the current stream before each forward,
    for per-step device inputs such as the modulation tables.  With
    timing=True the copies are bracketed by CUDA events on their streams and
    copy_times() returns their mean durations."""

    def __init__(self, model, rows, ridx, ctx=None, text=None, depth=3, timing=False):
        self.model, self.ridx, self.ctx, self.text = model, ridx, ctx, text
        dev = model.device
        self.device = dev
        self.slots = [torch.empty(rows, model.cfg.dim, dtype=torch.bfloat16, device=dev) for _ in range(depth)]
        self.freed = [None] * depth
        self.copy_in = torch.cuda.Stream(device=dev)
        self.copy_out = torch.cuda.Stream(device=dev)
        self.k = 0
        self.timing = timing
        self._ev = {"in": [], "out": []}
        self.cond_slots = [None] * depth  # per-slot device copies of the step's conditioning

    def _timed_copy(self, kind, stream, dst, src):
        if not self.timing:
            dst.copy_(src, non_blocking=True)
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dst.copy_(src, non_blocking=True)
        e1.record(stream)
        self._ev[kind].append((e0, e1))

    def copy_times(self):
        """{"in": mean ms, "out": mean ms} of the timed copies so far (synchronises)."""
        torch.cuda.synchronize(self.device)
        return {k: (sum(a.elapsed_time(b) for a, b in v) / len(v) if v else None) for k, v in self._ev.items()}

    def submit(self, x_host, out_host, before=None, cond_host=None):
        """One step.  cond_host (optional): pinned host tensors of per-step
        conditioning (e.g. the adaLN vectors); they are copied on the input copy
        stream into this slot's own device buffers, like x, and `before` is then
        called with the device copies (before(cond_dev)), so the compute stream
        issues no host copy that could queue behind another step's input copy."""
        i = self.k % len(self.slots)
        slot = self.slots[i]
        cur = torch.cuda.current_stream(self.device)
        cond_dev = None
        with torch.cuda.stream(self.copy_in):
            if self.freed[i] is not None:
                self.copy_in.wait_event(self.freed[i])
            self._timed_copy("in", self.copy_in, slot, x_host)
            if cond_host is not None:
                have = self.cond_slots[i]
                if have is None or len(have) != len(cond_host) or any(
                        d.shape != c.shape or d.dtype != c.dtype for d, c in zip(have, cond_host)):
                    # first use of the slot, or conditioning of another shape: its own device buffers
                    self.cond_slots[i] = [torch.empty(c.shape, dtype=c.dtype, device=self.device) for c in cond_host]
                cond_dev = self.cond_slots[i]
                for d, c in zip(cond_dev, cond_host):
                    d.copy_(c, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(self.copy_in)
        cur.wait_event(ready)
        if before is not None:
            before() if cond_host is None else before(cond_dev)
        y = self.model.forward(slot, self.ridx, self.ctx, self.text)
        done = torch.cuda.Event()
        done.record(cur)
        self.copy_out.wait_event(done)
        with torch.cuda.stream(self.copy_out):
            self._timed_copy("out", self.copy_out, out_host, y)
            freed = torch.cuda.Event()
            freed.record(self.copy_out)
        self.freed[i] = freed
        self.k += 1

    def flush(self):
        cur = torch.cuda.current_stream(self.device)
        cur.wait_stream(self.copy_in)
        cur.wait_stream(self.copy_out)
