"""Ulysses sequence<->head all-to-all for the H3 DiT block (host side).

Mirrors comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:
  SPContext                                 :140-155  (uneven base+rem row splits, no padding)
  _seq_gather / _seq_scatter                :158-176  (the exchange)
  a2a_gather_seq_scatter_heads(t, ctx)      :179-188  [s_local, H, D] -> [S, H/P, D]
  a2a_scatter_seq_gather_heads(t, ctx)      :191-198  [S, (H/P)*D] -> [s_local, H*D]
  sp_attention_overlap(q, k, v, ctx, ...)   :211-261  exchange/attention overlap by head groups
  overlap_groups(hp, world)                 :58,264-273
  gather_rows(local, counts, ctx, out_dim)  :378-389  padded all-gather of the final rows
and the known-answer start-up probe of sp_group.py:107-128 (for the NCCL group
and, given a PeerExchange, for the peer-memory back end).

Two exchange back ends, chosen per SPContext (`ctx.exchange`):
  * "nccl": pack kernel -> grouped NCCL send/recv (torch.distributed
    all_to_all_single on the tensor process group) -> unpack kernel.
  * "p2p": one kernel per direction that reads local rows and stores them
    straight into the destination rank's buffer over NVLink (CUDA IPC
    mappings), bracketed by flag barriers in peer memory.  Receive buffers
    are persistent and owned by the PeerExchange: a tensor returned by an
    exchange stays valid until the next exchange in the same direction.
The reference's 4-node ring relay (ring_a2a.py) has no counterpart: on
NVSwitch every rank reaches every other directly.
"""
import ctypes
import os

import torch
import torch.distributed as dist

from ._lib import check, lib, ptr, ptr_array, require_cuda, stream_of
from .trace import span


class SPContext:
    """Row-sharding descriptor for one forward pass (sp_forward.py:140-155)."""

    def __init__(self, rank, world, group, seq_len, exchange="nccl", peer=None):
        self.rank = rank
        self.world = world
        self.group = group
        self.seq_len = seq_len
        base, rem = divmod(seq_len, world)
        self.splits = [base + (1 if r < rem else 0) for r in range(world)]
        self.start = sum(self.splits[: rank])
        self.stop = self.start + self.splits[rank]
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"unknown exchange back end {exchange!r}")
        if exchange == "p2p" and peer is None:
            raise ValueError("the p2p exchange needs a PeerExchange")
        self.exchange = exchange
        self.peer = peer

    @property
    def local(self):
        return self.splits[self.rank]


def _p2p(ctx):
    """The PeerExchange of ctx when it selects the peer-memory back end, else None.
    A context without these attributes (the reference's own SPContext,
    sp_forward.py:140-155, passed by a patched caller) uses NCCL."""
    return ctx.peer if getattr(ctx, "exchange", "nccl") == "p2p" else None


# ---------------------------------------------------------------------------
# NCCL back end (pure torch.distributed; also runs on gloo/CPU for host tests)

def _seq_gather(out, send, ctx, width, async_op=False):
    """Every rank sends its rows (width elements each) to all and receives all rows."""
    return dist.all_to_all_single(out, send, output_split_sizes=[n * width for n in ctx.splits],
                                  input_split_sizes=[ctx.local * width] * ctx.world,
                                  group=ctx.group, async_op=async_op)


def _seq_scatter(out, send, ctx, width, async_op=False):
    """Inverse of _seq_gather: the holder of all rows hands each rank its rows."""
    return dist.all_to_all_single(out, send, output_split_sizes=[ctx.local * width] * ctx.world,
                                  input_split_sizes=[n * width for n in ctx.splits],
                                  group=ctx.group, async_op=async_op)


def _rows(t):
    """View t as [rows, row_elems] with unit element stride inside a row; returns (t2d, row stride)."""
    t2 = t.reshape(t.shape[0], -1) if t.dim() != 2 else t
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2, t2.stride(0)


def pack(t, world, width=None, block=None):
    """[s_local, P*chunk] (rows may be strided) -> [P, s_local, chunk] with the pack kernel.

    With width/block (elements): rows hold one block of `block` elements per
    rank and the first `width` of each go out (t already offset to the head
    group's first column; send is [P, s_local, width])."""
    require_cuda(t)
    if width is None:
        t2, ld = _rows(t)
        s_local, row_elems = t2.shape
        if row_elems % world:
            raise ValueError("pack: the row does not split into world chunks")
        width = block = row_elems // world
    else:
        t2, ld = t, t.stride(0)
        s_local = t.shape[0]
        if t.stride(-1) != 1 or width > block or (world - 1) * block + width > t.shape[1]:
            raise ValueError("pack: the group does not fit the row")
    send = torch.empty((world, s_local, width), dtype=t.dtype, device=t.device)
    es = t.element_size()
    with span("a2a_pack", 2 * s_local * world * width * es):
        check(lib.h3b_a2a_pack(ptr(t2), ld * es, ptr(send), s_local, width * es, block * es, world, stream_of(t)),
              "h3b_a2a_pack")
    return send


def unpack(recv, out=None, block=None):
    """[P, s_local, chunk] -> [s_local, P*chunk] with the unpack kernel.

    With out/block: rank j's chunk of row s lands at column j*block of `out`
    (a view offset to the head group's first column, unit column stride)."""
    require_cuda(recv)
    world, s_local, chunk = recv.shape
    recv = recv.contiguous()
    if out is None:
        out = torch.empty((s_local, world * chunk), dtype=recv.dtype, device=recv.device)
        block = chunk
    elif out.stride(-1) != 1 or out.shape[0] != s_local or chunk > block:
        raise ValueError("unpack: out does not match recv")
    es = recv.element_size()
    with span("a2a_unpack", 2 * recv.numel() * es):
        check(lib.h3b_a2a_unpack(ptr(recv), ptr(out), out.stride(0) * es, s_local, chunk * es, block * es, world,
                                 stream_of(recv)), "h3b_a2a_unpack")
    return out


def a2a_gather_seq_scatter_heads(t, ctx):
    """[s_local, H, D] -> [S_total, H/P, D]."""
    s_local, heads, dim = t.shape
    hp = heads // ctx.world
    if _p2p(ctx):
        return ctx.peer.fwd([t], ctx)[0]
    send = pack(t, ctx.world).view(-1)
    out = torch.empty(ctx.seq_len * hp * dim, dtype=t.dtype, device=t.device)
    _seq_gather(out, send, ctx, hp * dim)
    return out.view(ctx.seq_len, hp, dim)


def a2a_gather_qkv(q, k, v, ctx):
    """The three forward exchanges of one attention call at once: one p2p
    launch, or on NCCL three pack launches and three asynchronous
    all_to_all_single calls.  (One group of point-to-point sends/receives for
    all three tensors, batch_isend_irecv, measured 149 GB/s bus at P=2 against
    341 GB/s for the all_to_all_single calls, and was dropped.)"""
    if _p2p(ctx):
        return ctx.peer.fwd([q, k, v], ctx)
    s_local, heads, dim = q.shape
    hp = heads // ctx.world
    outs, reqs = [], []
    for t in (q, k, v):
        send = pack(t, ctx.world).view(-1)
        out = torch.empty(ctx.seq_len * hp * dim, dtype=t.dtype, device=t.device)
        reqs.append((_seq_gather(out, send, ctx, hp * dim, async_op=True), send))
        outs.append(out.view(ctx.seq_len, hp, dim))
    for work, _ in reqs:
        work.wait()
    return outs


def a2a_scatter_seq_gather_heads(t, ctx):
    """[S_total, (H/P)*D] -> [s_local, H*D]."""
    if _p2p(ctx):
        return ctx.peer.inv(t, ctx)
    chunk = t.shape[1]
    out = torch.empty(ctx.world * ctx.local * chunk, dtype=t.dtype, device=t.device)
    _seq_scatter(out, t.contiguous().view(-1), ctx, chunk)
    return unpack(out.view(ctx.world, ctx.local, chunk))


def overlap_groups(hp, world):
    """Number of head groups for the exchange/attention overlap (sp_forward.py:58,264-273).

    H3B_SP_OVERLAP_GROUPS, else the reference's MINIMAX_SP_OVERLAP_CHUNKS (0 or
    1: no overlap).  At world 4 MINIMAX_SP_OVERLAP_CHUNKS_W4 takes precedence and
    the count is lowered to the largest divisor of hp not above it, as in the
    reference.  Every rank must see the same value."""
    def env(name):
        return int(os.environ.get(name, "0") or 0)
    n = env("H3B_SP_OVERLAP_GROUPS") or env("MINIMAX_SP_OVERLAP_CHUNKS")
    if world == 4:
        n = env("MINIMAX_SP_OVERLAP_CHUNKS_W4") or n
        while n > 1 and hp % n:
            n -= 1
    return n


def sp_attention_overlap(q, k, v, ctx, attn, groups):
    """Exchange/attention overlap by head groups (sp_forward.py:211-261).

    q, k, v [s_local, H, Dh] (any row stride) -> [s_local, H*Dh].  The H/P heads
    a rank receives are split into `groups` groups of hc heads; group g's forward
    exchange (the hc heads j*hp + g*hc .. of every destination rank j), its
    attention `attn(q_g, k_g, v_g)` ([S, hc, Dh] each -> [S, hc*Dh]) and its
    inverse exchange are pipelined, so group g+1's transfer runs during group
    g's attention.  Each head is computed exactly as without the overlap, so
    the result is identical."""
    s_local, heads, dim = q.shape
    hp = heads // ctx.world
    if groups < 1 or hp % groups:
        raise ValueError(f"{groups} groups do not divide the {hp} heads of a rank")
    if _p2p(ctx):
        return ctx.peer.attention_overlap(q, k, v, ctx, attn, groups)
    P, hc = ctx.world, hp // groups
    w = hc * dim
    pending = []
    keep = []  # send/receive tensors of collectives still in flight
    for g in range(groups):
        trio = []
        for t in (q, k, v):
            t2, _ = _rows(t)
            send = pack(t2[:, g * w:], P, width=w, block=hp * dim)
            recv = torch.empty(ctx.seq_len * w, dtype=t.dtype, device=t.device)
            trio.append((recv, _seq_gather(recv, send.view(-1), ctx, w, async_op=True)))
            keep.append(send)
        pending.append(trio)
    final = torch.empty(s_local, heads * dim, dtype=q.dtype, device=q.device)
    outs = []
    for g in range(groups):
        parts = []
        for recv, work in pending[g]:
            work.wait()
            parts.append(recv.view(ctx.seq_len, hc, dim))
        o = attn(*parts).contiguous()
        ob = torch.empty(P * s_local * w, dtype=o.dtype, device=o.device)
        outs.append((g, ob, _seq_scatter(ob, o.view(-1), ctx, w, async_op=True)))
        keep.append(o)
    for g, ob, work in outs:
        work.wait()
        unpack(ob.view(P, s_local, w), out=final[:, g * w:], block=hp * dim)
    del keep
    return final


# ---------------------------------------------------------------------------
# Peer-memory back end

class PeerExchange:
    """Persistent IPC-mapped buffers and flags for the fused p2p all-to-all.

    Collective to construct (every rank of `group` calls it with the same
    arguments) and to `close()`.  Buffers: two sets of n_fwd receive buffers
    of [seq_len, chunk], one inverse output buffer of [max_local, world*chunk],
    one attention output buffer of [seq_len, chunk] that the peers read
    (inv_quant) (chunk = heads/world * head_dim elements), plus a uint32
    [world] flag array.

    Barriers.  The block's exchange pair -- gemm_fwd (the qkv projection
    storing into the owners' receive buffers) then inv_quant (the out
    projection's quantiser gathering every rank's attention output) -- needs
    two flag barriers per attention when it repeats: gemm_fwd alternates
    between the two receive sets, so when it directly follows an inv_quant
    it skips its entry barrier.  That is safe because a peer starts the next
    gemm_fwd only after passing the inv_quant barrier, which every rank
    reaches after its attention read the receive set written two exchanges
    back; and a rank refills its attention output buffer only after the next
    gemm_fwd's exit barrier, which every peer reaches after its gather of that
    buffer.  Any other call sequence (fwd, inv, the overlap, a first call)
    takes the entry barriers.
    """

    def __init__(self, group, rank, world, seq_len, heads, head_dim, dtype=torch.bfloat16, n_fwd=3,
                 timeout_s=None):
        if heads % world:
            raise ValueError(f"{heads} heads do not split over {world} ranks")
        self.group, self.rank, self.world = group, rank, world
        self.seq_len, self.heads, self.head_dim = seq_len, heads, head_dim
        self.chunk = heads // world * head_dim
        self.dtype = dtype
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        max_local = -(-seq_len // world)
        timeout_s = float(os.environ.get("H3B_PEER_TIMEOUT_S", "30")) if timeout_s is None else timeout_s
        self.timeout_ns = int(timeout_s * 1e9)
        self.recv_sets = [[torch.empty((seq_len, self.chunk), dtype=dtype, device=dev) for _ in range(n_fwd)]
                          for _ in range(2)]
        self.recv = self.recv_sets[0]  # the set fwd() and the overlap use
        self.out = torch.empty((max_local, world * self.chunk), dtype=dtype, device=dev)
        self.obuf = torch.empty((seq_len, self.chunk), dtype=dtype, device=dev)  # attention output, pulled by peers
        self.flags = torch.zeros(world, dtype=torch.int32, device=dev)
        self.epoch = 0
        self.n_gemm_fwd = 0  # gemm_fwd calls so far: call k uses receive set k % 2
        self._last = None  # "gemm_fwd" / "inv_quant" when the last call was one of the chained pair
        self.comm = None  # side stream of the exchange/attention overlap
        self._bases = []
        shared = self.recv_sets[0] + self.recv_sets[1] + [self.out, self.obuf, self.flags]
        mine = [self._handle(t) for t in shared]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine, group=group)
        peer = [[None] * world for _ in shared]  # peer[buffer][rank] = address in this process
        for j in range(world):
            for idx, (hb, off) in enumerate(gathered[j]):
                peer[idx][j] = shared[idx].data_ptr() if j == rank else self._open(hb, off)
        self.peer_recv_sets = [peer[:n_fwd], peer[n_fwd:2 * n_fwd]]
        self.peer_recv = self.peer_recv_sets[0]
        self.peer_out, self.peer_obuf, self.peer_flags = peer[2 * n_fwd], peer[2 * n_fwd + 1], peer[2 * n_fwd + 2]
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    @staticmethod
    def _handle(t):
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        check(lib.h3b_ipc_handle(ptr(t), h, ctypes.byref(off)), "h3b_ipc_handle")
        return h.raw, off.value

    def _open(self, hb, off):
        p, base = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib.h3b_ipc_open(hb, off, ctypes.byref(p), ctypes.byref(base)), "h3b_ipc_open")
        self._bases.append(base.value)
        return p.value

    def barrier(self, stream_tensor):
        self.epoch += 1
        arr, keep = ptr_array(self.peer_flags)
        with span("peer_barrier", 0):
            check(lib.h3b_peer_barrier(arr, self.world, self.rank, self.epoch, self.timeout_ns,
                                       stream_of(stream_tensor)), "h3b_peer_barrier")
        del keep

    def _group(self, groups):
        """(width in elements, hc) of one of `groups` head groups of a rank's chunk."""
        hp = self.heads // self.world
        if groups < 1 or hp % groups:
            raise ValueError(f"{groups} groups do not divide the {hp} heads of a rank")
        return self.chunk // groups, hp // groups

    def recv_views(self, n, ctx, g=0, groups=1, rset=0):
        """Views [S, hc, Dh] of head group g in the first n receive buffers of set
        rset.  Group g of width w occupies elements [g*seq_len*w, (g+1)*seq_len*w)
        of a buffer."""
        w, hc = self._group(groups)
        base = g * self.seq_len * w
        return [self.recv_sets[rset][i].view(-1)[base: base + ctx.seq_len * w].view(ctx.seq_len, hc, self.head_dim)
                for i in range(n)]

    def fwd_copy(self, tensors, ctx, g=0, groups=1):
        """Store head group g of this rank's rows of each tensor into every rank's
        receive buffers (no barrier: the caller brackets it)."""
        n = len(tensors)
        if n > len(self.recv):
            raise ValueError("more tensors than receive buffers")
        s_local, heads, dim = tensors[0].shape
        if heads != self.heads or dim != self.head_dim or ctx.seq_len > self.seq_len:
            raise ValueError("tensor shape does not match the PeerExchange buffers")
        srcs = [_rows(t) for t in tensors]
        ld = srcs[0][1]
        if any(s[1] != ld for s in srcs):
            srcs = [(t.contiguous(), t[0].numel()) for t, _ in srcs]
            ld = srcs[0][1]
        srcs = [t for t, _ in srcs]
        for t in srcs:
            require_cuda(t)
            if t.dtype != self.dtype or t.shape != srcs[0].shape:
                raise ValueError("all tensors must share shape and dtype")
        es = srcs[0].element_size()
        w, _ = self._group(groups)
        base = g * self.seq_len * w * es
        src_arr, k1 = ptr_array([t.data_ptr() for t in srcs])
        dst_arr, k2 = ptr_array([self.peer_recv[i][j] + base for i in range(n) for j in range(self.world)])
        off_rank = n * s_local * w * es * (self.world - 1)
        with span("a2a_fwd_p2p", off_rank):
            check(lib.h3b_a2a_fwd_p2p(n, src_arr, ld * es, dst_arr, s_local, ctx.start, w * es, self.chunk * es,
                                      g * w * es, self.world, stream_of(srcs[0])), "h3b_a2a_fwd_p2p")
        del k1, k2

    def gemm_fwd(self, xq, xs, w, ws, bias, ctx, norm_w=None, norm_eps=1e-6):
        """A projection fused with the forward exchange (h3b_int8_mm_scaled_a2a):
        the [s_local, n*H*Dh] product of the quantised rows (xq, xs) and w
        (n = 1..3 segments, e.g. the fused q|k|v projection) is stored by the
        GEMM's epilogue straight into every rank's receive buffers; with norm_w
        (bf16 [2, 128]) q and k get their per-head RMSNorm in the same epilogue.
        Returns the n views [S, H/P, Dh] of this rank's receive buffers."""
        from .linear import int8_mm_scaled_a2a
        D = self.heads * self.head_dim
        nseg = w.shape[0] // D
        if w.shape[0] != nseg * D or not 1 <= nseg <= len(self.recv) or ctx.seq_len > self.seq_len:
            raise ValueError("gemm_fwd: the projection does not match the PeerExchange buffers")
        if xq.shape[0] != ctx.local:
            raise ValueError("gemm_fwd: xq must hold this rank's rows")
        rset = self.n_gemm_fwd % 2
        dst = [self.peer_recv_sets[rset][t][j] for t in range(nseg) for j in range(self.world)]
        if self._last != "inv_quant":
            self.barrier(xq)  # entry: every rank's receive set is free (not needed in the chained pair)
        int8_mm_scaled_a2a(xq, w, xs, ws, bias, dst, ctx.start, D, self.head_dim, self.heads // self.world,
                           self.world, norm_w=norm_w, norm_eps=norm_eps)
        self.barrier(xq)  # exit: every rank's rows have arrived
        self.n_gemm_fwd += 1
        self._last = "gemm_fwd"
        return self.recv_views(nseg, ctx, rset=rset)

    def fwd(self, tensors, ctx):
        """tensors: n x [s_local, H, D] -> n views [S, H/P, D] of the receive buffers."""
        self._last = None
        self.barrier(tensors[0])
        self.fwd_copy(tensors, ctx)
        self.barrier(tensors[0])
        return self.recv_views(len(tensors), ctx)

    def inv_copy(self, t, ctx, g=0, groups=1):
        """Store t [S, w] (head group g of this rank's heads, unit column stride)
        into every rank's output buffer (no barrier: the caller brackets it)."""
        require_cuda(t)
        w, _ = self._group(groups)
        if t.dim() != 2 or t.shape[1] != w or t.stride(1) != 1 or t.dtype != self.dtype:
            raise ValueError("inv: t must be [S, width] with unit column stride")
        es = t.element_size()
        dst_arr, k1 = ptr_array(self.peer_out)
        splits = (ctypes.c_int64 * self.world)(*ctx.splits)
        off_rank = (ctx.seq_len - ctx.local) * w * es
        with span("a2a_inv_p2p", off_rank):
            check(lib.h3b_a2a_inv_p2p(ptr(t), t.stride(0) * es, dst_arr, splits, w * es, self.world * self.chunk * es,
                                      (self.rank * self.chunk + g * w) * es, self.world, stream_of(t)),
                  "h3b_a2a_inv_p2p")
        del k1

    def inv(self, t, ctx):
        """t [S, (H/P)*D] (unit stride along the row) -> [s_local, H*D] view of the output buffer."""
        self._last = None
        self.barrier(t)
        self.inv_copy(t, ctx)
        self.barrier(t)
        return self.out[: ctx.local]

    def inv_quant(self, o, ctx):
        """Inverse exchange fused with the out projection's quantiser.

        o: this rank's attention output [S, H/P, Dh] or [S, (H/P)*Dh] (any
        strides).  It is copied into this rank's shared output buffer; after a
        barrier every rank quantises its own rows, each gathered from all ranks'
        buffers over NVLink (h3b_a2a_inv_quant).  Returns (codes [s_local, H*Dh]
        int8, scales [s_local, 1] fp32), equal to quant_rowwise of the row the
        inverse exchange delivers.  The shared buffer is reused by the next call:
        every rank's gather of it precedes that rank's arrival at the next
        exchange's first barrier, which precedes the next copy into it."""
        require_cuda(o)
        S, hp = ctx.seq_len, self.heads // self.world
        if S > self.seq_len:
            raise ValueError("inv_quant: sequence longer than the PeerExchange buffers")
        if self._last != "gemm_fwd":
            self.barrier(o)  # the peers' gathers of the previous contents are done
        self.obuf[:S].view(S, hp, self.head_dim).copy_(o.reshape(S, hp, self.head_dim))
        self.barrier(o)
        K = self.heads * self.head_dim
        xq = torch.empty((ctx.local, K), dtype=torch.int8, device=o.device)
        xs = torch.empty((ctx.local, 1), dtype=torch.float32, device=o.device)
        es = self.obuf.element_size()
        arr, keep = ptr_array(self.peer_obuf)
        with span("quant_a2a", ctx.local * K * (es + 1) + 4 * ctx.local):
            check(lib.h3b_a2a_inv_quant(arr, self.chunk * es, ctx.start, ctx.local, self.chunk * es, self.world,
                                        ptr(xq), ptr(xs), stream_of(o)), "h3b_a2a_inv_quant")
        del keep
        self._last = "inv_quant"
        return xq, xs

    def attention_overlap(self, q, k, v, ctx, attn, groups):
        """sp_attention_overlap over peer memory.  The exchanges run on a
        high-priority side stream: one barrier (every rank's receive and output
        buffers are free: each rank's previous readers of them precede its
        arrival), then per group a copy and a barrier (group g has arrived
        everywhere); the attention of group g waits for that, and its inverse
        copy waits for the attention.  One last barrier: every rank's output
        buffer is complete.  Returns [s_local, H*D], a view of the output buffer."""
        self._last = None
        cur = torch.cuda.current_stream(q.device)
        if self.comm is None:
            self.comm = torch.cuda.Stream(device=q.device, priority=-100)
        comm = self.comm
        comm.wait_stream(cur)
        arrived = []
        with torch.cuda.stream(comm):
            self.barrier(q)
            for g in range(groups):
                self.fwd_copy([q, k, v], ctx, g, groups)
                self.barrier(q)
                ev = torch.cuda.Event()
                ev.record(comm)
                arrived.append(ev)
        keep = []  # attention outputs read by the side stream until it is joined
        for g in range(groups):
            cur.wait_event(arrived[g])
            o = attn(*self.recv_views(3, ctx, g, groups))
            keep.append(o)
            comm.wait_stream(cur)
            with torch.cuda.stream(comm):
                self.inv_copy(o, ctx, g, groups)
        with torch.cuda.stream(comm):
            self.barrier(q)
        cur.wait_stream(comm)
        del keep
        return self.out[: ctx.local]

    def close(self):
        torch.cuda.synchronize(self.device)
        for b in self._bases:
            check(lib.h3b_ipc_close(ctypes.c_void_p(b)), "h3b_ipc_close")
        self._bases = []


def gather_rows(local, counts, ctx, out_dim, device=None):
    """Every rank's row block, concatenated in rank order on every rank
    (sp_forward.py:378-389): blocks of counts[r] rows (possibly 0) of out_dim
    fp32 columns are padded to max(counts) rows for one all-gather, then the
    padding is dropped.  local: this rank's [counts[rank], out_dim] or None
    (then `device` names the device of the buffers)."""
    maxn = max(counts)
    dev = local.device if local is not None else (device or torch.device("cuda", torch.cuda.current_device()))
    buf = torch.zeros(maxn, out_dim, dtype=torch.float32, device=dev)
    if local is not None and local.shape[0]:
        buf[:local.shape[0]] = local
    gathered = torch.empty(ctx.world * maxn, out_dim, dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(gathered, buf, group=ctx.group)
    gathered = gathered.view(ctx.world, maxn, out_dim)
    return torch.cat([gathered[r, :counts[r]] for r in range(ctx.world) if counts[r] > 0], dim=0)


# ---------------------------------------------------------------------------

def startup_probe(rank, world, group, device, peer=None):
    """Known-answer check of the tensor process group (sp_group.py:107-128):
    all_reduce of rank+1 sums to P(P+1)/2 and all_to_all_single of
    arange(P) + rank*P returns arange(P)*P + rank.  With `peer` (a
    PeerExchange) the peer-memory back end is checked the same way
    (probe_peer).  Collective: every rank of the group calls it."""
    reduced = torch.tensor([rank + 1], dtype=torch.float32, device=device)
    dist.all_reduce(reduced, group=group)
    expected_sum = world * (world + 1) / 2
    if reduced.item() != expected_sum:
        raise RuntimeError(f"all_reduce returned {reduced.item()}, expected {expected_sum}")
    source = torch.arange(world, dtype=torch.int64, device=device) + rank * world
    received = torch.empty_like(source)
    dist.all_to_all_single(received, source, group=group)
    expected = torch.arange(world, dtype=torch.int64, device=device) * world + rank
    if not torch.equal(received, expected):
        raise RuntimeError(f"all_to_all_single returned {received.tolist()}, expected {expected.tolist()}")
    if peer is not None:
        probe_peer(peer, rank, world, group, device)


def _probe_values(rows, cols):
    """(row * 7 + column) % 251: integers below 256, exact in bf16."""
    return ((rows[:, None] * 7 + cols[None, :]) % 251).to(torch.bfloat16)


def probe_peer(peer, rank, world, group, device):
    """Known-answer round trip through the peer-memory back end, the p2p
    counterpart of the reference's start-up probe: each rank's rows of an
    [S, H, Dh] tensor of known values (S uneven over the ranks when the
    buffers allow) go through the forward exchange -- every rank must receive
    its heads of every row -- and the received rows back through the inverse
    -- every rank must get its own rows.  A mismatch on any rank raises on
    every rank (the verdict is all-reduced).  Collective."""
    H, Dh = peer.heads, peer.head_dim
    S = min(peer.seq_len, 16 * world + world - 1)
    ctx = SPContext(rank, world, group, S, exchange="p2p", peer=peer)
    cols = torch.arange(H * Dh, device=device, dtype=torch.int64)
    t = _probe_values(torch.arange(ctx.start, ctx.stop, device=device, dtype=torch.int64), cols).view(-1, H, Dh)
    got = peer.fwd([t], ctx)[0].reshape(S, -1)
    hp = H // world
    want = _probe_values(torch.arange(S, device=device, dtype=torch.int64), cols[rank * hp * Dh:(rank + 1) * hp * Dh])
    ok = torch.equal(got, want)
    back = peer.inv(got, ctx)
    ok = ok and torch.equal(back.reshape(ctx.local, -1), t.reshape(ctx.local, -1))
    bad = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
    dist.all_reduce(bad, group=group)
    if bad.item():
        raise RuntimeError(f"peer-memory exchange probe failed on {bad.item()} of {world} ranks")
