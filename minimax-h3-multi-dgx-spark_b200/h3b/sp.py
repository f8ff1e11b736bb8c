"""Ulysses sequence<->head all-to-all for the H3 DiT block (host side).

Mirrors comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py:
  SPContext                                 :140-155  (uneven base+rem row splits, no padding)
  _seq_gather / _seq_scatter                :158-176  (the exchange)
  a2a_gather_seq_scatter_heads(t, ctx)      :179-188  [s_local, H, D] -> [S, H/P, D]
  a2a_scatter_seq_gather_heads(t, ctx)      :191-198  [S, (H/P)*D] -> [s_local, H*D]
and the known-answer start-up probe of sp_group.py:107-128.

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


def pack(t, world):
    """[s_local, P*chunk] (rows may be strided) -> [P, s_local, chunk] with the pack kernel."""
    require_cuda(t)
    t2, ld = _rows(t)
    s_local, row_elems = t2.shape
    if row_elems % world:
        raise ValueError("pack: the row does not split into world chunks")
    chunk = row_elems // world
    send = torch.empty((world, s_local, chunk), dtype=t.dtype, device=t.device)
    es = t.element_size()
    with span("a2a_pack", 2 * s_local * row_elems * es):
        check(lib.h3b_a2a_pack(ptr(t2), ld * es, ptr(send), s_local, chunk * es, world, stream_of(t)), "h3b_a2a_pack")
    return send


def unpack(recv):
    """[P, s_local, chunk] -> [s_local, P*chunk] with the unpack kernel."""
    require_cuda(recv)
    world, s_local, chunk = recv.shape
    recv = recv.contiguous()
    out = torch.empty((s_local, world * chunk), dtype=recv.dtype, device=recv.device)
    with span("a2a_unpack", 2 * recv.numel() * recv.element_size()):
        check(lib.h3b_a2a_unpack(ptr(recv), ptr(out), s_local, chunk * recv.element_size(), world, stream_of(recv)),
              "h3b_a2a_unpack")
    return out


def a2a_gather_seq_scatter_heads(t, ctx):
    """[s_local, H, D] -> [S_total, H/P, D]."""
    s_local, heads, dim = t.shape
    hp = heads // ctx.world
    if ctx.exchange == "p2p":
        return ctx.peer.fwd([t], ctx)[0]
    send = pack(t, ctx.world).view(-1)
    out = torch.empty(ctx.seq_len * hp * dim, dtype=t.dtype, device=t.device)
    _seq_gather(out, send, ctx, hp * dim)
    return out.view(ctx.seq_len, hp, dim)


def a2a_gather_qkv(q, k, v, ctx):
    """The three forward exchanges of one attention call at once (one launch /
    one NCCL group instead of three)."""
    if ctx.exchange == "p2p":
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
    if ctx.exchange == "p2p":
        return ctx.peer.inv(t, ctx)
    chunk = t.shape[1]
    out = torch.empty(ctx.world * ctx.local * chunk, dtype=t.dtype, device=t.device)
    _seq_scatter(out, t.contiguous().view(-1), ctx, chunk)
    return unpack(out.view(ctx.world, ctx.local, chunk))


# ---------------------------------------------------------------------------
# Peer-memory back end

class PeerExchange:
    """Persistent IPC-mapped buffers and flags for the fused p2p all-to-all.

    Collective to construct (every rank of `group` calls it with the same
    arguments) and to `close()`.  Buffers: n_fwd receive buffers of
    [seq_len, chunk] and one inverse output buffer of [max_local, world*chunk]
    (chunk = heads/world * head_dim elements), plus a uint32 [world] flag array.
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
        self.recv = [torch.empty((seq_len, self.chunk), dtype=dtype, device=dev) for _ in range(n_fwd)]
        self.out = torch.empty((max_local, world * self.chunk), dtype=dtype, device=dev)
        self.flags = torch.zeros(world, dtype=torch.int32, device=dev)
        self.epoch = 0
        self._bases = []
        mine = [self._handle(t) for t in self.recv + [self.out, self.flags]]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine, group=group)
        self.peer_recv = [[None] * world for _ in range(n_fwd)]
        self.peer_out = [None] * world
        self.peer_flags = [None] * world
        for j in range(world):
            for idx, (hb, off) in enumerate(gathered[j]):
                if j == rank:
                    p = (self.recv + [self.out, self.flags])[idx].data_ptr()
                else:
                    p = self._open(hb, off)
                if idx < n_fwd:
                    self.peer_recv[idx][j] = p
                elif idx == n_fwd:
                    self.peer_out[j] = p
                else:
                    self.peer_flags[j] = p
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

    def fwd(self, tensors, ctx):
        """tensors: n x [s_local, H, D] -> n views [S, H/P, D] of the receive buffers."""
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
        src_arr, k1 = ptr_array([t.data_ptr() for t in srcs])
        dst_arr, k2 = ptr_array([self.peer_recv[i][j] for i in range(n) for j in range(self.world)])
        self.barrier(srcs[0])
        off_rank = n * s_local * self.chunk * es * (self.world - 1)
        with span("a2a_fwd_p2p", off_rank):
            check(lib.h3b_a2a_fwd_p2p(n, src_arr, ld * es, dst_arr, s_local, ctx.start, self.chunk * es, self.world,
                                      stream_of(srcs[0])), "h3b_a2a_fwd_p2p")
        self.barrier(srcs[0])
        del k1, k2
        hp = heads // self.world
        return [self.recv[i][: ctx.seq_len].view(ctx.seq_len, hp, dim) for i in range(n)]

    def inv(self, t, ctx):
        """t [S, (H/P)*D] (unit stride along the row) -> [s_local, H*D] view of the output buffer."""
        require_cuda(t)
        if t.dim() != 2 or t.shape[1] != self.chunk or t.stride(1) != 1 or t.dtype != self.dtype:
            raise ValueError("inv: t must be [S, chunk] with unit column stride")
        dst_arr, k1 = ptr_array(self.peer_out)
        splits = (ctypes.c_int64 * self.world)(*ctx.splits)
        self.barrier(t)
        off_rank = (ctx.seq_len - ctx.local) * self.chunk * t.element_size()
        with span("a2a_inv_p2p", off_rank):
            check(lib.h3b_a2a_inv_p2p(ptr(t), t.stride(0) * t.element_size(), dst_arr, splits,
                                      self.chunk * t.element_size(), self.world, self.rank, stream_of(t)),
                  "h3b_a2a_inv_p2p")
        self.barrier(t)
        del k1
        return self.out[: ctx.local]

    def close(self):
        torch.cuda.synchronize(self.device)
        for b in self._bases:
            check(lib.h3b_ipc_close(ctypes.c_void_p(b)), "h3b_ipc_close")
        self._bases = []


# ---------------------------------------------------------------------------

def startup_probe(rank, world, group, device):
    """Known-answer check of the tensor process group (sp_group.py:107-128):
    all_reduce of rank+1 sums to P(P+1)/2 and all_to_all_single of
    arange(P) + rank*P returns arange(P)*P + rank."""
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
