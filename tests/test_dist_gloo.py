"""Multi-rank host logic on CPU: world_size 2 over gloo (no GPU).

Covers the parts of the Ulysses path that are not kernels: SPContext's row
splits, the exchange calls with their split sizes (h3b.sp._seq_gather /
_seq_scatter, fed with oracle-packed buffers; whole and per head group), the
final layer's padded row gather, the start-up known-answer probe,
and failure detection -- a rank that never reaches the exchange makes the other
rank's collective fail within the process-group timeout instead of hanging.
"""
import os
import socket
import sys
import time
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=60):
    for p in (ROOT, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _worker_exchange(rank, world, port, S, q):
    try:
        _init(rank, world, port)
        from h3b import sp
        from oracle import sp_layout
        H, Dh = 8, 16
        ctx = sp.SPContext(rank, world, dist.group.WORLD, S)
        assert ctx.splits == sp_layout.splits(S, world)
        assert ctx.start == sp_layout.starts(S, world)[rank]
        # every rank draws all ranks' inputs from the same seeds -> local oracle
        ts = [torch.randn(n, H, Dh, generator=torch.Generator().manual_seed(100 + r)).to(torch.bfloat16)
              for r, n in enumerate(ctx.splits)]
        bits = [t.view(torch.int16).numpy().view(np.uint16) for t in ts]
        hp = H // world
        # forward: pack (oracle) -> exchange (product host code) -> [S, hp, Dh]
        # gloo has no 16-bit integer type: carry the bf16 bit patterns as float16
        # (all_to_all copies bytes, the values are never interpreted)
        send = torch.from_numpy(sp_layout.pack_fwd(bits[rank], world).view(np.float16)).reshape(-1)
        out = torch.empty(S * hp * Dh, dtype=torch.float16)
        sp._seq_gather(out, send, ctx, hp * Dh)
        ref = sp_layout.a2a_fwd(bits, world)[rank]
        np.testing.assert_array_equal(out.numpy().view(np.uint16).reshape(S, hp, Dh), ref)
        # inverse: each rank's [S, hp*Dh] -> [s_local, H*Dh] after unpack (oracle)
        outs = [torch.randn(S, hp * Dh, generator=torch.Generator().manual_seed(200 + r)).to(torch.bfloat16)
                for r in range(world)]
        obits = [o.view(torch.int16).numpy().view(np.uint16) for o in outs]
        recv = torch.empty(world * ctx.local * hp * Dh, dtype=torch.float16)
        sp._seq_scatter(recv, torch.from_numpy(obits[rank].view(np.float16)).reshape(-1), ctx, hp * Dh)
        got = sp_layout.unpack_inv(recv.numpy().view(np.uint16).reshape(world, ctx.local, hp * Dh), world)
        np.testing.assert_array_equal(got, sp_layout.a2a_inv(obits, world)[rank])
        # head groups of the exchange/attention overlap (sp_forward.py:211-261):
        # per group the exchange moves hc*Dh-wide rows; the groups reassemble both ways
        groups = 2
        w = hp // groups * Dh
        for g in range(groups):
            send = torch.from_numpy(sp_layout.pack_group(bits[rank], world, groups, g).view(np.float16)).reshape(-1)
            out = torch.empty(S * w, dtype=torch.float16)
            sp._seq_gather(out, send, ctx, w)
            np.testing.assert_array_equal(out.numpy().view(np.uint16).reshape(S, w),
                                          ref.reshape(S, hp * Dh)[:, g * w:(g + 1) * w])
        final = np.zeros((ctx.local, world, groups, w), np.uint16)
        for g in range(groups):
            recv = torch.empty(world * ctx.local * w, dtype=torch.float16)
            part = np.ascontiguousarray(obits[rank][:, g * w:(g + 1) * w])
            sp._seq_scatter(recv, torch.from_numpy(part.view(np.float16)).reshape(-1), ctx, w)
            final[:, :, g] = recv.numpy().view(np.uint16).reshape(world, ctx.local, w).transpose(1, 0, 2)
        np.testing.assert_array_equal(final.reshape(ctx.local, -1), sp_layout.a2a_inv(obits, world)[rank])
        # padded row gather of the final layer (sp_forward.py:378-389), uneven blocks incl. an empty one
        counts = [3, 0] + [2] * (world - 2)
        blocks = [torch.arange(n * 5, dtype=torch.float32).view(n, 5) + 100 * r for r, n in enumerate(counts)]
        got = sp.gather_rows(blocks[rank] if counts[rank] else None, counts, ctx, 5, device=torch.device("cpu"))
        assert torch.equal(got, torch.cat([b for b in blocks if b.shape[0]], dim=0))
        sp.startup_probe(rank, world, dist.group.WORLD, torch.device("cpu"))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


def _worker_dead_peer(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        from h3b import sp
        ctx = sp.SPContext(rank, world, dist.group.WORLD, 100)
        if rank == 1:
            q.put((rank, "left"))  # leaves between steps, before the exchange, with nothing in flight
            q.close()
            q.join_thread()
            os._exit(0)
        send = torch.zeros(ctx.local * 4, dtype=torch.float32)
        out = torch.empty(100 * 4, dtype=torch.float32)
        t0 = time.time()
        try:
            sp._seq_gather(out, send, ctx, 4)
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001
            q.put((rank, ("raised", time.time() - t0, type(e).__name__)))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


def _run(target, world, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            r, v = q.get(timeout=max(0.1, deadline - time.time()))
            results[r] = v
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("S", [1001, 64])
def test_exchange_world2_gloo(S):
    res = _run(_worker_exchange, 2, _free_port(), S)
    assert res == {0: "ok", 1: "ok"}, res


def test_dead_peer_fails_within_timeout():
    res = _run(_worker_dead_peer, 2, _free_port(), timeout=90)
    assert res.get(1) == "left", res
    r0 = res.get(0)
    assert isinstance(r0, tuple) and r0[0] == "raised", res
    assert r0[1] < 60, f"the surviving rank waited {r0[1]:.1f} s"


def test_overlap_groups_env(monkeypatch):
    """Group count of the exchange/attention overlap from the environment
    (sp_forward.py:58,264-273): off by default; at world 4 the count drops to a
    divisor of the rank's heads and the _W4 variable takes precedence."""
    sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))
    from h3b import sp
    for k in ("H3B_SP_OVERLAP_GROUPS", "MINIMAX_SP_OVERLAP_CHUNKS", "MINIMAX_SP_OVERLAP_CHUNKS_W4"):
        monkeypatch.delenv(k, raising=False)
    assert sp.overlap_groups(20, 2) == 0
    monkeypatch.setenv("MINIMAX_SP_OVERLAP_CHUNKS", "4")
    assert sp.overlap_groups(20, 2) == 4
    assert sp.overlap_groups(10, 4) == 2  # 4 does not divide 10 -> 2
    monkeypatch.setenv("MINIMAX_SP_OVERLAP_CHUNKS_W4", "5")
    assert sp.overlap_groups(10, 4) == 5
    monkeypatch.setenv("H3B_SP_OVERLAP_GROUPS", "5")
    assert sp.overlap_groups(5, 8) == 5


def test_peer_exchange_barrier_sequence(monkeypatch):
    """Host logic of the p2p exchange pair (no device work: kernels stubbed).
    gemm_fwd alternates between the two receive sets and skips its entry
    barrier only right after inv_quant; inv_quant takes an extra entry
    barrier unless it follows gemm_fwd; any other exchange call breaks the
    chain.  Every rank runs the same sequence, so all ranks take the same
    barriers."""
    import importlib
    import types

    hl = importlib.import_module("h3b.linear")  # the module (h3b.linear is also a function name)
    hsp = importlib.import_module("h3b.sp")

    events = []
    pe = object.__new__(hsp.PeerExchange)
    pe.world, pe.rank, pe.heads, pe.head_dim, pe.chunk, pe.seq_len = 2, 0, 4, 64, 128, 16
    pe.n_gemm_fwd, pe._last, pe.dtype = 0, None, torch.bfloat16
    pe.recv_sets = [[torch.zeros(16, 128, dtype=torch.bfloat16) for _ in range(3)] for _ in range(2)]
    pe.recv = pe.recv_sets[0]
    pe.peer_recv_sets = [[[100 * s + 10 * t + j for j in range(2)] for t in range(3)] for s in range(2)]
    pe.obuf = torch.zeros(16, 128, dtype=torch.bfloat16)
    pe.peer_obuf = [1, 2]
    pe.barrier = lambda t: events.append("B")
    monkeypatch.setattr(hsp, "require_cuda", lambda *a: None)
    monkeypatch.setattr(hsp, "stream_of", lambda t: None)
    monkeypatch.setattr(hsp, "ptr", lambda t: 0)
    monkeypatch.setattr(hsp, "lib", types.SimpleNamespace(h3b_a2a_inv_quant=lambda *a: events.append("Q") or 0))
    monkeypatch.setattr(hl, "int8_mm_scaled_a2a",
                        lambda xq, w, xs, ws, b, dst, *a, **k: events.append(("G", dst[0] // 100)))
    ctx = types.SimpleNamespace(seq_len=16, local=8, start=0)
    xq = torch.zeros(8, 256, dtype=torch.int8)
    w = torch.zeros(3 * 256, 256, dtype=torch.int8)
    o = torch.zeros(16, 128, dtype=torch.bfloat16)

    def gemm():
        pe.gemm_fwd(xq, None, w, None, None, ctx)

    gemm()
    pe.inv_quant(o, ctx)
    gemm()
    pe.inv_quant(o, ctx)
    gemm()
    pe.inv_quant(o, ctx)
    assert events == ["B", ("G", 0), "B", "B", "Q",     # first pair: entry, exit, inverse
                      ("G", 1), "B", "B", "Q",          # chained: no entry barrier, other set
                      ("G", 0), "B", "B", "Q"]
    events.clear()
    pe.inv_quant(o, ctx)  # not after gemm_fwd: entry barrier before refilling the shared buffer
    pe._last = None  # e.g. fwd() / the overlap ran in between
    gemm()
    assert events == ["B", "B", "Q", "B", ("G", 1), "B"]
