"""Ulysses exchange and the SP block on 2, 4 and 8 GPUs (one spawned process per GPU, NCCL).

Each world size runs when the host has that many GPUs (skipped otherwise).
Each rank draws every rank's inputs
from the same seeds, so it can check its own result against the numpy
restatement locally.  Checked bit-exactly:
  * the start-up known-answer probe (sp_group.py:107-128);
  * forward (q, k, v together) and inverse exchange, NCCL back end (pack kernel,
    all_to_all_single, unpack kernel) and peer-memory back end (fused p2p
    kernels + flag barriers), with an uneven row split;
  * the same exchanges done the reference's way (reshape + all_to_all_single);
  * the exchange/attention overlap by head groups (both back ends, several
    group counts) against the plain exchange;
  * configuration 2 at its full size (S=131072): forward + inverse exchange as
    an identity round trip on both back ends, forward equal to the reference's
    reshape + all_to_all_single;
  * two blocks of the 40-block step model (512 text tokens) over an uneven
    row split against the eager block loop;
  * one full DiT block (p2p exchange: fused into the qkv GEMM's epilogue and
    the out projection's quantiser, as separate kernels, and the overlap)
    against the eager PyTorch block using all_to_all_single.
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

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _worker(rank, world, port, q):
    try:
        for p in (ROOT, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"), os.path.join(ROOT, "tests")):
            if p not in sys.path:
                sys.path.insert(0, p)
        import torch.distributed as dist
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120), device_id=dev)
        import h3b
        from h3b import model as hm
        from oracle import sp_layout
        from oracle import torch_path as tp
        g = dist.group.WORLD
        h3b.startup_probe(rank, world, g, dev)
        H, Dh = 40, 128
        for S in (1001 + world, 8192):
            splits = sp_layout.splits(S, world)
            hp = H // world
            ins = [[torch.randn(splits[r], H, Dh, generator=torch.Generator().manual_seed(10 * i + r)).to(torch.bfloat16)
                    for r in range(world)] for i in range(3)]
            outs = [torch.randn(S, hp * Dh, generator=torch.Generator().manual_seed(99 + r)).to(torch.bfloat16)
                    for r in range(world)]
            ref_fwd = [sp_layout.a2a_fwd([_bits(t) for t in ins[i]], world)[rank] for i in range(3)]
            ref_inv = sp_layout.a2a_inv([_bits(o) for o in outs], world)[rank]
            mine = [ins[i][rank].to(dev) for i in range(3)]
            o_mine = outs[rank].to(dev)
            peer = h3b.PeerExchange(g, rank, world, S, H, Dh)
            h3b.startup_probe(rank, world, g, dev, peer=peer)  # the p2p known-answer round trip
            for exch in ("nccl", "p2p"):
                ctx = h3b.SPContext(rank, world, g, S, exchange=exch, peer=peer if exch == "p2p" else None)
                for rep in range(2):  # twice: the p2p buffers and flags are reused
                    got = h3b.a2a_gather_qkv(*mine, ctx)
                    for i in range(3):
                        np.testing.assert_array_equal(_bits(got[i]), ref_fwd[i], err_msg=f"{exch} fwd S={S} t={i}")
                    inv = h3b.a2a_scatter_seq_gather_heads(o_mine, ctx)
                    np.testing.assert_array_equal(_bits(inv), ref_inv, err_msg=f"{exch} inv S={S}")
            # exchange/attention overlap by head groups (sp_forward.py:211-261); the
            # routing is checked with an elementwise stand-in for attention
            def mix(a, b, c):
                return (a * 3 + b - c).reshape(a.shape[0], -1)
            ctx_n = h3b.SPContext(rank, world, g, S)
            o_ref = _bits(h3b.a2a_scatter_seq_gather_heads(mix(*h3b.a2a_gather_qkv(*mine, ctx_n)), ctx_n))
            for exch in ("nccl", "p2p"):
                ctx = h3b.SPContext(rank, world, g, S, exchange=exch, peer=peer if exch == "p2p" else None)
                for groups in sorted({n for n in (2, 5, hp) if n > 1 and hp % n == 0}):
                    for rep in range(2):
                        got = h3b.sp_attention_overlap(*mine, ctx, mix, groups)
                        np.testing.assert_array_equal(_bits(got), o_ref, err_msg=f"{exch} overlap {groups} S={S}")
            # the reference's own formulation
            ctx = h3b.SPContext(rank, world, g, S)
            np.testing.assert_array_equal(_bits(tp.a2a_gather_seq_scatter_heads(mine[0], ctx)), ref_fwd[0])
            np.testing.assert_array_equal(_bits(tp.a2a_scatter_seq_gather_heads(o_mine, ctx)), ref_inv)
            torch.cuda.synchronize(dev)
            dist.barrier(device_ids=[rank])
            peer.close()
        # configuration 2 at its full size: S=131072, q/k/v forward + inverse of the
        # received q is an identity round trip, on both back ends (and equal to
        # the reference's reshape + all_to_all_single formulation)
        S = 131072
        peer = h3b.PeerExchange(g, rank, world, S, H, Dh)
        ctx_n = h3b.SPContext(rank, world, g, S)
        mine = [torch.randn(ctx_n.local, H, Dh, generator=torch.Generator().manual_seed(1000 * i + rank))
                .to(torch.bfloat16).to(dev) for i in range(3)]
        ref_q = tp.a2a_gather_seq_scatter_heads(mine[0], ctx_n)
        for exch in ("nccl", "p2p"):
            ctx = h3b.SPContext(rank, world, g, S, exchange=exch, peer=peer if exch == "p2p" else None)
            for rep in range(2):
                qq, kk, vv = h3b.a2a_gather_qkv(*mine, ctx)
                assert torch.equal(qq.view(torch.int16), ref_q.view(torch.int16)), f"{exch} fwd at S={S}"
                back = h3b.a2a_scatter_seq_gather_heads(qq.reshape(S, -1), ctx)
                assert torch.equal(back.reshape(-1).view(torch.int16), mine[0].reshape(-1).view(torch.int16)), \
                    f"{exch} round trip at S={S}"
                back_v = h3b.a2a_scatter_seq_gather_heads(vv.reshape(S, -1), ctx)
                assert torch.equal(back_v.reshape(-1).view(torch.int16), mine[2].reshape(-1).view(torch.int16)), \
                    f"{exch} v round trip at S={S}"
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[rank])
        peer.close()
        del mine, ref_q
        # two blocks of the 40-block step model (512 text tokens, cross-attention)
        # over an uneven row split, p2p exchange, against the eager block loop
        cfg_s = hm.DiTConfig(n_blocks=2, text_len=512)
        S = 4128 + world - 1
        dit = hm.SynthDiT(cfg_s, dev, seed=23)
        full = torch.randn(S, cfg_s.dim, generator=torch.Generator().manual_seed(24)).to(torch.bfloat16)
        text = torch.randn(512, cfg_s.dim, generator=torch.Generator().manual_seed(25)).to(torch.bfloat16).to(dev)
        peer = h3b.PeerExchange(g, rank, world, S, cfg_s.heads, cfg_s.head_dim)
        ctx = h3b.SPContext(rank, world, g, S, exchange="p2p", peer=peer)
        x = full[ctx.start:ctx.stop].to(dev)
        ridx = torch.zeros(ctx.local, dtype=torch.int32, device=dev)
        y = dit.forward(x.clone(), ridx, ctx, text)
        y_ref = x.clone()
        for p in dit.params:
            y_ref = tp.block_forward(cfg_s, p, y_ref, ridx, h3b.SPContext(rank, world, g, S), text)
        torch.cuda.synchronize(dev)
        bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
        assert bad == 0, f"2-block step with text at world {world}: {bad} elements differ"
        dist.barrier(device_ids=[rank])
        peer.close()
        del dit
        # one full block at this world size against the eager block
        cfg = hm.DiTConfig()
        S = 4128
        p = hm.make_params(cfg, 0, 7, dev, R=2)
        full = torch.randn(S, cfg.dim, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
        peer = h3b.PeerExchange(g, rank, world, S, cfg.heads, cfg.head_dim)
        ctx = h3b.SPContext(rank, world, g, S, exchange="p2p", peer=peer)
        x = full[ctx.start:ctx.stop].to(dev)
        ridx = torch.zeros(ctx.local, dtype=torch.int32, device=dev)
        ridx[ctx.local // 2:] = 1
        y = hm.block_forward(cfg, p, x.clone(), ridx, ctx)
        y_ref = tp.block_forward(cfg, p, x.clone(), ridx, h3b.SPContext(rank, world, g, S))
        torch.cuda.synchronize(dev)
        bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
        assert bad == 0, f"block at world {world}: {bad} elements differ"
        # the same block with the exchanges as separate kernels
        hm.FUSED_EXCHANGE = False
        try:
            y3 = hm.block_forward(cfg, p, x.clone(), ridx, ctx)
        finally:
            hm.FUSED_EXCHANGE = True
        torch.cuda.synchronize(dev)
        bad = (y3.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
        assert bad == 0, f"unfused-exchange block at world {world}: {bad} elements differ"
        # a block with the per-head q/k norm: fused into the qkv GEMM's epilogue here
        cfg_n = hm.DiTConfig(qk_norm=True)
        p_n = hm.make_params(cfg_n, 0, 8, dev, R=2)
        y4 = hm.block_forward(cfg_n, p_n, x.clone(), ridx, ctx)
        y4_ref = tp.block_forward(cfg_n, p_n, x.clone(), ridx, h3b.SPContext(rank, world, g, S))
        torch.cuda.synchronize(dev)
        bad = (y4.view(torch.int16) != y4_ref.view(torch.int16)).sum().item()
        assert bad == 0, f"qk-norm block at world {world}: {bad} elements differ"
        # the same block with the exchange/attention overlap (one head per group)
        y2 = hm.block_forward(cfg, p, x.clone(), ridx, ctx, overlap_groups=cfg.heads // world)
        torch.cuda.synchronize(dev)
        bad = (y2.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
        assert bad == 0, f"overlapped block at world {world}: {bad} elements differ"
        assert h3b.status() == 0
        dist.barrier(device_ids=[rank])
        peer.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_and_block(world):
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 600
    while len(res) < world and time.time() < deadline:
        try:
            r, v = q.get(timeout=max(1.0, deadline - time.time()))
            res[r] = v
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res == {r: "ok" for r in range(world)}, res
