"""GPU parity of the Ulysses all-to-all kernels on one GPU (bit-exact).

Pack/unpack are checked against the numpy restatement of sp_forward.py:185/198.
The peer-memory exchange kernels (and the qkv GEMM whose epilogue does the
forward exchange, and the quantiser that gathers the inverse one) are checked by running every rank's launch on one GPU with all
"peer" buffers local: they never wait on anything, so this exercises their
full index arithmetic without a second GPU.  The
barrier kernel's bounded wait is checked by letting it wait for a flag that
nothing sets.  Multi-GPU runs are in test_gpu_multi.py.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from gpu_util import bits, randn_bf16
from oracle import sp_layout

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")
from h3b._lib import check, lib, ptr_array, STATUS_PEER_TIMEOUT  # noqa: E402

DEV = "cuda"
H, DH = 40, 128


@pytest.mark.parametrize("world,s_local", [(2, 1000), (4, 333), (8, 16384), (1, 10)])
def test_pack_unpack(world, s_local):
    t = randn_bf16((s_local, H, DH), seed=world * 100 + s_local)
    send = h3b.pack(t.to(DEV).reshape(s_local, H * DH), world)
    ref = sp_layout.pack_fwd(bits(t), world)
    np.testing.assert_array_equal(bits(send), ref)
    back = h3b.unpack(send)
    np.testing.assert_array_equal(bits(back), bits(t).reshape(s_local, H * DH))


def test_pack_strided_rows():
    """q of a fused qkv output: rows with stride 3*H*Dh are packed without a copy."""
    world, s_local = 4, 300
    qkv = randn_bf16((s_local, 3 * H * DH), seed=77)
    q = qkv.to(DEV)[:, H * DH:2 * H * DH]  # the k third, strided rows
    send = h3b.pack(q, world)
    ref = sp_layout.pack_fwd(bits(qkv)[:, H * DH:2 * H * DH].reshape(s_local, H, DH), world)
    np.testing.assert_array_equal(bits(send), ref)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _fwd_p2p(n, srcs, src_ld, dsts, s_local, row_start, width, block, offset, world):
    src, k1 = ptr_array([t.data_ptr() for t in srcs])
    dst, k2 = ptr_array(dsts)
    check(lib.h3b_a2a_fwd_p2p(n, src, src_ld, dst, s_local, row_start, width, block, offset, world, _stream()),
          "fwd_p2p")


def _inv_p2p(src, dsts, splits, width, dst_ld, offset, world):
    dst, k = ptr_array(dsts)
    sp = (ctypes.c_int64 * world)(*splits)
    check(lib.h3b_a2a_inv_p2p(ctypes.c_void_p(src.data_ptr()), src.stride(0) * 2, dst, sp, width, dst_ld, offset,
                              world, _stream()), "inv_p2p")


@pytest.mark.parametrize("world,S", [(2, 1001), (4, 4130), (8, 8192)])
def test_p2p_kernels_emulated(world, S):
    """Every rank's fwd/inv launch on one GPU against sp_layout.a2a_fwd / a2a_inv."""
    splits = sp_layout.splits(S, world)
    starts = sp_layout.starts(S, world)
    hp = H // world
    chunk = hp * DH
    qs = [randn_bf16((splits[r], H, DH), seed=1000 + r) for r in range(world)]
    ks = [randn_bf16((splits[r], H, DH), seed=2000 + r) for r in range(world)]
    recv_q = [torch.empty(S, chunk, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    recv_k = [torch.empty(S, chunk, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    qd = [q.to(DEV) for q in qs]
    kd = [k.to(DEV) for k in ks]
    for r in range(world):
        _fwd_p2p(2, [qd[r], kd[r]], H * DH * 2, [t.data_ptr() for t in recv_q] + [t.data_ptr() for t in recv_k],
                 splits[r], starts[r], chunk * 2, chunk * 2, 0, world)
    torch.cuda.synchronize()
    ref_q = sp_layout.a2a_fwd([bits(q) for q in qs], world)
    ref_k = sp_layout.a2a_fwd([bits(k) for k in ks], world)
    for j in range(world):
        np.testing.assert_array_equal(bits(recv_q[j]).reshape(S, hp, DH), ref_q[j])
        np.testing.assert_array_equal(bits(recv_k[j]).reshape(S, hp, DH), ref_k[j])
    # inverse: rank j holds o_j [S, chunk] (use a strided view to exercise src_ld)
    outs = [randn_bf16((S, chunk + 64), seed=3000 + j) for j in range(world)]
    od = [o.to(DEV)[:, :chunk] for o in outs]
    res = [torch.empty(splits[r], world * chunk, dtype=torch.bfloat16, device=DEV) for r in range(world)]
    for j in range(world):
        _inv_p2p(od[j], [t.data_ptr() for t in res], splits, chunk * 2, world * chunk * 2, j * chunk * 2, world)
    torch.cuda.synchronize()
    ref = sp_layout.a2a_inv([bits(o)[:, :chunk] for o in outs], world)
    for r in range(world):
        np.testing.assert_array_equal(bits(res[r]), ref[r])


@pytest.mark.parametrize("world,S,groups", [(2, 1001, 4), (4, 4130, 2), (8, 8192, 5), (2, 999, 20)])
def test_p2p_head_groups_emulated(world, S, groups):
    """Head-group exchanges (the overlap's per-group copies): group g of every
    destination rank's heads lands in that group's region of the receive buffer,
    and the per-group inverse copies assemble the same output as one exchange."""
    splits = sp_layout.splits(S, world)
    starts = sp_layout.starts(S, world)
    hp = H // world
    hc = hp // groups
    chunk, w = hp * DH, hc * DH
    qkv = [randn_bf16((splits[r], 3 * H * DH), seed=4000 + r) for r in range(world)]
    qkv_d = [t.to(DEV) for t in qkv]
    recv = [[torch.empty(S * chunk, dtype=torch.bfloat16, device=DEV) for _ in range(world)] for _ in range(3)]
    for g in range(groups):
        for r in range(world):
            srcs = [qkv_d[r][:, i * H * DH:] for i in range(3)]
            dsts = [recv[i][j].data_ptr() + g * S * w * 2 for i in range(3) for j in range(world)]
            _fwd_p2p(3, srcs, 3 * H * DH * 2, dsts, splits[r], starts[r], w * 2, chunk * 2, g * w * 2, world)
    torch.cuda.synchronize()
    for i in range(3):
        ref = sp_layout.a2a_fwd([bits(t)[:, i * H * DH:(i + 1) * H * DH].reshape(-1, H, DH) for t in qkv], world)
        for j in range(world):
            got = bits(recv[i][j]).reshape(groups, S, hc, DH)
            for g in range(groups):
                np.testing.assert_array_equal(got[g], ref[j][:, g * hc:(g + 1) * hc])
    outs = [[randn_bf16((S, w), seed=5000 + 37 * j + g) for g in range(groups)] for j in range(world)]
    res = [torch.empty(splits[r], world * chunk, dtype=torch.bfloat16, device=DEV) for r in range(world)]
    for g in range(groups):
        for j in range(world):
            _inv_p2p(outs[j][g].to(DEV), [t.data_ptr() for t in res], splits, w * 2, world * chunk * 2,
                     (j * chunk + g * w) * 2, world)
    torch.cuda.synchronize()
    ref = sp_layout.a2a_inv([np.concatenate([bits(o) for o in outs[j]], axis=1) for j in range(world)], world)
    for r in range(world):
        np.testing.assert_array_equal(bits(res[r]), ref[r])


@pytest.mark.parametrize("world,s_local,groups", [(2, 1000, 4), (8, 777, 5), (4, 64, 10)])
def test_pack_unpack_head_groups(world, s_local, groups):
    """Group pack/unpack of the NCCL overlap path against numpy slicing."""
    hp = H // world
    hc = hp // groups
    w = hc * DH
    qkv = randn_bf16((s_local, 3 * H * DH), seed=world + s_local)
    k = qkv.to(DEV)[:, H * DH:2 * H * DH]
    kb = bits(qkv)[:, H * DH:2 * H * DH].reshape(s_local, world, groups, w)
    final = torch.zeros(s_local, H * DH, dtype=torch.bfloat16, device=DEV)
    for g in range(groups):
        send = h3b.pack(k[:, g * w:], world, width=w, block=hp * DH)
        np.testing.assert_array_equal(bits(send), kb[:, :, g].transpose(1, 0, 2))
        h3b.unpack(send, out=final[:, g * w:], block=hp * DH)
    np.testing.assert_array_equal(bits(final), bits(qkv)[:, H * DH:2 * H * DH])


@pytest.mark.parametrize("world,S,heads,K", [(2, 1001, 40, 256), (4, 4130, 40, 384), (8, 2000, 40, 256),
                                             (1, 300, 8, 128), (2, 20000, 40, 5120), (8, 130, 16, 128)])
def test_gemm_a2a_emulated(world, S, heads, K):
    """The qkv GEMM with the exchange in its epilogue (h3b_int8_mm_scaled_a2a),
    every rank's launch on one GPU: each rank's receive buffers must equal the
    forward exchange (sp_layout.a2a_fwd) of the unfused GEMM outputs, and every
    receive row must be written (the buffers start as a sentinel pattern)."""
    from gpu_util import gen
    splits = sp_layout.splits(S, world)
    starts = sp_layout.starts(S, world)
    hp = heads // world
    D = heads * DH
    g = gen(world * 1000 + S + K)
    w = torch.randint(-127, 128, (3 * D, K), generator=g, dtype=torch.int8).to(DEV)
    ws = (torch.rand(3 * D, generator=g) * 9e-3 + 1e-3).to(DEV)
    bias = (torch.randn(3 * D, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    xq = [torch.randint(-127, 128, (n, K), generator=g, dtype=torch.int8).to(DEV) for n in splits]
    xs = [(torch.rand(n, 1, generator=g) * 0.05 + 1e-3).to(DEV) for n in splits]
    recv = [[torch.full((S, hp * DH), -7.0, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
            for _ in range(3)]
    dst = [recv[t][j].data_ptr() for t in range(3) for j in range(world)]
    for r in range(world):
        h3b.int8_mm_scaled_a2a(xq[r], w, xs[r], ws, bias, dst, starts[r], D, DH, hp, world)
    ys = [h3b.int8_mm_scaled(xq[r], w, xs[r], ws, bias=bias) for r in range(world)]
    torch.cuda.synchronize()
    assert h3b.status() == 0
    for t in range(3):
        ref = sp_layout.a2a_fwd([bits(y)[:, t * D:(t + 1) * D].reshape(-1, heads, DH) for y in ys], world)
        for j in range(world):
            np.testing.assert_array_equal(bits(recv[t][j]).reshape(S, hp, DH), ref[j], err_msg=f"t={t} j={j}")


@pytest.mark.parametrize("world,S", [(2, 1001), (4, 4130), (8, 2000), (8, 9)])
def test_inv_quant_emulated(world, S):
    """The out projection's quantiser gathering its rows from every rank's
    attention output (h3b_a2a_inv_quant), every rank's launch on one GPU: codes
    and scales equal quant_rowwise of the rows the inverse exchange delivers."""
    splits = sp_layout.splits(S, world)
    starts = sp_layout.starts(S, world)
    chunk = H // world * DH
    outs = [randn_bf16((S, chunk), seed=6000 + j, scale=1.0 + j) for j in range(world)]
    od = [o.to(DEV) for o in outs]
    ref_rows = sp_layout.a2a_inv([bits(o) for o in outs], world)
    src, keep = ptr_array([o.data_ptr() for o in od])
    for r in range(world):
        xq = torch.empty(splits[r], H * DH, dtype=torch.int8, device=DEV)
        xs = torch.empty(splits[r], 1, dtype=torch.float32, device=DEV)
        check(lib.h3b_a2a_inv_quant(src, chunk * 2, starts[r], splits[r], chunk * 2, world,
                                    ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(xs.data_ptr()), _stream()),
              "inv_quant")
        rows = torch.from_numpy(ref_rows[r].view(np.int16)).view(torch.bfloat16).to(DEV)
        q_ref, s_ref = h3b.quant_rowwise(rows)
        torch.cuda.synchronize()
        assert torch.equal(xq, q_ref), f"rank {r}: codes differ"
        assert torch.equal(xs.reshape(-1), s_ref.reshape(-1)), f"rank {r}: scales differ"


@pytest.mark.parametrize("world,S,heads,K", [(2, 1001, 40, 256), (8, 2000, 40, 384), (1, 300, 8, 128),
                                             (4, 4130, 40, 5120)])
def test_gemm_a2a_qknorm_emulated(world, S, heads, K):
    """The qkv GEMM with the per-head q/k RMSNorm and the exchange in its
    epilogue: each rank's receive buffers equal the forward exchange of
    F.rms_norm applied (on the GPU, per 128-wide head) to the unfused GEMM's q and
    k; v passes through unnormalised."""
    import torch.nn.functional as F
    from gpu_util import gen
    splits = sp_layout.splits(S, world)
    starts = sp_layout.starts(S, world)
    hp = heads // world
    D = heads * DH
    g = gen(world * 77 + S + K)
    w = torch.randint(-127, 128, (3 * D, K), generator=g, dtype=torch.int8).to(DEV)
    ws = (torch.rand(3 * D, generator=g) * 9e-3 + 1e-3).to(DEV)
    ws[:D // 2] *= 40  # wide per-head magnitudes for the norm
    bias = (torch.randn(3 * D, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    nw = (1 + 0.05 * torch.randn(2, DH, generator=g)).to(torch.bfloat16).to(DEV)
    xq = [torch.randint(-127, 128, (n, K), generator=g, dtype=torch.int8).to(DEV) for n in splits]
    xs = [(torch.logspace(-3, 0, n)[:, None] * 0.05).float().to(DEV) for n in splits]
    recv = [[torch.full((S, hp * DH), -7.0, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
            for _ in range(3)]
    dst = [recv[t][j].data_ptr() for t in range(3) for j in range(world)]
    for r in range(world):
        h3b.int8_mm_scaled_a2a(xq[r], w, xs[r], ws, bias, dst, starts[r], D, DH, hp, world, norm_w=nw, norm_eps=1e-6)
    outs = []
    for r in range(world):
        y = h3b.int8_mm_scaled(xq[r], w, xs[r], ws, bias=bias).view(-1, 3, heads, DH)
        q = F.rms_norm(y[:, 0], (DH,), nw[0], 1e-6)
        k = F.rms_norm(y[:, 1], (DH,), nw[1], 1e-6)
        outs.append([q, k, y[:, 2]])
    torch.cuda.synchronize()
    assert h3b.status() == 0
    for t in range(3):
        ref = sp_layout.a2a_fwd([bits(o[t].contiguous()) for o in outs], world)
        for j in range(world):
            np.testing.assert_array_equal(bits(recv[t][j]).reshape(S, hp, DH), ref[j], err_msg=f"t={t} j={j}")


def test_peer_barrier_times_out_and_reports():
    """A barrier whose peer never arrives gives up after its limit and records
    STATUS_PEER_TIMEOUT; the context stays usable and an arrived barrier passes."""
    world = 2
    f0 = torch.zeros(world, dtype=torch.int32, device=DEV)
    f1 = torch.zeros(world, dtype=torch.int32, device=DEV)
    arr, keep = ptr_array([f0.data_ptr(), f1.data_ptr()])
    h3b.clear_status()
    t0 = time.time()
    check(lib.h3b_peer_barrier(arr, world, 0, 1, int(0.3e9), _stream()), "barrier")
    st = h3b.status()
    elapsed = time.time() - t0
    assert st == STATUS_PEER_TIMEOUT
    assert elapsed < 10
    assert f1[0].item() == 1  # the signal to the peer was still delivered
    h3b.clear_status()
    f0[1] = 1  # the "peer" has arrived for epoch 1
    check(lib.h3b_peer_barrier(arr, world, 0, 1, int(5e9), _stream()), "barrier")
    assert h3b.status() == 0
    x = torch.ones(4, device=DEV) * 2
    assert x.sum().item() == 8.0
