"""GPU parity of the INT8 linear path (quantiser, tcgen05 GEMM, dequant epilogue).

Bar: bit-exact.  int8 activations and fp32 scales against the C oracle; int32
accumulators against the oracle (small) and cuBLAS torch._int_mm (large);
bf16 outputs against the oracle (small) and the same fp32 formula evaluated
by PyTorch elementwise ops on the GPU (large).
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import bits, gen, randn_bf16

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")
DEV = "cuda"


def _weights(N, K, seed):
    g = gen(seed)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    ws = torch.rand(N, generator=g) * 9e-3 + 1e-3
    bias = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    return w, ws, bias


@pytest.mark.parametrize("M,K", [(37, 5120), (4096, 5120), (129, 13824), (5, 8), (64, 256)])
def test_quant_bit_exact(M, K):
    x = randn_bf16((M, K), seed=M * 7 + K)
    x[0] = 0  # all-zero row: scale 0, codes 0
    if M > 2:
        x[2, 5] = 1e4  # one outlier dominates the row's scale
    if M > 4:
        # tiny rows: subnormal scales (1/s overflows to inf) and subnormal elements
        x[3] = (randn_bf16((K,), seed=M + 1).float() * 1e-39).to(torch.bfloat16)
        x[4] = (randn_bf16((K,), seed=M + 2).float() * 1e-36).to(torch.bfloat16)
    q_ref, s_ref = oracle.quant_rowwise(bits(x))
    xq, xs = h3b.quant_rowwise(x.to(DEV))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(xq.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(xs.cpu().numpy().reshape(-1), s_ref)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (129, 264, 384), (300, 8, 128), (40, 48, 256), (256, 512, 1024),
                                   (257, 520, 256), (128, 264, 384), (513, 776, 640)])
def test_gemm_small_vs_oracle(M, N, K):
    g = gen(M + N + K)
    xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w, ws, bias = _weights(N, K, seed=N + 1)
    xs = torch.rand(M, 1, generator=g) * 0.05 + 1e-3
    y_ref, acc_ref = oracle.int8_mm_scaled(xq.numpy(), w.numpy(), xs.numpy(), ws.numpy(), want_acc=True)
    yb_ref = oracle.int8_mm_scaled(xq.numpy(), w.numpy(), xs.numpy(), ws.numpy(), bias=bits(bias))
    xq_d, w_d, xs_d, ws_d, b_d = (t.to(DEV) for t in (xq, w, xs, ws, bias))
    acc = h3b.int8_mm_i32(xq_d, w_d)
    y = h3b.int8_mm_scaled(xq_d, w_d, xs_d, ws_d)
    yb = h3b.int8_mm_scaled(xq_d, w_d, xs_d, ws_d, bias=b_d)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(acc.cpu().numpy(), acc_ref)
    np.testing.assert_array_equal(bits(y), y_ref)
    np.testing.assert_array_equal(bits(yb), yb_ref)
    assert h3b.status() == 0


@pytest.mark.parametrize("name", ["gemm_small", "gemm_bigacc"])
def test_gemm_golden_inputs(golden_dir, name):
    """Golden inputs/outputs of the reference kernel itself.  The fixture holds the
    reference's fp32 epilogue values cast by truncation (Triton interpreter); the
    GPU's int32 sums pushed through the same fp32 epilogue must truncate to the
    fixture exactly, and the GPU's bf16 output is the nearest-even rounding of
    those same fp32 values."""
    d = dict(np.load(f"{golden_dir}/{name}.npz"))
    xq, w = torch.from_numpy(d["xq"]).to(DEV), torch.from_numpy(d["w"]).to(DEV)
    xs, ws = torch.from_numpy(d["xs"]).to(DEV), torch.from_numpy(d["ws"]).to(DEV)
    acc = h3b.int8_mm_i32(xq, w)
    y = h3b.int8_mm_scaled(xq, w, xs, ws)
    torch.cuda.synchronize()
    f = (acc.cpu().numpy().astype(np.float32) * d["xs"][:, None]) * d["ws"][None, :]
    np.testing.assert_array_equal(oracle.f32_to_bf16(f, oracle.TRUNC), d["out"])
    np.testing.assert_array_equal(bits(y), oracle.f32_to_bf16(f, oracle.RNE))
    np.testing.assert_array_equal(bits(y), oracle.int8_mm_scaled(d["xq"], d["w"], d["xs"], d["ws"]))


@pytest.mark.parametrize("M,N,K", [(4096, 5120, 5120), (1000, 15360, 5120), (777, 5120, 13824), (16000, 5120, 5120),
                                   (128, 5120, 5120), (100, 15360, 5120), (32768, 5120, 5120)])
def test_gemm_large_vs_cublas(M, N, K):
    g = gen(M ^ N ^ K)
    xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).to(DEV)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(DEV)
    bias = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    ref_acc = torch._int_mm(xq, w.t())
    acc = h3b.int8_mm_i32(xq, w)
    assert torch.equal(acc, ref_acc)
    y = h3b.int8_mm_scaled(xq, w, xs, ws, bias=bias)
    ref = ((ref_acc.float() * xs) * ws + bias.float()).to(torch.bfloat16)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    assert h3b.status() == 0


def test_linear_config0_vs_oracle():
    """Config 0 end to end (quant + GEMM + dequant + bias), oracle on a row sample."""
    M, N, K = 4096, 5120, 5120
    x = randn_bf16((M, K), seed=0)
    w, ws, bias = _weights(N, K, seed=1)
    y = h3b.linear(x.to(DEV), w.to(DEV), ws.to(DEV), bias.to(DEV))
    torch.cuda.synchronize()
    rows = np.r_[0:64, 2000:2064, M - 64:M]
    xr = bits(x)[rows]
    q, s = oracle.quant_rowwise(xr)
    ref = oracle.int8_mm_scaled(q, w.numpy(), s, ws.numpy(), bias=bits(bias))
    np.testing.assert_array_equal(bits(y)[rows], ref)


def test_rejects_bad_shapes():
    xq = torch.zeros(4, 100, dtype=torch.int8, device=DEV)
    w = torch.zeros(8, 100, dtype=torch.int8, device=DEV)
    with pytest.raises(h3b.H3BError):
        h3b.int8_mm_i32(xq, w)  # K % 128 != 0
    with pytest.raises(TypeError):
        h3b.quant_rowwise(torch.zeros(4, 16, dtype=torch.bfloat16))  # CPU tensor: no CPU path


@pytest.mark.parametrize("M,K,scale", [(4096, 13824, 3.0), (513, 5120, 0.3), (64, 128, 20.0)])
def test_gelu_quant_equals_torch_gelu_then_quant(M, K, scale):
    """GELU(tanh) fused into the quantiser == quant_rowwise(F.gelu(u, "tanh")) with
    PyTorch's own GELU on the GPU: any difference in the fp32 GELU arithmetic
    would move codes across rounding boundaries somewhere in these rows."""
    import torch.nn.functional as F
    u = randn_bf16((M, K), seed=M + K, scale=scale).to(DEV)
    q, s = h3b.gelu_quant(u)
    q_ref, s_ref = h3b.quant_rowwise(F.gelu(u, approximate="tanh"))
    torch.cuda.synchronize()
    assert torch.equal(s, s_ref), "row scales differ (GELU maxima differ)"
    assert torch.equal(q, q_ref), f"{(q != q_ref).sum().item()} codes differ"


def _all_bf16():
    """Every bf16 bit pattern once (zeros, subnormals, normals, infinities, NaNs)."""
    return torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)


def test_gelu_every_bf16_input_equals_torch():
    """The fast GELU (x / (1 + 2^w) with an error margin, PyTorch's formula only
    near a bf16 rounding midpoint) against F.gelu(approximate="tanh") on the GPU
    for all 65536 bf16 inputs: a bf16 -> bf16 function is fully determined by
    these, so equality here is equality everywhere.  NaN inputs must give NaN."""
    import torch.nn.functional as F
    x = _all_bf16().to(DEV)
    y = h3b.gelu_tanh(x)
    ref = F.gelu(x, approximate="tanh")
    torch.cuda.synchronize()
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(y), nan)
    bad = (y.view(torch.int16) != ref.view(torch.int16)) & ~nan
    assert bad.sum().item() == 0, f"{bad.sum().item()} inputs differ, e.g. bits {torch.nonzero(bad)[:8].flatten().tolist()}"
    # the odd-length tail of a call (n % 8 != 0) takes the pair path
    y2 = h3b.gelu_tanh(x[:1030].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y2.view(torch.int16), y[:1030].view(torch.int16))


def test_gelu_quant_every_bf16_input():
    """The GELU quantiser over rows that hold every finite bf16 value (shuffled,
    one huge-magnitude row group and one small one) == quant_rowwise(F.gelu(row))."""
    import torch.nn.functional as F
    x = _all_bf16()
    x = x[torch.isfinite(x.float())]
    perm = torch.randperm(x.numel(), generator=gen(3))
    x = x[perm][: (x.numel() // 512) * 512].view(-1, 512).to(DEV)
    small = x.float().abs() < 4
    xs = torch.where(small, x, torch.zeros_like(x))  # rows without the huge values: small absmax, fine codes
    for u in (x, xs):
        q, s = h3b.gelu_quant(u.contiguous())
        q_ref, s_ref = h3b.quant_rowwise(F.gelu(u, approximate="tanh"))
        torch.cuda.synchronize()
        assert torch.equal(s, s_ref) and torch.equal(q, q_ref)


def test_quant_half_integer_ties():
    """Rows whose quotients land exactly on (or next to) half-integers exercise the
    exact-division fallback; codes must match the oracle (round half to even)."""
    M, K = 64, 512
    g = gen(99)
    k = torch.randint(-126, 126, (M, K), generator=g).float()
    x = (k + 0.5)
    x[:, 0] = 127.0  # absmax 127 -> scale exactly 1, quotients exactly k + 0.5
    x[32:, 0] = 126.0  # scale 126/127: quotients just off half-integers
    x = x.to(torch.bfloat16)
    q_ref, s_ref = oracle.quant_rowwise(bits(x))
    xq, xs = h3b.quant_rowwise(x.to(DEV))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(xq.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(xs.cpu().numpy().reshape(-1), s_ref)


@pytest.mark.parametrize("M,K,group", [(37, 5120, 256), (4096, 5120, 256), (129, 13824, 256), (64, 256, 256),
                                       (300, 1024, 64), (5, 64, 64), (3, 32768, 256)])
def test_quant_convrot_bit_exact(M, K, group):
    """ConvRot quantiser (group-wise Walsh-Hadamard rotation, then absmax codes)
    against the C restatement, bit for bit; zero, outlier and tiny rows."""
    x = randn_bf16((M, K), seed=M * 5 + K + group)
    x[0] = 0
    if M > 2:
        x[2, 7] = 3e3
    if M > 4:
        x[3] = (randn_bf16((K,), seed=M + 11).float() * 1e-38).to(torch.bfloat16)
        x[4] = torch.randint(-8, 9, (K,), generator=gen(M)).to(torch.bfloat16)  # exact rotation, many ties
    q_ref, s_ref = oracle.quant_rowwise_convrot(bits(x), group)
    xq, xs = h3b.quant_rowwise_convrot(x.to(DEV), group)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(xs.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(xq.cpu().numpy(), q_ref)


def test_int8_linear_convrot_vs_oracle():
    """The patched int8_linear with convrot=True (the reference fast path's case):
    rotated quantiser + GEMM + dequant equals the oracle on a row sample; an
    unsupported group size raises NotImplementedError (the caller's fallback)."""
    M, N, K = 2048, 1536, 5120
    x = randn_bf16((M, K), seed=21)
    w, ws, _ = _weights(N, K, seed=22)
    y = h3b.int8_linear(x.to(DEV), w.to(DEV), ws.to(DEV), None, torch.bfloat16, convrot=True, convrot_groupsize=256)
    torch.cuda.synchronize()
    rows = np.r_[0:32, 1000:1032, M - 32:M]
    q, s = oracle.quant_rowwise_convrot(bits(x)[rows], 256)
    np.testing.assert_array_equal(bits(y)[rows], oracle.int8_mm_scaled(q, w.numpy(), s, ws.numpy()))
    with pytest.raises(NotImplementedError):
        h3b.int8_linear(x[:, :K // 2].to(DEV), w[:, :K // 2].to(DEV), ws.to(DEV), convrot=True, convrot_groupsize=128)


@pytest.mark.parametrize("M,K,group,scale", [(513, 5120, 256, 1.0), (64, 13824, 256, 4.0), (300, 1024, 64, 0.5)])
def test_swiglu_quant_convrot_equals_composition(M, K, group, scale):
    """SwiGLU fused into the ConvRot quantiser == PyTorch's own activation
    (F.silu(a.float()) * b.float() -> bf16, on the GPU) followed by the ConvRot
    quantiser, bit for bit; and that composition matches the C restatement."""
    import torch.nn.functional as F
    x = randn_bf16((M, 2 * K), seed=M + K + group, scale=scale).to(DEV)
    act = (F.silu(x[:, :K].float()) * x[:, K:].float()).to(torch.bfloat16)
    q, s = h3b.swiglu_quant_convrot(x, group)
    q_ref, s_ref = h3b.quant_rowwise_convrot(act.contiguous(), group)
    torch.cuda.synchronize()
    assert torch.equal(s, s_ref), "row scales differ"
    assert torch.equal(q, q_ref), f"{(q != q_ref).sum().item()} codes differ"
    rows = np.arange(0, M, max(1, M // 16))
    qo, so = oracle.quant_rowwise_convrot(bits(act)[rows], group)
    np.testing.assert_array_equal(q.cpu().numpy()[rows], qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1)[rows], so)


def test_int8_linear_swiglu_convrot():
    """int8_linear(input_act="swiglu", convrot=True) on x [M, 2K]: the reference
    fast path's fc2 call, equal to the oracle GEMM on the fused quantiser's codes."""
    M, N, K = 512, 1024, 2048
    x = randn_bf16((M, 2 * K), seed=31).to(DEV)
    w, ws, _ = _weights(N, K, seed=32)
    y = h3b.int8_linear(x, w.to(DEV), ws.to(DEV), None, torch.bfloat16, convrot=True, convrot_groupsize=256,
                        input_act="swiglu")
    q, s = h3b.swiglu_quant_convrot(x, 256)
    torch.cuda.synchronize()
    ref = oracle.int8_mm_scaled(q.cpu().numpy(), w.numpy(), s.cpu().numpy(), ws.numpy())
    np.testing.assert_array_equal(bits(y), ref)


def test_gemm_rows_independent_of_m():
    """A row's output does not depend on how many rows the launch has (tile
    width, pair/1-CTA kernel and wave count all change with M): the property the
    reference's final layer pads for (sp_forward.py:340-348) holds here without
    padding."""
    N, K = 5120, 5120
    x = randn_bf16((4128, K), seed=41)
    w, ws, b = _weights(N, K, seed=42)
    wd, wsd, bd = w.to(DEV), ws.to(DEV), b.to(DEV)
    full = h3b.linear(x.to(DEV), wd, wsd, bd)
    for lo, hi in ((0, 100), (0, 129), (1000, 1516), (3000, 4128), (7, 8)):
        part = h3b.linear(x[lo:hi].to(DEV), wd, wsd, bd)
        assert torch.equal(part.view(torch.int16), full[lo:hi].view(torch.int16)), (lo, hi)


@pytest.mark.parametrize("M,N,K", [(513, 13824, 5120), (100, 2048, 1024), (4096, 5120, 256)])
def test_gemm_gelu_epilogue_equals_torch_gelu(M, N, K):
    """GELU in the GEMM epilogue == F.gelu of the plain GEMM's bf16 output, bit for bit."""
    import torch.nn.functional as F
    g = gen(M + N + K + 5)
    xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w, ws, bias = _weights(N, K, seed=N + 7)
    xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).to(DEV)
    wd, wsd, bd = w.to(DEV), (ws * 40).to(DEV), bias.to(DEV)
    y = h3b.int8_mm_scaled(xq, wd, xs, wsd, bias=bd, act="gelu")
    ref = F.gelu(h3b.int8_mm_scaled(xq, wd, xs, wsd, bias=bd), approximate="tanh")
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), f"{(y != ref).sum().item()} elements differ"


@pytest.mark.parametrize("N,K", [(15360, 5120), (5120, 13824)])
def test_gemm_full_block_size_vs_cublas(N, K):
    """The block's qkv and down projections at the benchmark's full M=128000:
    int32 sums equal cuBLAS's torch._int_mm, bf16 outputs equal the fp32 formula."""
    M = 128000
    g = gen(N + K)
    xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).to(DEV)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).to(DEV)
    ref_acc = torch._int_mm(xq, w.t())
    acc = h3b.int8_mm_i32(xq, w)
    assert torch.equal(acc, ref_acc)
    del acc
    y = h3b.int8_mm_scaled(xq, w, xs, ws)
    ref = ((ref_acc.float() * xs) * ws).to(torch.bfloat16)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    assert h3b.status() == 0
