"""h3b against the reference's own Triton kernels, run natively on the GPU.

The reference's INT8 GEMM (comfyui_nodes/h3-linear-fast/int8_gemm_triton.py:32-83)
and its fused norm kernels (comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py:88-192)
import only torch and triton, so on the GPU box they JIT and run as the
reference ships them.  They are a second witness beside the CPU oracle and
PyTorch eager: h3b must produce the same bytes.  The modules are loaded,
unmodified, from baseline/_ref/comfyui_nodes (the reference has no installable
package for them; the directory is git-ignored); the tests skip without it.
"""
import importlib.util
import os

import pytest
import torch

from gpu_util import adversarial_rows, randn_bf16

pytestmark = pytest.mark.gpu

h3b = pytest.importorskip("h3b")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE = os.path.join(ROOT, "baseline", "_ref", "comfyui_nodes")
DEV = torch.device("cuda", 0)


def _load(rel, name):
    path = os.path.join(BASE, rel)
    if not os.path.exists(path):
        pytest.skip(f"the reference's Triton module is not installed under {BASE}")
    pytest.importorskip("triton")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref_gemm():
    return _load(os.path.join("h3-linear-fast", "int8_gemm_triton.py"), "h3ref_int8_gemm_triton")


@pytest.fixture(scope="module")
def ref_fuse():
    return _load(os.path.join("h3-fuse-graph", "h3_fuse_kernels.py"), "h3ref_h3_fuse_kernels")


@pytest.mark.parametrize("M,N,K", [(1000, 1024, 2048), (4096, 5120, 5120), (300, 15360, 5120), (777, 5120, 13824)])
def test_gemm_equals_reference_triton(ref_gemm, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N + K)
    xq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-4).to(DEV)
    ws = (torch.rand(N, generator=g) * 9e-3 + 1e-4).to(DEV)
    y_ref = ref_gemm.int8_mm_scaled(xq, w, xs, ws)
    y = h3b.int8_mm_scaled(xq, w, xs, ws)
    torch.cuda.synchronize()
    n_bad = (y.view(torch.int16) != y_ref.view(torch.int16)).sum().item()
    assert n_bad == 0, f"{n_bad} of {y.numel()} outputs differ from the reference's Triton GEMM"


@pytest.mark.parametrize("D", [5120, 5376])
def test_fused_chain_equals_reference_triton(ref_fuse, D):
    S, R = 2048, 3
    g = torch.Generator().manual_seed(D)
    x0 = adversarial_rows(S, D, 5).to(DEV)
    o = randn_bf16((S, D), 6).to(DEV)
    o2 = randn_bf16((S, D), 7).to(DEV)
    e = (0.1 * torch.randn(R, 6, D, generator=g)).to(torch.bfloat16).to(DEV)
    w1 = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    w2 = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(DEV)
    s1a, sha, ga, s1m, shm, gm = h3b.modulation_tables(*(e[:, i] for i in range(6)))
    ridx = torch.randint(0, R, (S,), generator=g, dtype=torch.int32).to(DEV)
    xa, xb = x0.clone(), x0.clone()
    h_ref = ref_fuse.norm_mod(xa, w1, 1e-6, ridx, s1a, sha)
    h = h3b.norm_mod(xb, w1, 1e-6, ridx, s1a, sha)
    h2_ref = ref_fuse.gate_norm_mod_(xa, o, ga, w2, 1e-6, ridx, s1m, shm)
    h2 = h3b.gate_norm_mod_(xb, o, ga, w2, 1e-6, ridx, s1m, shm)
    ref_fuse.gate_(xa, o2, gm, ridx)
    h3b.gate_(xb, o2, gm, ridx)
    torch.cuda.synchronize()
    for name, a, b in (("norm_mod", h, h_ref), ("gate_norm_mod_", h2, h2_ref), ("residual", xb, xa)):
        n_bad = (a.view(torch.int16) != b.view(torch.int16)).sum().item()
        assert n_bad == 0, f"{name}: {n_bad} elements differ from the reference's Triton kernel"
