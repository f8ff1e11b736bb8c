"""Generate the golden fixtures in this directory from the reference's own code.

Run once on a machine that has the reference checkout (it is read, never
copied):  python tests/golden/make_golden.py /path/to/reference

What runs:
  * comfyui_nodes/h3-linear-fast/int8_gemm_triton.py  _int8_mm_scaled_kernel (:32-66)
  * comfyui_nodes/h3-fuse-graph/h3_fuse_kernels.py    norm_mod / gate_norm_mod_ / gate_ (:174-192)
executed by Triton's CPU interpreter (TRITON_INTERPRET=1).  The interpreter
runs the kernels' arithmetic in numpy float32 with three documented
differences from the GPU: a float32 -> bf16 cast truncates instead of rounding
to nearest-even, "acc + x*x" is not contracted to a fused multiply-add, and
tl.math.rsqrt is 1/np.sqrt.  The oracle reproduces the fixtures exactly in the
matching mode (oracle.TRUNC, fma=False, RSQRT_RECIP); the product mode differs
only in those three switches.

Also recorded: the modulation-table expression of h3_fuse_patch.py:113,116
(`1.0 + scale.to(bf16)`) evaluated by PyTorch on CPU, which is the reference's
own statement run as written.

Inputs are drawn with torch.Generator on CPU (seeded), outputs saved as raw
bf16 bit patterns (uint16) in .npz files.
"""
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import zlib  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def adversarial_rows(g, S, D):
    """Row magnitudes spread over logspace(-2, 3) and the first 7 columns x50,
    the input recipe of the reference's tests/test_rmsnorm_exact.py:122-123."""
    x = torch.randn(S, D, generator=g) * torch.logspace(-2, 3, S)[:, None]
    x[:, :7] *= 50
    return x.to(torch.bfloat16)


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "comfyui_nodes", "h3-fuse-graph"))
    sys.path.insert(0, os.path.join(ref_root, "comfyui_nodes", "h3-linear-fast"))
    import triton
    import h3_fuse_kernels as fk
    import int8_gemm_triton as tg

    kern = tg._int8_mm_scaled_kernel.fn  # the jitted kernel under the autotuner

    # ---------------- INT8 GEMM + dequant epilogue
    gemm_cases = [("gemm_small", 40, 48, 256, 127, 0), ("gemm_bigacc", 24, 40, 2048, 127, 100)]
    for name, M, N, K, hi, lo in gemm_cases:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        if lo:
            # magnitudes in [lo, hi], one sign per row: |acc| exceeds 2^24, so
            # float(acc) itself rounds
            mag = torch.randint(lo, hi + 1, (M, K), generator=g)
            mag[1::2] *= -1
            xq = mag.to(torch.int8)
            w = torch.randint(lo, hi + 1, (N, K), generator=g).to(torch.int8)
        else:
            xq = torch.randint(-hi, hi + 1, (M, K), generator=g, dtype=torch.int8)
            w = torch.randint(-hi, hi + 1, (N, K), generator=g, dtype=torch.int8)
        xs = (torch.rand(M, 1, generator=g) * 0.05 + 1e-3).float()
        ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).float()
        out = torch.empty(M, N, dtype=torch.bfloat16)
        BM, BN, BK = 16, 16, 64
        grid = (triton.cdiv(M, BM) * triton.cdiv(N, BN),)
        kern[grid](xq, w, out, xs, ws, M, N, K, 1, xq.stride(0), w.stride(0), out.stride(0),
                   BM=BM, BN=BN, BK=BK, GROUP_M=8)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), xq=xq.numpy(), w=w.numpy(),
                            xs=xs.numpy().reshape(-1), ws=ws.numpy(), out=bits(out))
        print(name, M, N, K)

    # ---------------- fused norm / modulation / gate kernels
    norm_cases = [("norm_d1024", 6, 1024, 3, 1e-6, False), ("norm_d5120_adv", 4, 5120, 2, 1e-5, True),
                  ("norm_d1000_tail", 5, 1000, 3, 1e-6, False)]
    for name, S, D, R, eps, adv in norm_cases:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        x = adversarial_rows(g, S, D) if adv else torch.randn(S, D, generator=g).to(torch.bfloat16)
        o = torch.randn(S, D, generator=g).to(torch.bfloat16)
        w = (1 + 0.3 * torch.randn(D, generator=g)).to(torch.bfloat16)
        scale = (0.1 * torch.randn(R, D, generator=g)).to(torch.bfloat16)
        shift = (0.1 * torch.randn(R, D, generator=g)).to(torch.bfloat16)
        gate = (0.1 * torch.randn(R, D, generator=g)).to(torch.bfloat16)
        s1 = (1.0 + scale.to(torch.bfloat16)).contiguous()      # h3_fuse_patch.py:113,116
        ridx = torch.randint(0, R, (S,), generator=g, dtype=torch.int32)
        h_nm = fk.norm_mod(x, w, eps, ridx, s1, shift)
        x_g = x.clone()
        h_gnm = fk.gate_norm_mod_(x_g, o, gate, w, eps, ridx, s1, shift)
        x_gate = x.clone()
        fk.gate_(x_gate, o, gate, ridx)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), x=bits(x), o=bits(o), w=bits(w),
                            scale=bits(scale), shift=bits(shift), gate=bits(gate), s1=bits(s1),
                            ridx=ridx.numpy(), eps=np.float32(eps), h_norm_mod=bits(h_nm),
                            x_gate_norm_mod=bits(x_g), h_gate_norm_mod=bits(h_gnm), x_gate=bits(x_gate))
        print(name, S, D)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("H3_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference project root> (or set H3_REFERENCE_ROOT)")
    main(root)
