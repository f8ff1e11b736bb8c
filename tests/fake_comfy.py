"""A stand-in for ComfyUI's comfy.ldm.minimax.model.DiTBlock (not part of the
reference, not installable here) for the installer tests: the attributes the
fused forward reads (norm1/norm2 with eps, normalized_shape and weight,
adaln_proj, attn, mlp) and an eager forward in the order the reference's
docstring gives (h3_fuse_kernels.py:3-7): F.rms_norm -> *(1+scale) -> +shift,
attention, x += o*gate, norm again, mlp, x += o*gate."""
import types

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


class Norm:
    def __init__(self, w, eps):
        self.weight, self.eps = w, eps
        self.normalized_shape = (w.numel(),)
        self.comfy_cast_weights = False
        self.weight_function, self.bias_function = [], []


def _ridx(mod_segments, s, device):
    # rows no segment covers get table row 0, so every index stays in range
    r = torch.zeros(s, dtype=torch.long, device=device)
    for a, b, row in mod_segments:
        r[a:b] = row.to(device) if torch.is_tensor(row) else int(row)
    return r


class DiTBlock:
    def __init__(self, D, R, device, seed):
        g = torch.Generator().manual_seed(seed)
        self.norm1 = Norm((1 + 0.02 * torch.randn(D, generator=g)).to(BF16).to(device), 1e-6)
        self.norm2 = Norm((1 + 0.02 * torch.randn(D, generator=g)).to(BF16).to(device), 1e-6)
        self.e = (0.1 * torch.randn(R, 6, D, generator=g)).to(BF16).to(device)
        self.calls = 0

    def adaln_proj(self, t_emb):
        return tuple(self.e[:, i] for i in range(6))

    def attn(self, h, rope_freqs=None, transformer_options=None):
        return (h.float() * 0.75 - 0.1).to(BF16)

    def mlp(self, h):
        return torch.tanh(h.float() * 1.5).to(BF16)

    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}, attention=None):  # noqa: B006
        self.calls += 1
        attention = self.attn if attention is None else attention
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(t_emb)
        r = _ridx(mod_segments, x.shape[0], x.device)
        D = x.shape[1]
        h = F.rms_norm(x, (D,), self.norm1.weight, self.norm1.eps) * (1.0 + scale_msa.to(BF16))[r] + \
            shift_msa.to(BF16)[r]
        o = attention(h, rope_freqs=rope_freqs, transformer_options=transformer_options)
        x.addcmul_(o, gate_msa.to(BF16)[r])
        h = F.rms_norm(x, (D,), self.norm2.weight, self.norm2.eps) * (1.0 + scale_mlp.to(BF16))[r] + \
            shift_mlp.to(BF16)[r]
        o = self.mlp(h)
        x.addcmul_(o, gate_mlp.to(BF16)[r])
        return x


def module():
    """A fresh fake comfy.ldm.minimax.model module object."""
    return types.SimpleNamespace(DiTBlock=type("DiTBlock", (DiTBlock,), {}))
