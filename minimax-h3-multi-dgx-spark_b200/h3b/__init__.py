"""h3b -- B200-native (sm_100a) H3 video-DiT hot path.

Drop-in replacements for the three hooks of yuichi-suzuki-highdrama/minimax-h3-multi-dgx-spark:
  * INT8 linear            h3b.linear   (h3-linear-fast)
  * fused norm/mod/gate    h3b.fuse     (h3-fuse-graph)
  * Ulysses all-to-all     h3b.sp       (minimax-h3-sp)
All compute runs in libh3b.so (hand-written CUDA for sm_100a, C ABI in
include/h3b.h); this package is the host-side mirror of the reference's
operator interfaces.  Importing it fails if the library is not built.
h3b.model holds the synthetic DiT block / step that drives the path in the
benchmark and HostPipeline, the host-latent runner.
"""
from ._lib import H3BError, clear_status, lib, status  # noqa: F401
from .fuse import (gate_, gate_norm_mod_, gate_norm_mod_quant_, modulation_tables, norm_mod,  # noqa: F401
                   norm_mod_quant, rms_norm, row_index)
from .linear import (gelu_quant, gelu_tanh, int8_linear, int8_mm_i32, int8_mm_scaled, int8_mm_scaled_a2a, linear,  # noqa: F401
                     quant_rowwise, quant_rowwise_convrot, supported, swiglu_quant_convrot)
from .sp import (PeerExchange, SPContext, a2a_gather_qkv, a2a_gather_seq_scatter_heads,  # noqa: F401
                 a2a_scatter_seq_gather_heads, gather_rows, overlap_groups, pack, sp_attention_overlap, startup_probe, unpack)

__all__ = ["H3BError", "status", "clear_status", "norm_mod", "rms_norm", "gate_norm_mod_", "gate_", "row_index",
           "norm_mod_quant", "gate_norm_mod_quant_", "gelu_quant", "gelu_tanh",
           "modulation_tables", "quant_rowwise", "quant_rowwise_convrot", "swiglu_quant_convrot", "int8_mm_scaled", "int8_mm_scaled_a2a", "int8_mm_i32", "int8_linear",
           "linear",
           "supported", "SPContext", "PeerExchange", "a2a_gather_seq_scatter_heads", "a2a_scatter_seq_gather_heads",
           "a2a_gather_qkv", "sp_attention_overlap", "overlap_groups", "gather_rows", "pack", "unpack", "startup_probe"]
