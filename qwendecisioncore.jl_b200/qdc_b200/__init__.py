"""qdc_b200 -- host side of libqdc_b200.so, the B200 (sm_100a) implementation
of QwenDecisionCore.jl's fused per-layer kernels.

The package directory `qwendecisioncore.jl_b200/` holds the CUDA sources
(csrc/), the build recipe (build.py), this Python mirror of the reference's
hook interface, and the Julia `ccall` extension for the reference itself
(julia/QwenDecisionCoreB200Ext.jl).  Import it with that directory on
sys.path:  `import qdc_b200`.
"""
from ._lib import (ArgumentError, DimensionMismatch, QdcError, QDC_BF16, QDC_F32,
                   declared_symbols, load)
from .ops import (Context, context, native_attn_gate, native_bf16_to_f32, native_delta_conv_norm,
                  native_delta_gates, native_delta_solve, native_f32_to_bf16,
                  native_gated_rms, native_gather, native_gather_rms, native_mlp_gate,
                  native_q_k_norm_rope, native_qk_norm_rope, native_residual_add_rms,
                  native_residual_rms, native_rms, rope_table)

from .backbone import (QwenBackbone, backbone_hidden, backbone_last_hidden, batch_backbone_hidden,
                       check_sequence)
from .model import Config

__all__ = [
    "QwenBackbone", "backbone_hidden", "backbone_last_hidden", "batch_backbone_hidden",
    "check_sequence", "Config",
    "ArgumentError", "DimensionMismatch", "QdcError", "QDC_BF16", "QDC_F32", "Context", "context",
    "declared_symbols", "load", "native_attn_gate", "native_bf16_to_f32", "native_delta_conv_norm",
    "native_delta_gates", "native_delta_solve", "native_f32_to_bf16",
    "native_gated_rms", "native_gather", "native_gather_rms", "native_mlp_gate",
    "native_q_k_norm_rope", "native_qk_norm_rope", "native_residual_add_rms",
    "native_residual_rms", "native_rms", "rope_table",
]
