"""gdn_b200: the Qwen3.5 gated-delta (GatedDeltaNet) operator on NVIDIA B200.

Python host side of libgdn_b200.so (hand-written sm_100a CUDA behind the C
ABI in include/gdn_api.h). The public API mirrors the reference
conferencebeefwood46/mlx-lean-moe's ``qwen3_5.gated_delta`` module and its
``RecurrentCache``; CUDA tensors replace MLX arrays.
"""

from .gated_delta import (
    DecodePlan,
    check_device_errors,
    forget_gate,
    gated_delta_decode,
    gated_delta_scan,
    gated_delta_scan_varlen,
    gated_delta_step,
)
from .attention import AttentionShape, GrowingKVCache, Qwen3_5Attention, attention_core
from .linear_attention import LinearAttentionShape, Qwen3_5LinearAttention, gated_delta_block
from .quantized import LinearWeights, QuantScheme, as_linear, concat_rows, dequantize, quantized_linear
from .recurrent_cache import BatchedRecurrentCache, RecurrentCache

__all__ = [
    "AttentionShape",
    "BatchedRecurrentCache",
    "GrowingKVCache",
    "Qwen3_5Attention",
    "attention_core",
    "DecodePlan",
    "LinearAttentionShape",
    "LinearWeights",
    "QuantScheme",
    "Qwen3_5LinearAttention",
    "RecurrentCache",
    "as_linear",
    "check_device_errors",
    "concat_rows",
    "dequantize",
    "forget_gate",
    "gated_delta_block",
    "gated_delta_decode",
    "gated_delta_scan",
    "gated_delta_scan_varlen",
    "gated_delta_step",
    "quantized_linear",
]
