"""trials_b200: FP8 128x128 block-scaled Mixture-of-Experts layer for NVIDIA B200.

Hand-written sm_100a CUDA kernels (TMA + tcgen05/TMEM grouped GEMMs, warp-scan
routing, fused quantisation) behind a C ABI (include/b200moe.h), with a Python
surface that mirrors the reference's drop-in calls.
"""
from .moe import (  # noqa: F401
    ActivationType,
    QuantType,
    _moe_decode_megakernel_full,
    expert_map_from_mask,
    fused_moe,
    layer_error_word,
    moe_align_block_size,
    moe_decode_megakernel_full,
    per_block_quant_fp8,
    per_token_group_quant_fp8,
    read_device_error,
    select_experts,
)

__version__ = "0.1.0"
