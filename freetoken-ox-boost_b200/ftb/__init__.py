"""ftb - a B200-native (sm_100a) NVFP4 fused-MoE layer with FreeToken's MoE backend API.

Host code is Python/PyTorch; all device work runs in ``libftb.so`` (hand-written CUDA,
C ABI in ``include/ftb.h``), loaded through ctypes. There is no CPU or Triton fallback.
"""
from .banks import Nvfp4Bank, bank_bytes_per_expert
from .checkpoint import bank_from_modelopt, bank_to_modelopt, moe_layers_in
from .ds_fp4 import DsFp4Bank, fused_experts_ds_fp4, nvfp4_from_ds_fp4
from .ep import EpGroup, ExpertParallelMoE
from .experts import B200Nvfp4Experts, Nvfp4MoELayer, select_nvfp4_backend
from .fused_nvfp4 import (fused_experts_decode_nvfp4_marlin, fused_experts_decode_nvfp4_split,
                          fused_experts_nvfp4, moe_align_block_size, moe_decode, moe_prefill,
                          moe_prefill_fp4, quant_nvfp4)
from .fused_route import fused_route, fused_route_ranked, fused_topk, router_logits

__all__ = [
    "Nvfp4Bank", "bank_bytes_per_expert", "B200Nvfp4Experts", "Nvfp4MoELayer",
    "select_nvfp4_backend", "fused_experts_decode_nvfp4_marlin",
    "fused_experts_decode_nvfp4_split", "fused_experts_nvfp4",
    "moe_align_block_size", "moe_decode", "moe_prefill", "moe_prefill_fp4", "quant_nvfp4",
    "fused_route", "fused_route_ranked", "fused_topk", "router_logits",
    "bank_from_modelopt", "bank_to_modelopt", "moe_layers_in", "EpGroup", "ExpertParallelMoE",
    "DsFp4Bank", "fused_experts_ds_fp4", "nvfp4_from_ds_fp4",
]
