"""dsv41_flash_offload_b200: B200-native routed-expert MoE FFN over EXL3 3.0-bpw mul1 weights.

A drop-in for the reference (0xSero/dsv41-flash-offload) hot path behind its own entry points:
  exl3.apply_exl3_fused_moe   the vllm_exl3 fused-MoE op (patches/vllm-exl3-host-dma.patch:203-449)
  dma_gemm.run_batch          runtime/dma_gemm.py's busy-expert GEMM
  tier.tier_forward           the CPU-tier expert call (kernels/cpu_avx2/ft_tier_ext.cpp:177-191)
backed by hand-written sm_100a kernels in libdsv41_b200.so (C ABI: include/dsv41_b200.h).
"""
from .exl3 import (Exl3MoELayer, apply_exl3_experts, apply_exl3_fused_moe, combine, decode_dense,  # noqa: F401
                   permute, read_status, workspace_bytes, FAT_EXPERT_THRESHOLD, SWIGLU_LIMIT_DEFAULT)
from ._lib import Dsv41Error, load as load_library  # noqa: F401

__all__ = ["Exl3MoELayer", "apply_exl3_fused_moe", "apply_exl3_experts", "permute", "combine", "decode_dense",
           "read_status", "workspace_bytes", "load_library", "Dsv41Error"]
