"""ratchet_b200 - a B200-native (sm_100a) block-scaled FP4 grouped GEMM.

Drop-in for the reference operator `fp4_grouped_gemm(a, a_sf, b, b_sf, m_indices)`
(kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788) plus the NVFP4 x NVFP4
per-group-list operator `nvfp4_grouped_gemm`, both on one hand-written tcgen05
kernel behind the C ABI in include/fgg_api.h.
"""
from ._lib import FggError
from .ops import (WeightPack, clear_caches, fp4_grouped_gemm, interleave_gate_up, last_status,
                  nvfp4_expert_mlp, nvfp4_grouped_gemm, nvfp4_grouped_gemm_rows,
                  nvfp4_grouped_gemm_silu_mul, pack_weights, quantize_nvfp4)

__all__ = ["fp4_grouped_gemm", "nvfp4_grouped_gemm", "nvfp4_grouped_gemm_rows",
           "nvfp4_grouped_gemm_silu_mul",
           "interleave_gate_up", "nvfp4_expert_mlp", "pack_weights", "WeightPack",
           "quantize_nvfp4", "last_status", "clear_caches", "FggError"]
__version__ = "0.2.0"
