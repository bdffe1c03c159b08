"""loki_b200: B200-native (sm_100a) DeepSeek-R1 MoE layer behind loki's fused-layer MoE ABI.

The compute lives in libloki_moe.so (CUDA kernels + C ABI, include/loki_moe.h and
include/loki_fused_moe.h); this package is its host-side Python mirror.  Build with
`python -m loki_b200.build`.
"""
from .native import HIDDEN, MOE_INTER, N_EXPERTS, EXPERT_MATRIX_BYTES, lib  # noqa: F401

__all__ = ["HIDDEN", "MOE_INTER", "N_EXPERTS", "EXPERT_MATRIX_BYTES", "lib"]
