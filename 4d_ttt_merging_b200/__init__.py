"""B200-native (sm_100a) token-merged global attention for VGGT-Omega.

A drop-in for the Triton kernels and token-plan reductions of shuang-yang18/4D_TTT_merging:
the merge step (cosine-similarity GEMM with fused argmax / top-4), mass-bias attention
(tcgen05 tensor cores, TMEM accumulators, TMA tiles) and the top-4 sparse-convex projection
in both directions (CSR-segmented, atomics-free).  The host layer below keeps the reference's
names, arguments and exceptions; every computation runs in ``_lib/libvggt_b200.so`` through
its C ABI (``include/vggt_b200.h``).  There is no CPU fallback.

The package directory name starts with a digit, so import it with
``importlib.import_module("4d_ttt_merging_b200")``.
"""
from __future__ import annotations

from . import _clib
from ._clib import device_error_flags, library_path
from .ops import (
    PlanCSR,
    build_plan_csr,
    deterministic_weighted_normalizer,
    four_support_active_set,
    four_support_projected_gradient,
    mass_bias_attention,
    mass_bias_attention_into,
    merge_argmax,
    row_gather,
    row_normalize_bf16,
    similarity_topk,
    streaming_top4,
)
from .token_plan import TokenPlan, WeightedBilinearTokenPlan
from .planners import build_fastvggt_plan, build_ttt_protected_uniform_convex_plan, build_uniform_convex_plan
from .attention_block import GlobalAttention, compute_attention
from .install import install, uninstall
from . import parallel, ttt_kernels

__all__ = [
    "GlobalAttention",
    "PlanCSR",
    "build_fastvggt_plan",
    "build_ttt_protected_uniform_convex_plan",
    "build_uniform_convex_plan",
    "compute_attention",
    "install",
    "uninstall",
    "TokenPlan",
    "WeightedBilinearTokenPlan",
    "build_plan_csr",
    "deterministic_weighted_normalizer",
    "device_error_flags",
    "four_support_active_set",
    "four_support_projected_gradient",
    "library_path",
    "mass_bias_attention",
    "mass_bias_attention_into",
    "merge_argmax",
    "row_gather",
    "row_normalize_bf16",
    "similarity_topk",
    "streaming_top4",
]


def load_library():
    """Load the shared library now (raises RuntimeError when it has not been built)."""
    return _clib.lib()
