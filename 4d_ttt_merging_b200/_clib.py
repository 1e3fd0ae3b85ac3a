"""ctypes binding of ``libvggt_b200.so`` (the C ABI declared in ``include/vggt_b200.h``).

The library is loaded from ``_lib/`` inside this package; there is no fallback. Status codes
are mapped to the exception types the reference raises: ``VB200_EINVAL`` -> ``ValueError``,
everything else -> ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libvggt_b200.so"

F32, BF16, F16 = 0, 1, 2
EINVAL, ECUDA, EUNSUPPORTED = -1, -2, -3

_DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float
_p_i64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes)
_SIGNATURES = {
    "vb200_version": (_c_int, []),
    "vb200_last_error": (ctypes.c_char_p, []),
    "vb200_launch_count": (ctypes.c_ulonglong, []),
    "vb200_device_error_flags": (_c_int, [ctypes.POINTER(ctypes.c_uint), _c_int]),
    "vb200_mass_bias_attention_workspace_size": (_c_size, [_c_i64]),
    "vb200_mass_bias_attention_split_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "vb200_mass_bias_attention_plan": (_c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_int, _p_i64]),
    "vb200_sim_topk_split": (_c_int, [_c_i64, _c_int, _c_int]),
    "vb200_mass_bias_attention": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _p_i64, _p_i64, _p_i64, _p_i64, _c_vp, _c_size, _c_vp],
    ),
    "vb200_mass_bias_attention_noalloc": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _p_i64, _p_i64, _p_i64, _p_i64, _c_vp],
    ),
    "vb200_exp2_poly": (_c_int, [_c_vp, _c_vp, _c_i64, _c_vp]),
    "vb200_plan_csr_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "vb200_plan_csr_build": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_size, _c_vp],
    ),
    "vb200_plan_csr_build_grouped": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_vp, _c_vp],
    ),
    "vb200_proj_scatter": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp],
    ),
    "vb200_proj_scatter_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "vb200_qkv_head_stats": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_float, _c_vp, _c_size, _c_vp]),
    "vb200_geometry_shortlist": (
        _c_int, [_c_vp, _c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_i64, _c_float, _c_vp, _c_vp, _c_vp, _c_vp],
    ),
    "vb200_geometry_guard": (
        _c_int,
        [_c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_float, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp],
    ),
    "vb200_row_l2_normalize": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_float, _c_vp, _c_vp]),
    "vb200_local_top2_match": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_vp],
    ),
    "vb200_integer_warp": (_c_int, [_c_int, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp]),
    "vb200_motion_cues": (
        _c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp],
    ),
    "vb200_sensitivity_labels": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_float, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp],
    ),
    "vb200_proj_scatter_numerators": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_size,
         _c_vp],
    ),
    "vb200_rank_reduce_rows": (
        _c_int, [_c_int, _c_vp, _c_int, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_vp],
    ),
    "vb200_compact_qkv_workspace_size": (_c_size, [_c_i64, _c_i64]),
    "vb200_compact_qkv": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_float, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp,
         _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_vp, _c_size, _c_vp],
    ),
    "vb200_compact_qkv_peer": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_float, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp,
         _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_vp, _c_int, _c_int, _c_i64, _c_i64, _c_vp, _c_size, _c_vp],
    ),
    "vb200_head_layernorm": (
        _c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_float, _c_vp, _c_i64, _c_vp],
    ),
    "vb200_proj_gather": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64,
         _c_i64, _c_i64, _c_int, _c_vp],
    ),
    "vb200_plan_hot_rows": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_vp]),
    "vb200_proj_gather_hot_capacity": (_c_int, [_c_int, _c_i64]),
    "vb200_proj_gather_hot": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64,
         _c_vp, _c_vp, _c_vp, _c_int, _c_vp],
    ),
    "vb200_row_gather": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp]),
    "vb200_peer_gather": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_vp, _c_i64, _c_vp]),
    "vb200_peer_push": (_c_int, [_c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_int, _c_i64, _c_i64, _c_vp]),
    "vb200_peer_barrier": (_c_int, [_c_vp, _c_int, _c_int, _c_vp, _c_i64, _c_vp]),
    "vb200_row_normalize_bf16": (
        _c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_float, _c_vp, _c_i64, _c_vp],
    ),
    "vb200_sim_topk": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_i64, _c_vp,
         _c_vp, _c_vp],
    ),
    "vb200_merge_assign_workspace_size": (_c_size, [_c_i64, _c_i64]),
    "vb200_merge_assign": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_size, _c_vp],
    ),
    "vb200_support_fit": (
        _c_int,
        [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_int, _c_vp],
    ),
    "vb200_support_certificate": (
        _c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp],
    ),
    "vb200_row_max_dot": (_c_int, [_c_int, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_int, _c_i64, _c_i64, _c_vp, _c_vp]),
    "vb200_four_support_projected_gradient": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_int, _c_vp]),
    "vb200_four_support_active_set": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_float, _c_vp]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None


def library_path() -> Path:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the shared library once; raise RuntimeError when it has not been built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"{_LIB_PATH} is missing: build it with `python 4d_ttt_merging_b200/build.py` "
                "(there is no CPU fallback)"
            )
        handle = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc == 0:
        return
    msg = lib().vb200_last_error().decode(errors="replace")
    if rc == EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def strides3(t: torch.Tensor):
    return (_c_i64 * 3)(*t.stride()[:3])


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} requires CUDA tensors on an sm_100 device (no CPU fallback)")


def device_error_flags(clear: bool = True) -> int:
    """OR of the kernels' device error words (bit 0: a bounded wait ran out; bit 1: an index
    outside its range).  Synchronises the device."""
    flags = ctypes.c_uint(0)
    check(lib().vb200_device_error_flags(ctypes.byref(flags), int(clear)), "vb200_device_error_flags")
    return int(flags.value)
