"""The flow-free TTT pre-pass kernels under the reference's names
(vggt_omega/utils/ttt_kernels.py): descriptor normalisation, exact-window local top-2 matching,
the integer border warp, fused motion cues and fused sensitivity labels, each one sm_100a
launch through the C ABI (``vb200_row_l2_normalize`` ... ``vb200_sensitivity_labels``).

Signatures, output layouts and exception types follow the reference wrappers; nothing here
computes on the CPU (``RuntimeError`` for non-CUDA tensors).
"""
from __future__ import annotations

import torch

from . import _clib as C

__all__ = [
    "kernels_ready",
    "normalize_rows",
    "local_top2_match",
    "integer_gather_warp",
    "fused_motion_cues",
    "fused_sensitivity_labels",
]


def kernels_ready(value: torch.Tensor) -> bool:
    """True when ``value`` lives on a CUDA device (the reference's ``triton_ready``)."""
    return value.is_cuda


def normalize_rows(value: torch.Tensor) -> torch.Tensor:
    """fp32 rows divided by max(L2 norm, 1e-6), one launch (ttt_kernels.py:233-249; the
    reference's default path is ``F.normalize(value.float(), dim=-1, eps=1e-6)``)."""
    C.require_cuda(value, "normalize_rows")
    flat = value.reshape(-1, value.shape[-1]).contiguous()
    out = torch.empty(flat.shape, device=flat.device, dtype=torch.float32)
    rc = C.lib().vb200_row_l2_normalize(C.dtype_code(flat.dtype), flat.data_ptr(), flat.shape[0], flat.shape[1],
                                        1e-6, out.data_ptr(), C.stream_of(flat.device))
    C.check(rc, "normalize_rows")
    return out.reshape(value.shape)


def local_top2_match(source: torch.Tensor, target: torch.Tensor, radius_y: int, radius_x: int, *,
                     reverse_order: bool = False):
    """Exact-window cosine top-2 of ``[pairs,H,W,C]`` descriptors (ttt_kernels.py:252-277):
    -> (best, second, dy, dx), each ``[pairs,H,W]`` (fp32, fp32, int64, int64)."""
    if not source.is_cuda:
        raise RuntimeError("local_top2_match requires CUDA tensors on an sm_100 device (no CPU fallback)")
    if source.shape != target.shape or source.ndim != 4:
        raise ValueError("source and target descriptors must share [pairs,H,W,C]")
    pairs, H, W, Cd = source.shape
    rows = pairs * H * W
    source = source.contiguous()
    target = target.to(source.dtype).contiguous()
    dev = source.device
    best = torch.empty(rows, device=dev, dtype=torch.float32)
    second = torch.empty_like(best)
    dy = torch.empty(rows, device=dev, dtype=torch.int32)
    dx = torch.empty_like(dy)
    rc = C.lib().vb200_local_top2_match(
        C.dtype_code(source.dtype), source.data_ptr(), target.data_ptr(), pairs, H, W, Cd, int(radius_y),
        int(radius_x), int(bool(reverse_order)), best.data_ptr(), second.data_ptr(), dy.data_ptr(), dx.data_ptr(),
        C.stream_of(dev))
    C.check(rc, "local_top2_match")
    shape = (pairs, H, W)
    return best.view(shape), second.view(shape), dy.view(shape).long(), dx.view(shape).long()


def integer_gather_warp(field: torch.Tensor, flow: torch.Tensor) -> torch.Tensor:
    """Border-clamped integer warp, equal to align-corners border ``grid_sample`` at integer
    flow (ttt_kernels.py:280-297)."""
    if not field.is_cuda:
        raise RuntimeError("integer_gather_warp requires CUDA tensors on an sm_100 device (no CPU fallback)")
    if field.ndim != 4 or flow.shape != (*field.shape[:3], 2):
        raise ValueError("field/flow must be [B,H,W,C] and [B,H,W,2]")
    B, H, W, Cd = field.shape
    field = field.contiguous()
    flow = flow.to(torch.float32).contiguous()
    out = torch.empty_like(field)
    rc = C.lib().vb200_integer_warp(C.dtype_code(field.dtype), field.data_ptr(), flow.data_ptr(), B, H, W, Cd,
                                    out.data_ptr(), C.stream_of(field.device))
    C.check(rc, "integer_gather_warp")
    return out


def fused_motion_cues(forward_flow: torch.Tensor, backward_flow: torch.Tensor, predicted: torch.Tensor,
                      forward_confidence: torch.Tensor, backward_confidence: torch.Tensor):
    """Residual aggregation, confidence propagation and 3x3 boundaries in one launch
    (ttt_kernels.py:300-318) -> (residual, confidence, boundary), each ``[F,H,W]`` fp32."""
    if not predicted.is_cuda:
        raise RuntimeError("fused_motion_cues requires CUDA tensors on an sm_100 device (no CPU fallback)")
    F, H, W, channels = predicted.shape
    if channels != 4:
        raise ValueError("predicted motion must have four channels")
    f32 = lambda t: t.to(torch.float32).contiguous()
    ff, bf, pr, fc, bc = (f32(t) for t in (forward_flow, backward_flow, predicted, forward_confidence,
                                           backward_confidence))
    if F > 1 and (ff.shape != (F - 1, H, W, 2) or bf.shape != ff.shape or fc.shape != (F - 1, H, W)
                  or bc.shape != fc.shape):
        raise ValueError("flows must be [F-1,H,W,2] and confidences [F-1,H,W]")
    outs = [torch.empty((F, H, W), device=pr.device, dtype=torch.float32) for _ in range(3)]
    rc = C.lib().vb200_motion_cues(ff.data_ptr(), bf.data_ptr(), pr.data_ptr(), fc.data_ptr(), bc.data_ptr(), F, H,
                                   W, *(o.data_ptr() for o in outs), C.stream_of(pr.device))
    C.check(rc, "fused_motion_cues")
    return tuple(outs)


def fused_sensitivity_labels(residual: torch.Tensor, confidence: torch.Tensor, boundary: torch.Tensor, *,
                             uncertain_confidence: float, residual_scale: torch.Tensor, boundary_scale: torch.Tensor,
                             residual_threshold: torch.Tensor, boundary_threshold: torch.Tensor):
    """Cue normalisation, sensitivity and the preliminary label predicates in one launch
    (ttt_kernels.py:321-341) -> (sensitivity fp32, low_confidence bool, raw_event bool)."""
    if not residual.is_cuda:
        raise RuntimeError("fused_sensitivity_labels requires CUDA tensors on an sm_100 device (no CPU fallback)")
    F, H, W = residual.shape
    dev = residual.device
    f32 = lambda t: t.to(torch.float32).contiguous()
    scalar = lambda t: torch.as_tensor(t, dtype=torch.float32, device=dev).reshape(1).contiguous()
    res, conf, bnd = f32(residual), f32(confidence), f32(boundary)
    rs, bs, rt, bt = (scalar(t) for t in (residual_scale, boundary_scale, residual_threshold, boundary_threshold))
    sens = torch.empty((F, H, W), device=dev, dtype=torch.float32)
    low = torch.empty((F, H, W), device=dev, dtype=torch.int8)
    event = torch.empty_like(low)
    rc = C.lib().vb200_sensitivity_labels(
        res.data_ptr(), conf.data_ptr(), bnd.data_ptr(), residual.numel(), H * W, float(uncertain_confidence),
        rs.data_ptr(), bs.data_ptr(), rt.data_ptr(), bt.data_ptr(), sens.data_ptr(), low.data_ptr(), event.data_ptr(),
        C.stream_of(dev))
    C.check(rc, "fused_sensitivity_labels")
    return sens, low.bool(), event.bool()
