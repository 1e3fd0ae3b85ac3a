"""numpy restatement of the flow-free TTT pre-pass (TEST ORACLE): descriptor normalisation,
exact-window local top-2 matching and the correspondences built on it, the integer border
warp, motion cues and sensitivity labels.

  * normalize_rows       vggt_omega/utils/ttt_kernels.py:233-249 (F.normalize, eps 1e-6)
  * local_top2_match     ttt_kernels.py:45-101 / :252-277 (row-major candidate offsets,
                         reversed for the backward match; strict '>' keeps the first maximum)
  * correspondences      vggt_omega/utils/token_matching.py:353-498 (forward / backward top-2,
                         cycle error, confidence = similarity x margin x cycle term)
  * integer_warp         ttt_kernels.py:104-127 / :280-297
  * motion_cues          ttt_kernels.py:130-196 / :300-318
  * sensitivity_labels   ttt_kernels.py:199-230 / :321-341

Dot products run in float64 over float32 inputs; everything else in float32 as the reference.
Pinned by tests/test_oracle_golden.py against outputs of the reference's own CPU code
(tests/golden/make_golden.py).  TEST INFRASTRUCTURE ONLY: imported by tests/ and never by the
product package.
"""
from __future__ import annotations

import numpy as np

__all__ = ["normalize_rows", "local_top2_match", "correspondences", "integer_warp", "motion_cues",
           "sensitivity_labels"]


def normalize_rows(x, eps: float = 1e-6) -> np.ndarray:
    """x / max(||x||_2, eps) along the last axis, float32."""
    x = np.asarray(x, dtype=np.float32)
    norm = np.sqrt(np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)).astype(np.float32)
    return (x / np.maximum(norm, np.float32(eps))).astype(np.float32)


def _offsets(ry: int, rx: int, reverse: bool) -> list[tuple[int, int]]:
    out = [(oy, ox) for oy in range(-ry, ry + 1) for ox in range(-rx, rx + 1)]
    return [(-oy, -ox) for oy, ox in out] if reverse else out


def local_top2_match(source, target, radius_y: int, radius_x: int, reverse_order: bool = False):
    """source/target [pairs, H, W, C] -> (best, second float64, dy, dx int64), each [pairs, H, W].
    Candidates outside the grid score -inf; a candidate becomes the best only when strictly
    greater; second = the old best on replacement, else max(second, candidate)."""
    s = np.asarray(source, dtype=np.float64)
    t = np.asarray(target, dtype=np.float64)
    P, H, W, _ = s.shape
    best = np.full((P, H, W), -np.inf)
    second = np.full((P, H, W), -np.inf)
    dy = np.zeros((P, H, W), np.int64)
    dx = np.zeros((P, H, W), np.int64)
    yy, xx = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    for oy, ox in _offsets(radius_y, radius_x, reverse_order):
        ty, tx = yy + oy, xx + ox
        inside = (ty >= 0) & (ty < H) & (tx >= 0) & (tx < W)
        sim = np.einsum("phwc,phwc->phw", s, t[:, np.clip(ty, 0, H - 1), np.clip(tx, 0, W - 1)])
        sim = np.where(inside[None], sim, -np.inf)
        better = sim > best
        second = np.where(better, best, np.maximum(second, sim))
        best = np.where(better, sim, best)
        dy = np.where(better, oy, dy)
        dx = np.where(better, ox, dx)
    return best, second, dy, dx


def correspondences(descriptors, search_radius: int = 4, minimum_similarity: float = .35, cycle_scale: float = 1.5):
    """descriptors [T, H, W, C] -> forward_flow, backward_flow [T-1, H, W, 2] (dx, dy; float32)
    and forward / backward confidence [T-1, H, W] (float32)."""
    d = np.asarray(descriptors, dtype=np.float32)
    T, H, W, _ = d.shape
    ry, rx = min(search_radius, H - 1), min(search_radius, W - 1)
    fb, fs, fdy, fdx = local_top2_match(d[:-1], d[1:], ry, rx)
    bb, bs, bdy, bdx = local_top2_match(d[1:], d[:-1], ry, rx, reverse_order=True)
    yy, xx = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    p = np.arange(T - 1)[:, None, None]
    fty, ftx = np.clip(yy + fdy, 0, H - 1), np.clip(xx + fdx, 0, W - 1)
    fcycle = np.sqrt(((fdy + bdy[p, fty, ftx]) ** 2 + (fdx + bdx[p, fty, ftx]) ** 2).astype(np.float32))
    bsy, bsx = np.clip(yy + bdy, 0, H - 1), np.clip(xx + bdx, 0, W - 1)
    bcycle = np.sqrt(((bdy + fdy[p, bsy, bsx]) ** 2 + (bdx + fdx[p, bsy, bsx]) ** 2).astype(np.float32))

    def confidence(best, second, cycle):
        best, second = best.astype(np.float32), second.astype(np.float32)
        sim = np.clip((best - np.float32(minimum_similarity)) / np.float32(1.0 - minimum_similarity), 0, 1)
        margin = 1.0 / (1.0 + np.exp(-(((best - second) - np.float32(.005)) / np.float32(.01))))
        cyc = np.exp(np.float32(-.5) * (cycle / np.float32(cycle_scale)) ** 2)
        return np.clip(sim * margin * cyc, 0, 1).astype(np.float32)

    fflow = np.stack([fdx, fdy], -1).astype(np.float32)
    bflow = np.stack([bdx, bdy], -1).astype(np.float32)
    return fflow, bflow, confidence(fb, fs, fcycle), confidence(bb, bs, bcycle)


def integer_warp(field, flow) -> np.ndarray:
    """field [B, H, W, C], flow [B, H, W, 2] (x, y) -> field sampled at the border-clamped
    position (x + trunc(flow_x), y + trunc(flow_y))."""
    field = np.asarray(field)
    flow = np.asarray(flow, dtype=np.float32)
    B, H, W, _ = field.shape
    yy, xx = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
    sx = np.clip(xx[None] + np.trunc(flow[..., 0]).astype(np.int64), 0, W - 1)
    sy = np.clip(yy[None] + np.trunc(flow[..., 1]).astype(np.int64), 0, H - 1)
    return field[np.arange(B)[:, None, None], sy, sx]


def _box_mean(v: np.ndarray) -> np.ndarray:
    """3 x 3 zero-padded mean of v [F, H, W], each term divided by 9 before the sum, summed in
    row-major offset order (float32)."""
    F, H, W = v.shape
    pad = np.zeros((F, H + 2, W + 2), np.float32)
    pad[:, 1:-1, 1:-1] = v
    acc = np.zeros((F, H, W), np.float32)
    for oy in range(3):
        for ox in range(3):
            acc = (acc + pad[:, oy:oy + H, ox:ox + W] / np.float32(9.0)).astype(np.float32)
    return acc


def motion_cues(forward_flow, backward_flow, predicted, forward_conf, backward_conf):
    """-> residual, confidence, boundary [F, H, W] float32 (F = predicted frames)."""
    pred = np.asarray(predicted, dtype=np.float32)
    F, H, W, _ = pred.shape
    ff = np.zeros((F, H, W, 2), np.float32)
    bf = np.zeros((F, H, W, 2), np.float32)
    fc = np.ones((F, H, W), np.float32)
    bc = np.ones((F, H, W), np.float32)
    has_f = np.zeros((F, 1, 1), bool)
    has_b = np.zeros((F, 1, 1), bool)
    if F > 1:
        ff[:-1] = forward_flow
        bf[1:] = backward_flow
        fc[:-1] = forward_conf
        bc[1:] = backward_conf
        has_f[:-1] = True
        has_b[1:] = True
    pf = np.where(has_f[..., None], pred[..., :2], 0).astype(np.float32)
    pb = np.where(has_b[..., None], pred[..., 2:], 0).astype(np.float32)
    hyp = lambda a: np.sqrt(a[..., 0] ** 2 + a[..., 1] ** 2).astype(np.float32)
    f_res, b_res = hyp(ff - pf), hyp(bf - pb)
    count = has_f.astype(np.float32) + has_b.astype(np.float32)
    fm = np.stack([_box_mean(ff[..., 0]), _box_mean(ff[..., 1])], -1)
    bm = np.stack([_box_mean(bf[..., 0]), _box_mean(bf[..., 1])], -1)
    f_bnd, b_bnd = hyp(ff - fm), hyp(bf - bm)
    denom = np.maximum(count, 1).astype(np.float32)
    return ((f_res + b_res) / denom).astype(np.float32), np.minimum(fc, bc), ((f_bnd + b_bnd) / denom).astype(np.float32)


def sensitivity_labels(residual, confidence, boundary, *, uncertain_confidence, residual_scale, boundary_scale,
                       residual_threshold, boundary_threshold):
    """-> sensitivity float32, low_confidence bool, raw_event bool, each [F, H, W]."""
    res = np.asarray(residual, np.float32)
    conf = np.asarray(confidence, np.float32)
    bnd = np.asarray(boundary, np.float32)
    F = res.shape[0]
    later = (np.arange(F) > 0)[:, None, None]
    novelty = np.float32(1) - conf
    ru = np.clip(res / max(np.float32(residual_scale), np.float32(1e-6)), 0, 1)
    bu = np.clip(bnd / max(np.float32(boundary_scale), np.float32(1e-6)), 0, 1)
    sens = np.clip(np.float32(.45) * novelty + np.float32(.35) * ru + np.float32(.20) * bu, 0, 1).astype(np.float32)
    uc = np.float32(uncertain_confidence)
    low = later & (conf < uc)
    event = later & (((res >= np.float32(residual_threshold)) & (conf >= uc)) | (bnd >= np.float32(boundary_threshold))
                     | (novelty >= np.float32(.55)))
    return sens, low, event
