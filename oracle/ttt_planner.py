"""numpy restatement of the reference's released merge planner (TEST ORACLE):
``build_ttt_protected_uniform_convex_plan`` (vggt_omega/models/sparse_convex.py:1738-2016) on
its feature-only support route (support_geometry_weight = 0, the function's default) and its
Pareto-guarded geometry route (support_geometry_weight > 0 with a guard tolerance; the released
configuration uses 0.01 and 0).

Pieces, each citing the reference lines it restates:
  * uniform_2x2_tables / cell_table      sparse_convex.py:1327-1368, :1194-1203
  * protected_skeleton                   :1371-1434 (uniform anchors, 4x4 macro-cell top-1 pruning)
  * ttt_event_bases                      :1268-1324 (TTT-proposed residual event bases)
  * fit_temporal_local                   :440-684   (per 8-frame group bf16 top-4, 32-step
                                                     projected gradient, certificate, global fallback)
  * fit_global                           :168-330   (_adaptive_fit_fused, the exact global route)
  * build_plan                           :1738-2016

Features are bf16 values held in float32 arrays; dot products and solves run in float64 (the
reference uses fp32), bf16 score rounding is emulated exactly, and every ranking is a stable
descending sort (ties to the lower index; the reference's torch.topk leaves tie order open).
TEST INFRASTRUCTURE ONLY: imported by tests/ and never by the product package.
"""
from __future__ import annotations

import math

import numpy as np

from . import ref

__all__ = ["cell_table", "uniform_2x2_tables", "protected_skeleton", "ttt_event_bases", "certificate",
           "fit_supports", "geometry_shortlist", "geometry_residual", "guard_choose", "fit_temporal_local", "fit_global", "build_plan", "LOCAL_FRAME_GROUP"]

LOCAL_FRAME_GROUP = 8  # sparse_convex.py:31


def cell_table(height: int, width: int, cell: int) -> np.ndarray:
    """[cells, cell*cell] patch ids of each cell x cell block (row-major), -1 padded
    (sparse_convex.py:1194-1203)."""
    rows = []
    for top in range(0, height, cell):
        for left in range(0, width, cell):
            ids = [y * width + x for y in range(top, min(top + cell, height)) for x in range(left, min(left + cell, width))]
            rows.append(ids + [-1] * (cell * cell - len(ids)))
    return np.asarray(rows, dtype=np.int64)


def uniform_2x2_tables(frames: int, patch_hw):
    """(first [P], positions [F-1, cells2x2], grouped [F-1, macro, 4], first_table [macro, 16]):
    one seeded random patch per 2x2 cell of every later frame (CPU generator, seed 0) grouped into
    4x4 macro cells in position order (sparse_convex.py:1327-1368)."""
    height, width = patch_hw
    patches = height * width
    first = np.arange(patches, dtype=np.int64)
    if frames <= 1:
        e = np.zeros((0, 0, 0), np.int64)
        return first, e, e, e
    rows, cols = np.arange(0, height, 2), np.arange(0, width, 2)
    choice = ref.torch_cpu_rand(0, (frames - 1) * len(rows) * len(cols) * 2).reshape(frames - 1, len(rows), len(cols), 2)
    row = rows[None, :, None] + (choice[..., 0] * np.minimum(height - rows, 2)[None, :, None].astype(np.float32)).astype(np.int64)
    col = cols[None, None, :] + (choice[..., 1] * np.minimum(width - cols, 2)[None, None, :].astype(np.float32)).astype(np.int64)
    positions = (row * width + col).reshape(frames - 1, -1)
    macro_cols, macro_rows = (width + 3) // 4, (height + 3) // 4
    macro = ((positions // width) // 4) * macro_cols + ((positions % width) // 4)
    grouped = np.full((frames - 1, macro_rows * macro_cols, 4), -1, dtype=np.int64)
    for f in range(frames - 1):
        counts = np.zeros(macro_rows * macro_cols, np.int64)
        for pos, grp in zip(positions[f], macro[f]):
            grouped[f, grp, counts[grp]] = f * patches + patches + pos
            counts[grp] += 1
    return first, positions, grouped, cell_table(height, width, 4)


def protected_skeleton(features, frames: int, patch_hw, top1_threshold: float = 0.95):
    """(basis ids sorted, stats): frame 0 plus every later frame's uniform anchors; an anchor
    other than its macro cell's slot 0 is pruned when its best fp32 cosine to a reference-frame
    patch of the cell, the cell's slot 0 or the previous frame's slot 0 reaches the threshold
    (sparse_convex.py:1371-1434)."""
    first, _, grouped, first_table = uniform_2x2_tables(frames, patch_hw)
    patches = patch_hw[0] * patch_hw[1]
    if frames <= 1:
        return first, dict(initial_uniform_bases=len(first), protected_uniform_bases=len(first),
                           top1_pruned_uniform_bases=0)
    f64 = np.asarray(features, np.float64)
    valid = grouped >= 0
    safe = np.maximum(grouped, 0)
    protected = safe[..., 0]
    current = protected[..., None]
    previous = np.concatenate([np.full_like(protected[:1], -1), protected[:-1]], axis=0)[..., None]
    reference = np.broadcast_to(first_table[None], (frames - 1,) + first_table.shape)
    target = np.concatenate([reference, current, previous], axis=-1)
    target_valid = target >= 0
    score = np.einsum("fmsd,fmtd->fmst", f64[safe], f64[np.maximum(target, 0)])
    score = np.where(target_valid[..., None, :], score, -np.inf)
    top1 = score.max(axis=-1)
    removable = valid & (np.arange(4)[None, None] > 0)
    pruned = removable & (top1 >= top1_threshold)
    kept = valid & ~pruned
    basis = np.unique(np.concatenate([first, safe[kept]]))
    return basis, dict(initial_uniform_bases=int(patches + valid.sum()), protected_uniform_bases=int(len(basis)),
                       top1_pruned_uniform_bases=int(pruned.sum()))


def _topk_desc(values, k):
    """Indices of the k largest values, stable (ties to the lower index)."""
    return np.argsort(-np.asarray(values, np.float64), kind="stable")[:k]


def ttt_event_bases(features, geometry, labels, sensitivity, excluded, *, frames: int, patch_hw, amount: int,
                    geometry_weight: float = 0.01):
    """TTT-proposed event bases (sparse_convex.py:1268-1324): sensitive patches (label 1, not
    excluded) binned by (4-frame time bin, 0.5-wide xyz bins); per bin the patch closest to the
    bin's normalised mean feature and mean geometry (+0.005 sensitivity), lowest id on ties; more
    bins than ``amount``: bins ranked by mean sensitivity x sqrt(size); fewer: filled with the
    most sensitive remaining patches.  Returns sorted unique patch ids."""
    if geometry_weight < 0:
        raise ValueError("TTT event geometry weight must be nonnegative")
    patches = patch_hw[0] * patch_hw[1]
    labels = np.asarray(labels)
    ids = np.nonzero((labels == 1) & ~np.asarray(excluded, bool))[0]
    if amount <= 0 or not len(ids):
        return ids[:0]
    geometry = np.asarray(geometry, np.float32)
    sens = np.asarray(sensitivity, np.float32)
    geo = geometry[ids]
    xyz_bin = np.clip(np.floor((geo[:, :3] + np.float32(4.0)) / np.float32(0.5)).astype(np.int64), 0, 31)
    time_bin = (ids // patches) // 4
    code = ((time_bin * 37 + xyz_bin[:, 0]) * 37 + xyz_bin[:, 1]) * 37 + xyz_bin[:, 2]
    _, inverse = np.unique(code, return_inverse=True)
    groups = int(inverse.max()) + 1
    counts = np.bincount(inverse, minlength=groups)
    cf = np.asarray(features, np.float64)[ids]
    cg = geometry[ids].astype(np.float64)
    sums = np.zeros((groups, cf.shape[1]))
    np.add.at(sums, inverse, cf)
    mean = sums / counts[:, None]
    center_f = mean / np.maximum(np.linalg.norm(mean, axis=1, keepdims=True), 1e-8)
    gsum = np.zeros((groups, 4))
    np.add.at(gsum, inverse, cg)
    center_g = gsum / counts[:, None]
    score = ((cf * center_f[inverse]).sum(-1) - geometry_weight * ((cg - center_g[inverse]) ** 2).sum(-1)
             + 0.005 * sens[ids].astype(np.float64))
    best = np.full(groups, -np.inf)
    np.maximum.at(best, inverse, score)
    sentinel = len(labels)
    cand = np.where(score == best[inverse], ids, sentinel)
    rep = np.full(groups, sentinel, np.int64)
    np.minimum.at(rep, inverse, cand)
    rep = rep[rep < sentinel]
    if len(rep) > amount:
        ssum = np.zeros(groups)
        np.add.at(ssum, inverse, sens[ids].astype(np.float64))
        group_score = ssum / counts * np.sqrt(counts.astype(np.float64))
        rep = rep[_topk_desc(group_score, amount)]
    if len(rep) < amount:
        chosen = np.zeros(len(labels), bool)
        chosen[rep] = True
        remaining = ids[~chosen[ids]]
        fill = min(amount - len(rep), len(remaining))
        if fill:
            rep = np.concatenate([rep, remaining[_topk_desc(sens[remaining], fill)]])
    return np.unique(rep)


def certificate(source, supports, alpha):
    """(cosine, residual, reconstruction norm) of the convex reconstruction
    sum_c alpha_c supports_c (F.cosine_similarity with eps 1e-8, as the reference)."""
    x = np.asarray(source, np.float64)
    recon = np.einsum("sc,scd->sd", np.asarray(alpha, np.float64), np.asarray(supports, np.float64))
    nx, nr = np.linalg.norm(x, axis=1), np.linalg.norm(recon, axis=1)
    cos = (x * recon).sum(1) / (np.maximum(nx, 1e-8) * np.maximum(nr, 1e-8))
    return cos, np.linalg.norm(x - recon, axis=1), nr


def fit_supports(features, source_ids, support_ids, steps: int = 32):
    """The reference's solve for given supports: fp32 Gram / rhs, the 32-step projected
    gradient, then the certificate.  -> (weights, cosine, residual, reconstruction norm)."""
    f = np.asarray(features, np.float64)
    x = f[source_ids]
    sup = f[support_ids]
    gram = np.einsum("sid,sjd->sij", sup, sup).astype(np.float32)
    rhs = np.einsum("sid,sd->si", sup, x).astype(np.float32)
    w = ref.projected_gradient(gram, rhs, steps)
    return (w,) + certificate(x, sup, w)


def _top4(features, query_ids, basis_ids):
    """Stable top-4 basis ids of each query by bf16 score (sparse_convex.py:546-552, :264)."""
    f = np.asarray(features, np.float32)
    _, idx = ref.similarity_topk(f[query_ids], f[basis_ids], 4)
    return np.asarray(basis_ids)[idx]


def _certified(fit, threshold):
    """The certificate of a fit (support, weights, cosine, residual, norm): cosine >= tau,
    residual <= sqrt(2 (1 - tau)), reconstruction norm >= 0.8 (sparse_convex.py:648-653)."""
    limit = (2.0 * (1.0 - threshold)) ** 0.5
    return (fit[2] >= threshold) & (fit[3] <= limit) & (fit[4] >= 0.80)


def geometry_shortlist(features, geometry, query_ids, basis_ids, weight: float):
    """The Pareto-guard selection (sparse_convex.py:502-531 local, :263-306 global): bf16 feature
    scores; a top-16 shortlist (top-min(16, basis)); joint = score - w * sum_d (g_s - g_c)^2 in
    float32 (squares summed in order d = 0..3); the joint top-4 positions, reordered by feature
    score (stable descending, so equal scores keep the joint order).  Every ranking here is a
    stable descending sort (ties to the lower position; the reference's torch.topk leaves tie
    order open).  -> (feature top-4 basis ids, joint basis ids), each [S, 4]."""
    f = np.asarray(features, np.float32)
    query_ids = np.asarray(query_ids, np.int64)
    basis_ids = np.asarray(basis_ids, np.int64)
    vals, idx = ref.similarity_topk(f[query_ids], f[basis_ids], min(16, len(basis_ids)))
    g = np.asarray(geometry, np.float32)
    diff = (g[query_ids][:, None, :] - g[basis_ids[idx]]).astype(np.float32)
    sq = (diff * diff).astype(np.float32)
    dist = (((sq[..., 0] + sq[..., 1]).astype(np.float32) + sq[..., 2]).astype(np.float32) + sq[..., 3])
    joint = (vals.astype(np.float32) - (np.float32(weight) * dist.astype(np.float32)).astype(np.float32))
    jpos = np.argsort(-joint.astype(np.float32), axis=1, kind="stable")[:, :4]
    canon = np.argsort(-np.take_along_axis(vals, jpos, 1), axis=1, kind="stable")
    jpos = np.take_along_axis(jpos, canon, 1)
    return basis_ids[idx[:, :4]], basis_ids[np.take_along_axis(idx, jpos, 1)]


def geometry_residual(geometry, source_ids, support_ids, weights):
    """|| g_s - sum_c w_c g_{support_c} || (sparse_convex.py:577-582, :325-330)."""
    g = np.asarray(geometry, np.float64)
    recon = np.einsum("sc,scd->sd", np.asarray(weights, np.float64), g[np.asarray(support_ids, np.int64)])
    return np.linalg.norm(g[np.asarray(source_ids, np.int64)] - recon, axis=1)


def guard_choose(features, geometry, source_ids, feature_ids, joint_ids, tolerance: float):
    """Both solves and the Pareto guard (sparse_convex.py:586-639, :335-367): the joint set wins
    only where it differs from the feature top-4, its cosine and residual are no worse (up to
    the tolerance) and its 4-D residual is strictly smaller.  -> (support, weights, cosine,
    residual, norm, chosen mask)."""
    feat = fit_supports(features, source_ids, feature_ids)
    joint = fit_supports(features, source_ids, joint_ids)
    changed = np.any(joint_ids != feature_ids, axis=1)
    gf = geometry_residual(geometry, source_ids, feature_ids, feat[0])
    gj = geometry_residual(geometry, source_ids, joint_ids, joint[0])
    choose = (joint[1] + tolerance >= feat[1]) & (joint[2] <= feat[2] + tolerance) & (gj < gf) & changed
    pick = lambda a, b: np.where(choose.reshape((-1,) + (1,) * (np.ndim(a) - 1)), a, b)
    return (pick(joint_ids, feature_ids),) + tuple(pick(j, f) for j, f in zip(joint, feat)) + (choose,)


def fit_global(features, basis_ids, threshold: float, source_ids, geometry=None, geometry_weight: float = 0.0,
               guard_tolerance=None, stats=None):
    """_adaptive_fit_fused with the one-hot shortcut off (the default): top-4 over the whole
    basis, then the solve and certificate of every row; with geometry_weight > 0 and a guard
    tolerance, the top-16 shortlist, joint re-rank and Pareto guard (:263-367)."""
    if geometry_weight > 0 and guard_tolerance is not None:
        fids, jids = geometry_shortlist(features, geometry, source_ids, basis_ids, geometry_weight)
        out = guard_choose(features, geometry, source_ids, fids, jids, guard_tolerance)
        if stats is not None:
            stats["guard_selected"] = stats.get("guard_selected", 0) + int(out[5].sum())
        return out[:5]
    if geometry_weight > 0:
        raise ValueError("the joint-metric route (geometry weight without a guard tolerance) is not restated")
    support = _top4(features, source_ids, basis_ids)
    return (support,) + fit_supports(features, source_ids, support)


def fit_temporal_local(features, basis_ids, *, frames: int, patches: int, threshold: float, source_ids,
                       frame_group: int = LOCAL_FRAME_GROUP, geometry=None, geometry_weight: float = 0.0,
                       guard_tolerance=None, stats=None):
    """_adaptive_fit_temporal_local (sparse_convex.py:440-684) on its feature route: sources of
    frames [b, b + 8) (b = 1, 9, ...) search the basis of frame 0 and frames [max(1, b - 1),
    min(F - 1, b + 8)]; rows that fail the certificate (and reference-frame sources, which no
    group covers) take the global route.  With geometry_weight > 0 and a guard tolerance, each
    group's selection is the guarded shortlist (geometry_shortlist / guard_choose;
    sparse_convex.py:502-531, :586-639) and the fallback is the guarded global route.
    -> (support ids [S, 4], weights, cosine, residual, reconstruction norm)."""
    guard = geometry_weight > 0 and guard_tolerance is not None
    if geometry_weight > 0 and not guard:
        raise ValueError("the joint-metric route (geometry weight without a guard tolerance) is not restated")
    source_ids = np.asarray(source_ids, np.int64)
    basis_ids = np.asarray(basis_ids, np.int64)
    n = len(source_ids)
    support = np.full((n, 4), basis_ids[0] if len(basis_ids) else 0, np.int64)
    weights = np.zeros((n, 4), np.float32)
    cos = np.zeros(n)
    res = np.zeros(n)
    norm = np.zeros(n)
    assigned = np.zeros(n, bool)
    sf, bf = source_ids // patches, basis_ids // patches
    for begin in range(1, frames, frame_group):
        end = min(begin + frame_group, frames)
        rows = np.nonzero((sf >= begin) & (sf < end))[0]
        if not len(rows):
            continue
        lo, hi = max(1, begin - 1), min(frames - 1, end)
        local = basis_ids[(bf == 0) | ((bf >= lo) & (bf <= hi))]
        if guard:
            fids, jids = geometry_shortlist(features, geometry, source_ids[rows], local, geometry_weight)
            sup, w, c, r, nr, chosen = guard_choose(features, geometry, source_ids[rows], fids, jids, guard_tolerance)
            if stats is not None:  # counted before the fallback, as the reference counts
                stats["guard_selected"] = stats.get("guard_selected", 0) + int(chosen.sum())
        else:
            sup = _top4(features, source_ids[rows], local)
            w, c, r, nr = fit_supports(features, source_ids[rows], sup)
        support[rows], weights[rows], cos[rows], res[rows], norm[rows] = sup, w, c, r, nr
        assigned[rows] = True
    fit = (support, weights, cos, res, norm)
    fallback = np.nonzero(~(assigned & _certified(fit, threshold)))[0]
    if len(fallback):
        g = fit_global(features, basis_ids, threshold, source_ids[fallback], geometry, geometry_weight,
                       guard_tolerance, stats)
        for dst, val in zip(fit, g):
            dst[fallback] = val
    return fit


def build_plan(tokens, *, frames: int, tokens_per_frame: int, patch_token_start: int, patch_hw, threshold: float,
               labels, sensitivity, geometry, top1_prune_threshold: float = 0.95,
               sensitive_event_ratio: float = 0.02, selection_geometry_weight: float = 0.01,
               support_geometry_weight: float = 0.0, support_geometry_guard_tolerance=None):
    """build_ttt_protected_uniform_convex_plan (sparse_convex.py:1738-2016): the feature route,
    or with support_geometry_weight > 0 and a guard tolerance the Pareto-guarded geometry route
    (both fits of :1845-1891 take geometry, weight and tolerance).
    tokens [N, D] float32.  Returns dict(keep, source, parent (compact ids), weights, normalizer,
    special, special_compact, stable_basis, event_proposal, event, accepted)."""
    height, width = patch_hw
    patches = height * width
    patch_count = frames * patches
    total = tokens.shape[0]
    if total != frames * tokens_per_frame or patch_token_start + patches != tokens_per_frame:
        raise ValueError("invalid protected TTT token layout")
    patch_ids = (np.arange(frames)[:, None] * tokens_per_frame + patch_token_start + np.arange(patches)[None]).ravel()
    features = ref.normalize_bf16(np.asarray(tokens, np.float32)[patch_ids], 1e-8)
    gkw = dict(geometry=np.asarray(geometry, np.float32) if support_geometry_weight else None,
               geometry_weight=support_geometry_weight, guard_tolerance=support_geometry_guard_tolerance)
    stable, stats = protected_skeleton(features, frames, patch_hw, top1_prune_threshold)
    stable_mask = np.zeros(patch_count, bool)
    stable_mask[stable] = True
    freed = stats["top1_pruned_uniform_bases"]
    pruning = top1_prune_threshold <= 1.0
    budget = freed if pruning else int(round(sensitive_event_ratio * patch_count))
    proposal = ttt_event_bases(features, geometry, labels, sensitivity, stable_mask, frames=frames, patch_hw=patch_hw,
                               amount=2 * budget, geometry_weight=selection_geometry_weight)
    event = proposal[:0]
    if budget and len(proposal):
        efit = fit_temporal_local(features, stable, frames=frames, patches=patches, threshold=threshold,
                                  source_ids=proposal, **gkw)
        cand = np.nonzero(~_certified(efit, threshold))[0]
        if len(cand) > budget:
            priority = (np.asarray(sensitivity, np.float32)[proposal[cand]].astype(np.float64) * efit[3][cand])
            cand = cand[_topk_desc(priority, budget)]
        event = proposal[cand]
    basis = np.unique(np.concatenate([stable, event]))
    basis_mask = np.zeros(patch_count, bool)
    basis_mask[basis] = True
    source = np.nonzero(~basis_mask)[0]
    fit_stats = {"guard_selected": 0}
    fit = fit_temporal_local(features, basis, frames=frames, patches=patches, threshold=threshold, source_ids=source,
                             stats=fit_stats, **gkw)
    accepted = _certified(fit, threshold)
    rows = np.nonzero(accepted)[0]
    source_local, support_local, weights = source[rows], fit[0][rows], fit[1][rows].astype(np.float32)
    kept = np.ones(patch_count, bool)
    kept[source_local] = False
    keep_local = np.nonzero(kept)[0]
    special = (np.arange(frames)[:, None] * tokens_per_frame + np.arange(patch_token_start)[None]).ravel()
    keep = np.sort(np.concatenate([special, patch_ids[keep_local]]))
    o2c = np.full(total, -1, np.int64)
    o2c[keep] = np.arange(len(keep))
    parent = o2c[patch_ids[support_local]]
    if (parent < 0).any():
        raise RuntimeError("protected TTT convex support must remain physical")
    norm = ref.normalizer(parent, weights, len(keep))
    return dict(keep=keep, source=patch_ids[source_local], parent=parent, weights=weights, normalizer=norm,
                special=special, special_compact=o2c[special], stable_basis=stable, event_proposal=proposal,
                event=event, accepted=accepted, fit_source=source, fit=fit, features=features,
                guard_selected=fit_stats["guard_selected"])
