"""Merge-step planners on B200.

``build_fastvggt_plan`` is a drop-in for vggt_omega/models/token_merging.py:1045-1122 (same
signature, same seeded destination choice, same stable ranking): the host builds only the
static destination / protected / source tables (they depend on the layout and the seed,
exactly as in the reference, and are cached), everything data-dependent runs on the device —
row normalisation to bf16, the similarity GEMM with fused argmax (tcgen05), the stable
descending ranking and the keep / inverse maps — with no host synchronisation.

``build_uniform_convex_plan`` is the four-support planner the single-block benchmark uses: a
fixed keep set (every special token plus evenly spaced patch anchors, exactly
``total // merge_factor`` tokens), top-4 support retrieval inside frame groups (tcgen05 GEMM
with fused top-4), the support Gram and the 32-step projected-gradient convex fit fused in
one kernel (sparse_convex.py:2308-2321 / sparse_convex_kernels.py:214-280), then a
``WeightedBilinearTokenPlan`` with ``key_log_mass = log(mass)`` (sparse_convex.py:2448-2470).
"""
from __future__ import annotations

import functools
import math

import torch

from . import _clib as C
from .ops import build_plan_csr, row_normalize_bf16, similarity_topk
from .token_plan import TokenPlan, WeightedBilinearTokenPlan

__all__ = ["build_fastvggt_plan", "build_uniform_convex_plan", "build_ttt_protected_uniform_convex_plan",
           "fastvggt_tables", "ttt_skeleton_tables", "uniform_keep_layout"]

FAST_MATCH_SOURCE_CHUNK = 5000


@functools.lru_cache(maxsize=32)
def fastvggt_tables(frames: int, tokens_per_frame: int, patch_token_start: int, patch_hw: tuple[int, int],
                    merge_ratio: float, protect_ratio: float, seed: int):
    """Static tables of the FastVGGT plan (host, cached): source and destination token ids
    and the number of sources to remove (token_merging.py:1068-1096)."""
    total = frames * tokens_per_frame
    height, width = patch_hw
    patches = height * width
    patch_ids = (torch.arange(frames)[:, None] * tokens_per_frame + patch_token_start + torch.arange(patches))
    destination = torch.zeros(total, dtype=torch.bool)
    destination[patch_ids[0]] = True
    generator = torch.Generator(device="cpu").manual_seed(seed)
    rows = torch.arange(0, height, 2)
    cols = torch.arange(0, width, 2)
    choices = torch.rand(frames - 1, len(rows), len(cols), 2, generator=generator)
    row = rows[None, :, None] + (choices[..., 0] * (height - rows).clamp(max=2)[None, :, None]).long()
    col = cols[None, None, :] + (choices[..., 1] * (width - cols).clamp(max=2)[None, None, :]).long()
    selected = (row * width + col).reshape(frames - 1, -1)
    destination[patch_ids[1:].gather(1, selected).flatten()] = True
    protected = torch.ones(total, dtype=torch.bool)
    protected[patch_ids.flatten()] = False
    protected[patch_ids[0]] = True
    count = int(total * protect_ratio)
    if count:
        protected[torch.arange(0, total, max(1, total // count))[:count]] = True
    source_indices = (~(destination | protected)).nonzero().flatten()
    destination_indices = destination.nonzero().flatten()
    removed = min(int(total * merge_ratio), source_indices.numel())
    return source_indices, destination_indices, removed


@torch.no_grad()
def build_fastvggt_plan(tokens: torch.Tensor, *, frames: int, tokens_per_frame: int, patch_token_start: int,
                        patch_hw: tuple[int, int], merge_ratio: float = 0.9, protect_ratio: float = 0.10,
                        seed: int = 0, match_chunk_size: int = FAST_MATCH_SOURCE_CHUNK) -> TokenPlan:
    """FastVGGT argmax merge for Omega's interleaved layout (token_merging.py:1045-1122).

    ``match_chunk_size`` is accepted for signature compatibility; the fused kernel never
    materialises the score matrix, so no chunking is needed."""
    del match_chunk_size
    if not (0.0 <= merge_ratio <= 1.0 and 0.0 <= protect_ratio <= 1.0):
        raise ValueError("FastVGGT ratios must lie in [0, 1]")
    batch, total, _ = tokens.shape
    if total != frames * tokens_per_frame or patch_token_start + math.prod(patch_hw) != tokens_per_frame:
        raise ValueError("Invalid Omega FastVGGT frame/patch/special-token layout")
    C.require_cuda(tokens, "build_fastvggt_plan")
    dev = tokens.device
    identity = torch.arange(total, device=dev).expand(batch, -1)
    if frames == 1 or merge_ratio == 0:
        return TokenPlan(identity, identity, total)
    src_cpu, dst_cpu, removed = fastvggt_tables(frames, tokens_per_frame, patch_token_start, tuple(patch_hw),
                                                float(merge_ratio), float(protect_ratio), int(seed))
    if removed == 0:
        return TokenPlan(identity, identity, total)
    src_idx = src_cpu.to(dev, non_blocking=True)
    dst_idx = dst_cpu.to(dev, non_blocking=True)
    keeps, inverses = [], []
    lib = C.lib()
    ws_bytes = lib.vb200_merge_assign_workspace_size(src_idx.numel(), total)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    for b in range(batch):
        x = tokens[b]
        source_metric = row_normalize_bf16(x, src_idx)
        destination_metric = row_normalize_bf16(x, dst_idx)
        best, target = similarity_topk(source_metric, destination_metric, 1)
        keep = torch.empty(total - removed, dtype=torch.int64, device=dev)
        inverse = torch.empty(total, dtype=torch.int64, device=dev)
        rc = lib.vb200_merge_assign(best.data_ptr(), target.data_ptr(), src_idx.data_ptr(), dst_idx.data_ptr(),
                                    src_idx.numel(), dst_idx.numel(), total, removed, keep.data_ptr(),
                                    inverse.data_ptr(), ws.data_ptr(), ws_bytes, C.stream_of(dev))
        C.check(rc, "merge_assign")
        keeps.append(keep)
        inverses.append(inverse)
    return TokenPlan(torch.stack(keeps), torch.stack(inverses), total)


@functools.lru_cache(maxsize=32)
def uniform_keep_layout(frames: int, tokens_per_frame: int, special: int, merge_factor: int, group_frames: int):
    """Host tables of the uniform four-support plan (cached): keep ids (all special tokens +
    evenly spaced patch anchors, exactly total // merge_factor), source ids, special ids,
    and per-frame-group row ranges of sources and keeps (both sorted by token id)."""
    if frames % group_frames:
        raise ValueError("frames must be a multiple of group_frames")
    total = frames * tokens_per_frame
    kept_total = total // merge_factor
    groups = frames // group_frames
    base, extra = divmod(kept_total, groups)
    patches = tokens_per_frame - special
    keep_parts, src_parts, q_begin, b_begin = [], [], [0], [0]
    for g in range(groups):
        f0 = g * group_frames
        frame_ids = torch.arange(f0, f0 + group_frames)
        spec = (frame_ids[:, None] * tokens_per_frame + torch.arange(special)[None]).flatten()
        gp = (frame_ids[:, None] * tokens_per_frame + special + torch.arange(patches)[None]).flatten()
        n_anchor = base + (1 if g < extra else 0) - spec.numel()
        if n_anchor <= 0 or n_anchor > gp.numel():
            raise ValueError("merge factor leaves no room for patch anchors")
        anchors = gp[(torch.arange(n_anchor) * gp.numel()) // n_anchor]
        keep_g = torch.sort(torch.cat([spec, anchors])).values
        mask = torch.ones(group_frames * tokens_per_frame, dtype=torch.bool)
        mask[keep_g - f0 * tokens_per_frame] = False
        src_g = torch.nonzero(mask).flatten() + f0 * tokens_per_frame
        keep_parts.append(keep_g)
        src_parts.append(src_g)
        q_begin.append(q_begin[-1] + src_g.numel())
        b_begin.append(b_begin[-1] + keep_g.numel())
    keep = torch.cat(keep_parts)
    source = torch.cat(src_parts)
    special_ids = (torch.arange(frames)[:, None] * tokens_per_frame + torch.arange(special)[None]).flatten()
    original_to_compact = torch.full((total,), -1, dtype=torch.long)
    original_to_compact[keep] = torch.arange(keep.numel())
    return dict(keep=keep, source=source, special=special_ids,
                special_compact=original_to_compact[special_ids],
                q_begin=torch.tensor(q_begin), b_begin=torch.tensor(b_begin))


@torch.no_grad()
def build_uniform_convex_plan(tokens: torch.Tensor, *, frames: int, tokens_per_frame: int,
                              patch_token_start: int, merge_factor: int = 4, group_frames: int = 4,
                              steps: int = 32, preserve_queries: bool = False,
                              dense_special_queries: bool = False, _tables_on=None) -> WeightedBilinearTokenPlan:
    """Four-support convex plan with a uniform keep set; see the module docstring.
    tokens [1, N, D] (the attention input after norm1)."""
    if tokens.shape[0] != 1:
        raise ValueError("sparse-convex compaction currently supports batch size one")
    C.require_cuda(tokens, "build_uniform_convex_plan")
    dev = tokens.device
    total = tokens.shape[1]
    if total != frames * tokens_per_frame:
        raise ValueError("invalid frame/token layout for sparse-convex compaction")
    lay = uniform_keep_layout(frames, tokens_per_frame, patch_token_start, merge_factor, group_frames)
    dl = _device_layout(lay, dev)
    x = tokens[0]
    S, K = dl["source"].numel(), dl["keep"].numel()
    # normalised features in one buffer, written in gathered order: rows [0, S) the sources,
    # rows [S, S + K) the keeps (every token is read once; no separate gathers)
    feat = row_normalize_bf16(x, dl["source_keep"])
    src_feat, basis_feat = feat[:S], feat[S:]
    _, parent = similarity_topk(src_feat, basis_feat, 4, query_begin=lay["q_begin"], basis_begin=lay["b_begin"])
    alpha = torch.empty((S, 4), device=dev, dtype=torch.float32)
    parent_rows = parent + S  # rows of the supports in feat
    rc = C.lib().vb200_support_fit(C.BF16, feat.data_ptr(), feat.shape[0], feat.stride(0),
                                   None, parent_rows.data_ptr(), S,
                                   feat.shape[1], None, None, alpha.data_ptr(), int(steps), C.stream_of(dev))
    C.check(rc, "support_fit")
    grouped = dl["max_group_rows"] * 4 <= 8 * 1024 and dl["max_group_sources"] * 4 <= 16 * 1024
    csr = build_plan_csr(parent, alpha, K, src_rows=dl["source"],
                         groups=(dl["q_begin"], dl["b_begin"], dl["max_group_rows"], dl["max_group_sources"])
                         if grouped else None)
    normalizer = csr.mass.view(1, K, 1)
    return WeightedBilinearTokenPlan(
        csr=csr,
        keep=dl["keep"][None], source_original=dl["source"][None], source_parent_compact=parent[None],
        source_pool_weights=alpha[None], source_restore_weights=alpha[None], original_tokens=total,
        normalizer=normalizer, preserve_queries=preserve_queries, preserve_destination_keys=preserve_queries,
        dense_special_queries=dense_special_queries, special_query_original=dl["special"],
        special_query_compact=dl["special_compact"], key_log_mass=csr.log_mass[None],
        metadata={"planner": "uniform_convex_top4", "merge_factor": merge_factor, "group_frames": group_frames},
    )


_DEVICE_LAYOUTS: dict = {}


def _device_layout(lay: dict, dev: torch.device) -> dict:
    key = (id(lay), str(dev))
    hit = _DEVICE_LAYOUTS.get(key)
    if hit is None:
        hit = {k: lay[k].to(dev) for k in ("keep", "source", "special", "special_compact", "q_begin", "b_begin")}
        hit["source_keep"] = torch.cat([hit["source"], hit["keep"]])  # feature-row order of the planner
        hit["max_group_rows"] = int((lay["b_begin"][1:] - lay["b_begin"][:-1]).max())
        hit["max_group_sources"] = int((lay["q_begin"][1:] - lay["q_begin"][:-1]).max())
        _DEVICE_LAYOUTS[key] = hit
    return hit


# ------------------------------------------------------------------------------------------
# The released planner: build_ttt_protected_uniform_convex_plan
# ------------------------------------------------------------------------------------------
LOCAL_FRAME_GROUP = 8  # frames per temporal-local support search (sparse_convex.py:31)


@functools.lru_cache(maxsize=32)
def ttt_skeleton_tables(frames: int, patch_hw: tuple[int, int]):
    """Static tables of the protected uniform skeleton (host, cached), following
    sparse_convex.py:1327-1368: one patch per 2x2 cell of every later frame drawn from a fresh
    CPU generator seeded 0 (the same draw as the uniform planners), grouped by 4x4 macro cell in
    position order (slot 0 is the protected anchor), and for every (frame, cell, slot) the
    candidate targets that can make a non-protected anchor redundant: the reference frame's
    patches of the cell, the cell's slot-0 anchor and the previous frame's slot-0 anchor.
    -> dict(first [P], anchors [F-1, cells, 4] (-1 = empty slot), targets [F-1, cells, 4, T])."""
    height, width = patch_hw
    patches = height * width
    first = torch.arange(patches)
    if frames <= 1:
        empty = torch.empty((0, 0, 4), dtype=torch.long)
        return dict(first=first, anchors=empty, targets=torch.empty((0, 0, 4, 18), dtype=torch.long))
    generator = torch.Generator(device="cpu").manual_seed(0)
    rows, cols = torch.arange(0, height, 2), torch.arange(0, width, 2)
    draw = torch.rand(frames - 1, len(rows), len(cols), 2, generator=generator)
    r = rows[None, :, None] + (draw[..., 0] * (height - rows).clamp(max=2)[None, :, None]).long()
    c = cols[None, None, :] + (draw[..., 1] * (width - cols).clamp(max=2)[None, None, :]).long()
    position = (r * width + c).reshape(frames - 1, -1)
    cells_x, cells_y = (width + 3) // 4, (height + 3) // 4
    cell = (position // width // 4) * cells_x + (position % width) // 4
    anchors = torch.full((frames - 1, cells_x * cells_y, 4), -1, dtype=torch.long)
    for f in range(frames - 1):
        filled = [0] * (cells_x * cells_y)
        for p, g in zip(position[f].tolist(), cell[f].tolist()):
            anchors[f, g, filled[g]] = (f + 1) * patches + p
            filled[g] += 1
    reference = torch.full((cells_x * cells_y, 16), -1, dtype=torch.long)
    for g in range(cells_x * cells_y):
        top, left = (g // cells_x) * 4, (g % cells_x) * 4
        ids = [y * width + x for y in range(top, min(top + 4, height)) for x in range(left, min(left + 4, width))]
        reference[g, :len(ids)] = torch.tensor(ids)
    protected = anchors[..., 0]
    previous = torch.cat([torch.full_like(protected[:1], -1), protected[:-1]])
    per_cell = torch.cat([reference[None].expand(frames - 1, -1, -1), protected[..., None], previous[..., None]], -1)
    targets = per_cell[:, :, None, :].expand(-1, -1, 4, -1).contiguous()
    return dict(first=first, anchors=anchors, targets=targets)


def _feature_fit(features: torch.Tensor, source_ids: torch.Tensor, support_ids: torch.Tensor, steps: int = 32):
    """The reference's solve for given supports (sparse_convex.py:558-583): fp32 Gram and rhs of
    the four supports, 32 projected-gradient steps (vb200_support_fit), then the certificate
    (vb200_support_certificate).  -> (weights [S,4], cosine, residual, reconstruction norm)."""
    S = source_ids.numel()
    dev = features.device
    alpha = torch.empty((S, 4), device=dev, dtype=torch.float32)
    cos, res, nrm = (torch.empty(S, device=dev, dtype=torch.float32) for _ in range(3))
    if S == 0:
        return alpha, cos, res, nrm
    src = source_ids.to(torch.int64).contiguous()
    sup = support_ids.to(torch.int64).contiguous()
    lib, stream = C.lib(), C.stream_of(dev)
    dt, rows, stride, D = C.dtype_code(features.dtype), features.shape[0], features.stride(0), features.shape[1]
    C.check(lib.vb200_support_fit(dt, features.data_ptr(), rows, stride, src.data_ptr(), sup.data_ptr(), S, D,
                                  None, None, alpha.data_ptr(), int(steps), stream), "support_fit")
    C.check(lib.vb200_support_certificate(dt, features.data_ptr(), rows, stride, src.data_ptr(), sup.data_ptr(),
                                          alpha.data_ptr(), S, D, cos.data_ptr(), res.data_ptr(), nrm.data_ptr(),
                                          stream), "support_certificate")
    return alpha, cos, res, nrm


def _certified(cos, res, nrm, threshold: float) -> torch.Tensor:
    """cosine >= tau, residual <= sqrt(2 (1 - tau)), reconstruction norm >= 0.8
    (sparse_convex.py:648-653, 1870-1874, 1898-1902)."""
    return (cos >= threshold) & (res <= (2.0 * (1.0 - threshold)) ** 0.5) & (nrm >= 0.80)


def _guarded_fit(features, geometry, query_ids, basis_list, weight: float, tolerance: float,
                 query_begin=None, basis_begin=None):
    """The Pareto-guarded geometry route for the queries against their basis rows (grouped like
    similarity_topk): the tcgen05 top-16 feature shortlist, the joint re-rank
    (vb200_geometry_shortlist), both fits (feature top-4 and joint set, each vb200_support_fit +
    vb200_support_certificate) and the guard (vb200_geometry_guard); sparse_convex.py:502-531,
    586-639 and 263-367.  -> (support ids [S,4], weights, cosine, residual, norm, chosen int32 [S])."""
    from .ops import row_gather
    dev = features.device
    S = query_ids.numel()
    vals16, idx16 = similarity_topk(row_gather(features, query_ids), row_gather(features, basis_list), 16,
                                    query_begin=query_begin, basis_begin=basis_begin)
    qgeo = geometry.index_select(0, query_ids).contiguous()
    bgeo = geometry.index_select(0, basis_list).contiguous()
    fidx = torch.empty((S, 4), device=dev, dtype=torch.long)
    jidx = torch.empty((S, 4), device=dev, dtype=torch.long)
    changed = torch.empty(S, device=dev, dtype=torch.int32)
    lib, stream = C.lib(), C.stream_of(dev)
    C.check(lib.vb200_geometry_shortlist(vals16.data_ptr(), idx16.data_ptr(), S, 16, qgeo.data_ptr(), bgeo.data_ptr(),
                                         basis_list.numel(), float(weight), fidx.data_ptr(), jidx.data_ptr(),
                                         changed.data_ptr(), stream), "geometry_shortlist")
    fids = basis_list.index_select(0, fidx.reshape(-1)).view(S, 4).contiguous()
    jids = basis_list.index_select(0, jidx.reshape(-1)).view(S, 4).contiguous()
    ffit = _feature_fit(features, query_ids, fids)
    jfit = _feature_fit(features, query_ids, jids)
    out_ids = torch.empty((S, 4), device=dev, dtype=torch.long)
    out_w = torch.empty((S, 4), device=dev, dtype=torch.float32)
    out_c, out_r, out_n = (torch.empty(S, device=dev, dtype=torch.float32) for _ in range(3))
    chosen = torch.empty(S, device=dev, dtype=torch.int32)
    src = query_ids.to(torch.int64).contiguous()
    C.check(lib.vb200_geometry_guard(
        S, geometry.data_ptr(), geometry.shape[0], src.data_ptr(), fids.data_ptr(), ffit[0].data_ptr(),
        ffit[1].data_ptr(), ffit[2].data_ptr(), ffit[3].data_ptr(), jids.data_ptr(), jfit[0].data_ptr(),
        jfit[1].data_ptr(), jfit[2].data_ptr(), jfit[3].data_ptr(), changed.data_ptr(), float(tolerance),
        out_ids.data_ptr(), out_w.data_ptr(), out_c.data_ptr(), out_r.data_ptr(), out_n.data_ptr(), chosen.data_ptr(),
        stream), "geometry_guard")
    return out_ids, out_w, out_c, out_r, out_n, chosen


def _fit_global(features, basis_ids, source_ids, guard=None):
    """The exact global route (_adaptive_fit_fused, sparse_convex.py:168-330, one-hot shortcut
    off): top-4 of every source over the whole basis, then the solve; with ``guard`` =
    (geometry, weight, tolerance, counter) the guarded geometry route (:263-367)."""
    from .ops import row_gather
    if guard is not None:
        geometry, weight, tolerance, counter = guard
        out = _guarded_fit(features, geometry, source_ids, basis_ids, weight, tolerance)
        counter.append(out[5])
        return out[:5]
    q = row_gather(features, source_ids)
    b = row_gather(features, basis_ids)
    _, idx = similarity_topk(q, b, 4)
    support = basis_ids[idx]
    return (support,) + _feature_fit(features, source_ids, support)


def _fit_temporal_local(features, basis_ids, *, frames: int, patches: int, threshold: float, source_ids,
                        guard=None):
    """_adaptive_fit_temporal_local (sparse_convex.py:440-684), feature route: sources of frames
    [b, b + 8) (b = 1, 9, ...) take their top-4 among the basis of frame 0 and frames
    [max(1, b - 1), min(F - 1, b + 8)] (one grouped tcgen05 search for all groups), one fused
    solve, the certificate; uncertified rows (and reference-frame sources, which no group covers)
    take the global route.  With ``guard`` = (geometry, weight, tolerance, counter) every search
    is the Pareto-guarded geometry route (_guarded_fit); each launch's chosen flags are appended
    to ``counter``.  basis_ids / source_ids sorted ascending.
    -> (support ids [S,4], weights, cosine, residual, reconstruction norm)."""
    from .ops import row_gather
    dev = features.device
    n = source_ids.numel()
    if n == 0 or basis_ids.numel() == 0:
        empty = torch.zeros((n, 4), device=dev, dtype=torch.long)
        return (empty,) + _feature_fit(features, source_ids, empty)
    starts = list(range(1, frames, LOCAL_FRAME_GROUP))
    ends = [min(b + LOCAL_FRAME_GROUP, frames) for b in starts]
    lo = [max(1, b - 1) for b in starts]
    hi = [min(frames - 1, e) for e in ends]
    cut = torch.tensor([1] + starts + ends + lo + [h + 1 for h in hi], device=dev) * patches
    g = len(starts)
    pos = torch.cat([torch.searchsorted(source_ids, cut[1:1 + 2 * g]),
                     torch.searchsorted(basis_ids, torch.cat([cut[:1], cut[1 + 2 * g:]]))]).tolist()  # one sync
    s_pos, b_pos = pos[:2 * g], pos[2 * g:]
    s_begin, s_end = s_pos[:g], s_pos[g:]
    b0, b_lo, b_hi = b_pos[0], b_pos[1:1 + g], b_pos[1 + g:]
    # one query row per grouped source, one concatenated basis list per group
    # (consecutive groups: frames [1, 9), [9, 17), ... so their sources form one contiguous run)
    b_lists, qb, bb = [], [0], [0]
    for k in range(g):
        b_lists.append(torch.cat([basis_ids[:b0], basis_ids[b_lo[k]:b_hi[k]]]))
        qb.append(qb[-1] + s_end[k] - s_begin[k])
        bb.append(bb[-1] + b_lists[-1].numel())
    rows = torch.arange(s_begin[0], s_end[-1], device=dev)
    local_basis = torch.cat(b_lists)
    support = basis_ids[:1].expand(n, 4).clone()
    weights = torch.zeros((n, 4), device=dev, dtype=torch.float32)
    cos, res, nrm = (torch.zeros(n, device=dev, dtype=torch.float32) for _ in range(3))
    assigned = torch.zeros(n, device=dev, dtype=torch.bool)
    if rows.numel() and guard is not None:
        geometry, weight, tolerance, counter = guard
        fit = _guarded_fit(features, geometry, source_ids[rows], local_basis, weight, tolerance,
                           query_begin=torch.tensor(qb), basis_begin=torch.tensor(bb))
        counter.append(fit[5])
        chosen, fit = fit[0], fit[1:5]
    elif rows.numel():
        _, idx = similarity_topk(row_gather(features, source_ids[rows]), row_gather(features, local_basis), 4,
                                 query_begin=torch.tensor(qb), basis_begin=torch.tensor(bb))
        chosen = local_basis[idx]
        fit = _feature_fit(features, source_ids[rows], chosen)
    if rows.numel():
        support[rows], weights[rows] = chosen, fit[0]
        cos[rows], res[rows], nrm[rows] = fit[1], fit[2], fit[3]
        assigned[rows] = True
    fallback = torch.nonzero(~(assigned & _certified(cos, res, nrm, threshold))).flatten()
    if fallback.numel():
        gfit = _fit_global(features, basis_ids, source_ids[fallback], guard)
        support[fallback], weights[fallback] = gfit[0], gfit[1]
        cos[fallback], res[fallback], nrm[fallback] = gfit[2], gfit[3], gfit[4]
    return support, weights, cos, res, nrm


class _EventTables:
    """The feature-independent part of the TTT event-base selection for one clip: the sensitive
    patches, their time / xyz bins, the bins' mean geometry and the score terms that do not
    depend on the features, the bins kept when there are more than ``amount``, and the fill
    count.  The global layers of one forward pass the same labels, sensitivity and geometry, so
    the planner computes these once per clip (the last few clips are kept) and only the feature
    terms per layer."""

    _cache: list = []
    _KEEP = 4

    def __init__(self, geometry, labels, sensitivity, excluded, patches: int, amount: int, geometry_weight: float):
        self.inputs = (geometry.clone(), labels.clone(), sensitivity.clone(), excluded.clone())
        self.patches, self.amount, self.weight = patches, amount, geometry_weight
        ids = torch.nonzero((labels == 1) & ~excluded).flatten()
        self.ids = ids
        self.n = ids.numel()
        if amount <= 0 or self.n == 0:
            return
        geo = geometry.index_select(0, ids)
        xyz = torch.floor((geo[:, :3] + 4.0) / 0.5).long().clamp(0, 31)
        time_bin = (ids // patches) // 4
        code = ((time_bin * 37 + xyz[:, 0]) * 37 + xyz[:, 1]) * 37 + xyz[:, 2]
        _, inverse = torch.unique(code, return_inverse=True)
        groups = int(inverse.max()) + 1
        counts = torch.bincount(inverse, minlength=groups)
        order = inverse.argsort(stable=True)
        center_g = torch.segment_reduce(geo.index_select(0, order), "mean", lengths=counts)
        sens = sensitivity.index_select(0, ids)
        self.inverse, self.groups, self.counts, self.order = inverse, groups, counts, order
        self.geo_term = geometry_weight * (geo - center_g.index_select(0, inverse)).square().sum(-1)
        self.sens_term = 0.005 * sens
        self.sens = sens
        self.select = None
        if groups > amount:
            group_score = torch.segment_reduce(sens.index_select(0, order), "mean", lengths=counts) * counts.float().sqrt()
            self.select = group_score.topk(amount).indices
        self.fill = min(amount - groups, self.n - groups) if groups < amount else 0

    def matches(self, geometry, labels, sensitivity, excluded, patches, amount, geometry_weight) -> bool:
        g, l, s, e = self.inputs
        if (patches, amount, geometry_weight) != (self.patches, self.amount, self.weight):
            return False
        if g.shape != geometry.shape or l.shape != labels.shape or s.shape != sensitivity.shape \
                or e.shape != excluded.shape or g.device != geometry.device:
            return False
        same = ((g != geometry).any() | (l != labels).any() | (s != sensitivity).any() | (e != excluded).any())
        return not bool(same)

    @classmethod
    def get(cls, *args):
        for t in cls._cache:
            if t.matches(*args):
                return t
        t = cls(*args)
        cls._cache = [t] + cls._cache[: cls._KEEP - 1]
        return t


def _ttt_event_bases(features, geometry, labels, sensitivity, excluded, *, patches: int, amount: int,
                     geometry_weight: float) -> torch.Tensor:
    """TTT-proposed event bases (sparse_convex.py:1268-1324) on the device: sensitive patches
    (label 1, not excluded) binned by 4-frame time bin and 0.5-wide xyz bins; per bin the patch
    whose feature is closest to the bin's normalised mean feature, with a geometry penalty and a
    0.005 sensitivity bonus (lowest id on ties); with more bins than ``amount`` the bins with the
    largest mean sensitivity x sqrt(size) win; with fewer, the most sensitive remaining patches
    fill up.  Sorted unique patch ids.  The binning and every feature-independent term come
    from the clip's cached _EventTables; per call only the feature terms are computed."""
    tab = _EventTables.get(geometry, labels, sensitivity, excluded, patches, amount, geometry_weight)
    ids = tab.ids
    if amount <= 0 or tab.n == 0:
        return ids[:0]
    inverse = tab.inverse
    feat = features.index_select(0, ids).float()
    mean_f = torch.segment_reduce(feat.index_select(0, tab.order), "mean", lengths=tab.counts)
    center_f = torch.nn.functional.normalize(mean_f, dim=-1, eps=1e-8)
    score = (feat * center_f.index_select(0, inverse)).sum(-1) - tab.geo_term + tab.sens_term
    best = torch.full((tab.groups,), -torch.inf, device=ids.device)
    best.scatter_reduce_(0, inverse, score, reduce="amax", include_self=True)
    sentinel = labels.numel()
    candidate = torch.where(score == best.index_select(0, inverse), ids, torch.full_like(ids, sentinel))
    rep = torch.full((tab.groups,), sentinel, device=ids.device, dtype=torch.long)
    rep.scatter_reduce_(0, inverse, candidate, reduce="amin", include_self=True)  # every bin has a member
    if tab.select is not None:
        rep = rep.index_select(0, tab.select)
    elif tab.fill > 0:
        chosen = torch.zeros(sentinel, device=ids.device, dtype=torch.bool)
        chosen[rep] = True
        masked = torch.where(chosen.index_select(0, ids), torch.full_like(tab.sens, -torch.inf), tab.sens)
        rep = torch.cat([rep, ids.index_select(0, masked.topk(tab.fill).indices)])
    return torch.sort(rep).values


@torch.no_grad()
def build_ttt_protected_uniform_convex_plan(
        tokens: torch.Tensor, *, frames: int, tokens_per_frame: int, patch_token_start: int,
        patch_hw: tuple[int, int], threshold: float, labels: torch.Tensor, sensitivity: torch.Tensor,
        geometry: torch.Tensor, max_support: int = 4, preserve_queries: bool = False,
        preserve_destination_keys: bool | None = None, top1_prune_threshold: float = .95,
        sensitive_event_ratio: float = .02, selection_geometry_weight: float = .01,
        support_geometry_weight: float = 0.0, support_geometry_guard_tolerance: float | None = None,
        fixed_dynamic_mask: torch.Tensor | None = None) -> WeightedBilinearTokenPlan:
    """Protected uniform skeleton plus TTT-proposed residual event bases, the reference's
    released planner (vggt_omega/models/sparse_convex.py:1738-2016), on B200.

    Steps: bf16 patch features (row normalisation kernel, eps 1e-8); the protected uniform
    skeleton with 4x4 top-1 pruning (vb200_row_max_dot); TTT event proposals (at most twice the
    freed budget) kept only where the skeleton cannot certify them; the temporal-local support
    search (grouped tcgen05 top-4 per 8-frame group), the fused Gram + 32-step projected-gradient
    fit and its certificate, with the global route for uncertified sources; sources that still
    fail stay physical; the plan's CSR and masses on the device.  Supports come from the feature
    route (support_geometry_weight = 0, the default) or, with support_geometry_weight > 0 and a
    guard tolerance (the released configuration: 0.01 and 0), from the Pareto-guarded geometry
    route: a top-16 feature shortlist re-ranked by 4-D distance, both sets fitted, the joint set
    kept only where it is no worse in feature space and strictly better in 4-D.  The joint-metric
    route (a geometry weight without a guard tolerance) and the fixed-topology /
    fixed-dynamic-basis variants behind environment switches are not built."""
    import os
    if tokens.shape[0] != 1 or max_support != 4:
        raise ValueError("protected TTT planner requires batch one and four supports")
    if support_geometry_weight and support_geometry_guard_tolerance is None:
        raise ValueError("the joint-metric support route (support_geometry_weight without a guard tolerance) "
                         "is not built; pass support_geometry_guard_tolerance")
    if support_geometry_guard_tolerance is not None and support_geometry_guard_tolerance < 0:
        raise ValueError("the 4-D feature guard tolerance must be nonnegative")
    if os.environ.get("VGGT_TTT_FIXED_TOPOLOGY", "0") == "1" or os.environ.get("VGGT_TTT_FIXED_DYNAMIC_BASIS_PATH"):
        raise ValueError("the fixed-topology and fixed-dynamic-basis planner variants are not built")
    C.require_cuda(tokens, "build_ttt_protected_uniform_convex_plan")
    height, width = patch_hw
    patches = height * width
    patch_count = frames * patches
    total, dev = tokens.shape[1], tokens.device
    if total != frames * tokens_per_frame or patch_token_start + patches != tokens_per_frame:
        raise ValueError("invalid protected TTT token layout")
    if labels.numel() != patch_count or sensitivity.numel() != patch_count:
        raise ValueError("TTT labels/sensitivity must contain one value per patch token")
    if geometry.shape != (patch_count, 4):
        raise ValueError("TTT geometry must be [frames*patches,4]")
    if selection_geometry_weight < 0 or support_geometry_weight < 0:
        raise ValueError("TTT geometry weights must be nonnegative")
    labels = labels.to(device=dev, dtype=torch.long).reshape(-1)
    sensitivity = sensitivity.to(device=dev, dtype=torch.float32).reshape(-1)
    geometry = geometry.to(device=dev, dtype=torch.float32)
    patch_ids = (torch.arange(frames, device=dev)[:, None] * tokens_per_frame + patch_token_start
                 + torch.arange(patches, device=dev)[None]).flatten()
    features = row_normalize_bf16(tokens[0], patch_ids, eps=1e-8)
    guard_counter: list[torch.Tensor] = []
    guard = ((geometry.contiguous(), float(support_geometry_weight), float(support_geometry_guard_tolerance), [])
             if support_geometry_weight else None)

    # protected uniform skeleton (sparse_convex.py:1371-1434)
    tab = ttt_skeleton_tables(frames, tuple(patch_hw))
    first = tab["first"].to(dev)
    pruned = torch.zeros(0, device=dev, dtype=torch.bool)
    if frames > 1:
        anchors = tab["anchors"].to(dev)
        valid = anchors >= 0
        query = anchors.clamp_min(0).reshape(-1)
        targets = tab["targets"].to(dev).reshape(query.numel(), -1)
        top1 = torch.empty(query.numel(), device=dev, dtype=torch.float32)
        C.check(C.lib().vb200_row_max_dot(C.dtype_code(features.dtype), features.data_ptr(), features.shape[0],
                                          features.stride(0), query.data_ptr(), targets.data_ptr(), targets.shape[1],
                                          query.numel(), features.shape[1], top1.data_ptr(), C.stream_of(dev)),
                "row_max_dot")
        removable = valid & (torch.arange(4, device=dev) > 0)
        pruned = removable & (top1.view_as(valid) >= top1_prune_threshold)
        stable = torch.unique(torch.cat([first, anchors[valid & ~pruned]]))
    else:
        stable = first
    freed = int(pruned.sum())
    pruning = top1_prune_threshold <= 1.0
    budget = freed if pruning else int(round(sensitive_event_ratio * patch_count))
    stable_mask = torch.zeros(patch_count, device=dev, dtype=torch.bool)
    stable_mask[stable] = True

    # TTT event proposals, kept where the skeleton cannot certify them (:1815-1880)
    if fixed_dynamic_mask is not None:
        if fixed_dynamic_mask.numel() != patch_count:
            raise ValueError("predicted fixed dynamic basis mask has the wrong token count")
        event = torch.nonzero(fixed_dynamic_mask.to(device=dev, dtype=torch.bool).reshape(-1)).flatten()
        event = event[~stable_mask.index_select(0, event)]
        proposal = event
    else:
        proposal = _ttt_event_bases(features, geometry, labels, sensitivity, stable_mask, patches=patches,
                                    amount=2 * budget, geometry_weight=selection_geometry_weight)
        event = proposal[:0]
        if budget and proposal.numel():
            efit = _fit_temporal_local(features, stable, frames=frames, patches=patches, threshold=threshold,
                                       source_ids=proposal, guard=guard)
            cand = torch.nonzero(~_certified(efit[2], efit[3], efit[4], threshold)).flatten()
            if cand.numel() > budget:
                priority = sensitivity.index_select(0, proposal.index_select(0, cand)) * efit[3].index_select(0, cand)
                cand = cand.index_select(0, priority.topk(budget).indices)
            event = proposal.index_select(0, cand)

    # every remaining patch: temporal-local fit, certificate, global fallback (:1882-1902)
    basis = torch.unique(torch.cat([stable, event]))
    basis_mask = torch.zeros(patch_count, device=dev, dtype=torch.bool)
    basis_mask[basis] = True
    source = torch.nonzero(~basis_mask).flatten()
    if guard is not None:  # the reported count covers the final fit, as the reference's does
        guard = guard[:3] + (guard_counter,)
    support, weights, cos, res, nrm = _fit_temporal_local(features, basis, frames=frames, patches=patches,
                                                          threshold=threshold, source_ids=source, guard=guard)
    accepted = _certified(cos, res, nrm, threshold)
    rows = torch.nonzero(accepted).flatten()
    source_local = source.index_select(0, rows)
    support_local = support.index_select(0, rows)
    weights = weights.index_select(0, rows).float().contiguous()

    # the plan (:1932-1976)
    kept_mask = torch.ones(patch_count, device=dev, dtype=torch.bool)
    kept_mask[source_local] = False
    keep_local = torch.nonzero(kept_mask).flatten()
    special = (torch.arange(frames, device=dev)[:, None] * tokens_per_frame
               + torch.arange(patch_token_start, device=dev)[None]).flatten()
    keep = torch.sort(torch.cat([special, patch_ids.index_select(0, keep_local)])).values
    original_to_compact = torch.full((total,), -1, device=dev, dtype=torch.long)
    original_to_compact[keep] = torch.arange(keep.numel(), device=dev)
    parent = original_to_compact.index_select(0, patch_ids.index_select(0, support_local.reshape(-1)))
    parent = parent.view(-1, 4)
    counts = torch.stack([(parent < 0).any().long(), (~accepted).sum()]
                         + [c.sum().long() for c in guard_counter]).tolist()  # one sync for the checks
    if counts[0]:
        raise RuntimeError("protected TTT convex support must remain physical")
    source_original = patch_ids.index_select(0, source_local)
    csr = build_plan_csr(parent, weights, keep.numel(), src_rows=source_original)
    mass = csr.mass.view(1, -1, 1)
    return WeightedBilinearTokenPlan(
        csr=csr, keep=keep[None], source_original=source_original[None], source_parent_compact=parent[None],
        source_pool_weights=weights[None], source_restore_weights=weights[None], original_tokens=total,
        normalizer=mass, preserve_queries=preserve_queries,
        preserve_destination_keys=preserve_queries if preserve_destination_keys is None else preserve_destination_keys,
        dense_special_queries=True, special_query_original=special,
        special_query_compact=original_to_compact.index_select(0, special), key_log_mass=csr.log_mass[None],
        metadata={"planner": "ttt_protected_uniform_residual_convex_v1", "threshold": float(threshold),
                  "max_support": 4, "top1_prune_threshold": float(top1_prune_threshold),
                  "top1_pruning_enabled": bool(pruning), "protected_uniform_bases": int(stable.numel()),
                  "top1_pruned_uniform_bases": freed, "sensitive_event_budget": budget,
                  "sensitive_event_proposals": int(proposal.numel()), "sensitive_event_bases": int(event.numel()),
                  "fit_failure_promotions": int(counts[1]), "physical_patch_tokens": int(keep_local.numel()),
                  "selection_geometry_weight": float(selection_geometry_weight),
                  "support_geometry_weight": float(support_geometry_weight),
                  "support_geometry_guard_tolerance": support_geometry_guard_tolerance,
                  "geometry_guard_enabled": guard is not None,
                  "geometry_guard_selected": int(sum(counts[2:]))},
    )
