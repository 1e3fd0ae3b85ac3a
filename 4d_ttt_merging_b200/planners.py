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

__all__ = ["build_fastvggt_plan", "build_uniform_convex_plan", "fastvggt_tables", "uniform_keep_layout"]

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
    csr = build_plan_csr(parent, alpha, K, src_rows=dl["source"])
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
        hit = {k: lay[k].to(dev) for k in ("keep", "source", "special", "special_compact")}
        hit["source_keep"] = torch.cat([hit["source"], hit["keep"]])  # feature-row order of the planner
        _DEVICE_LAYOUTS[key] = hit
    return hit
