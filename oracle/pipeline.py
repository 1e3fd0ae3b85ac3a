"""numpy restatement of one benchmark step (TEST ORACLE / CPU baseline): the four-support
convex merge plan with a uniform keep set, then the global-attention block with that plan.

The plan follows the reference's sparse-convex planners (vggt_omega/models/sparse_convex.py):
bf16 cosine top-4 support retrieval inside frame groups (:546-552), Gram / rhs of the supports
and the 32-step projected-gradient simplex fit (:2308-2321, sparse_convex_kernels.py:214-280),
mass = 1 + pooled weights and key_log_mass = log(mass) (:2448-2470).  The keep set is the
uniform anchor layout of 4d_ttt_merging_b200.planners.uniform_keep_layout, restated here.
The block is ``ref.global_attention_forward`` without dense special queries.
"""
from __future__ import annotations

import numpy as np

from . import ref

__all__ = ["uniform_layout", "convex_plan", "block_step"]


def uniform_layout(frames: int, tokens_per_frame: int, special: int, merge_factor: int, group_frames: int):
    """Keep set: every special token plus evenly spaced patch anchors (anchor k of a group's
    P patches is patch floor(k * P / A)), total // merge_factor tokens split evenly over the
    frame groups; sources are the other tokens.  Returns keep, source and per-group ranges."""
    total = frames * tokens_per_frame
    groups = frames // group_frames
    base, extra = divmod(total // merge_factor, groups)
    patches = tokens_per_frame - special
    keep, src, qb, bb = [], [], [0], [0]
    for g in range(groups):
        f0 = g * group_frames
        fr = np.arange(f0, f0 + group_frames)
        spec = (fr[:, None] * tokens_per_frame + np.arange(special)[None]).ravel()
        gp = (fr[:, None] * tokens_per_frame + special + np.arange(patches)[None]).ravel()
        n_anchor = base + (1 if g < extra else 0) - spec.size
        anchors = gp[(np.arange(n_anchor) * gp.size) // n_anchor]
        kg = np.sort(np.concatenate([spec, anchors]))
        mask = np.ones(group_frames * tokens_per_frame, bool)
        mask[kg - f0 * tokens_per_frame] = False
        sg = np.nonzero(mask)[0] + f0 * tokens_per_frame
        keep.append(kg)
        src.append(sg)
        qb.append(qb[-1] + sg.size)
        bb.append(bb[-1] + kg.size)
    return np.concatenate(keep), np.concatenate(src), np.array(qb), np.array(bb)


def _normalize_bf16(x):
    x64 = np.asarray(x, np.float64)
    n = np.sqrt((x64 * x64).sum(axis=1, keepdims=True))
    return ref.round_bf16((x64 / np.maximum(n, 1e-12)).astype(np.float32))


def convex_plan(tokens, layout, steps: int = 32):
    """tokens [N, D]; returns dict(keep, source, parent (compact ids), weights, normalizer)."""
    keep, src, qb, bb = layout
    feat = _normalize_bf16(tokens)
    parent = np.empty((src.size, 4), np.int64)
    for g in range(len(qb) - 1):
        q = feat[src[qb[g]:qb[g + 1]]]
        b = feat[keep[bb[g]:bb[g + 1]]]
        _, idx = ref.similarity_topk(q, b, 4)
        parent[qb[g]:qb[g + 1]] = idx + bb[g]
    sup = feat[keep[parent]].astype(np.float64)  # [S,4,D]
    x = feat[src].astype(np.float64)
    gram = np.einsum("sid,sjd->sij", sup, sup).astype(np.float32)
    rhs = np.einsum("sid,sd->si", sup, x).astype(np.float32)
    w = ref.projected_gradient(gram, rhs, steps)
    norm = ref.normalizer(parent, w, keep.size)
    return dict(keep=keep, source=src, parent=parent, weights=w, normalizer=norm,
                special=np.zeros(0, np.int64), special_compact=np.zeros(0, np.int64))


def block_step(tokens, params: dict, layout, heads: int = 16):
    """One benchmark step: plan + block forward (fp64/fp32 numpy).  tokens [N, D]."""
    plan = convex_plan(tokens, layout)
    return ref.global_attention_forward(tokens, params, plan, heads=heads, preserve_queries=False,
                                        dense_special=False)
