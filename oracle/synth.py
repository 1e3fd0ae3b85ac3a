"""Seeded synthetic inputs with the shapes and value distributions of the workloads the
reference's metric is quoted on (no dataset or checkpoint is involved).

* ``c1_inputs``   config 1: N = frames*1029 tokens merged to M, Q/K/V ~ N(0,1), integer masses
                  from a multinomial, top-4 parents distinct per token, softmax(N(0,1)) weights.
* ``zipf_plan``   config 5: parents drawn Zipf(s) over [0, M) (distinct per source),
                  Dirichlet(1,1,1,1) weights.
* ``uniform_keep``  an evenly spaced keep set of exactly K tokens per frame group.
"""
from __future__ import annotations

import numpy as np

__all__ = ["c1_inputs", "zipf_plan", "uniform_keep", "random_plan"]


def random_plan(rng: np.random.Generator, N: int, M: int, corners: int = 4):
    """keep = M sorted distinct tokens, sources = the rest, each with `corners` distinct
    parents in [0, M) and softmax(N(0,1)) weights."""
    keep = np.sort(rng.choice(N, size=M, replace=False))
    mask = np.ones(N, dtype=bool)
    mask[keep] = False
    src = np.nonzero(mask)[0]
    S = src.size
    parent = np.empty((S, corners), dtype=np.int64)
    for s in range(S):
        parent[s] = rng.choice(M, size=corners, replace=False)
    logits = rng.standard_normal((S, corners)).astype(np.float32)
    w = np.exp(logits - logits.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return keep, src, parent, w


def c1_inputs(seed: int = 0, frames: int = 4, tokens_per_frame: int = 1029, heads: int = 16,
              head_dim: int = 64, merged: int | None = None):
    """Config-1 style inputs (fp32): q [1,H,N,64], k/v [1,H,M,64], mass = 1 + Multinomial(N-M)
    (positive integers summing to N), and a random top-4 plan."""
    rng = np.random.default_rng(seed)
    N = frames * tokens_per_frame
    M = merged if merged is not None else N // 4
    q = rng.standard_normal((1, heads, N, head_dim)).astype(np.float32)
    k = rng.standard_normal((1, heads, M, head_dim)).astype(np.float32)
    v = rng.standard_normal((1, heads, M, head_dim)).astype(np.float32)
    mass = (1 + rng.multinomial(N - M, np.full(M, 1.0 / M))).astype(np.float32)
    keep, src, parent, w = random_plan(rng, N, M)
    return dict(q=q, k=k, v=v, mass=mass, log_mass=np.log(mass).astype(np.float32),
                keep=keep, src=src, parent=parent, weights=w, N=N, M=M)


def zipf_plan(seed: int, N: int, M: int, s: float = 1.1, corners: int = 4):
    """Config-5 plan: keep = M evenly spaced tokens, sources = the rest; each source draws
    `corners` distinct parents from Zipf(s) over [0, M) (rank r has weight r^-s, ranks mapped
    to compact ids by a seeded permutation) and Dirichlet(1,...,1) weights."""
    rng = np.random.default_rng(seed)
    keep = np.linspace(0, N, M, endpoint=False).astype(np.int64)
    mask = np.ones(N, dtype=bool)
    mask[keep] = False
    src = np.nonzero(mask)[0]
    S = src.size
    p = np.arange(1, M + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    perm = rng.permutation(M)
    draws = rng.choice(M, size=(S, corners * 3), p=p)
    parent = np.empty((S, corners), dtype=np.int64)
    for i in range(S):
        row = draws[i]
        _, first = np.unique(row, return_index=True)
        picked = row[np.sort(first)][:corners]
        while picked.size < corners:  # rejection for distinctness
            extra = rng.choice(M, size=corners * 3, p=p)
            row = np.concatenate([picked, extra])
            _, first = np.unique(row, return_index=True)
            picked = row[np.sort(first)][:corners]
        parent[i] = perm[picked]
    w = rng.dirichlet(np.ones(corners), size=S).astype(np.float32)
    return keep, src, parent, w


def uniform_keep(frames: int, tokens_per_frame: int, special: int, keep_per_group: int,
                 group_frames: int) -> np.ndarray:
    """Keep set of exactly ``keep_per_group`` tokens per group of ``group_frames`` frames: all
    special tokens plus evenly spaced patch tokens (anchor_k = floor(k * P / A))."""
    assert frames % group_frames == 0
    keep = []
    patches = tokens_per_frame - special
    for g in range(frames // group_frames):
        f0 = g * group_frames
        spec = [(f0 + f) * tokens_per_frame + t for f in range(group_frames) for t in range(special)]
        n_anchor = keep_per_group - len(spec)
        group_patches = np.array([(f0 + f) * tokens_per_frame + special + t
                                  for f in range(group_frames) for t in range(patches)])
        pick = (np.arange(n_anchor, dtype=np.int64) * group_patches.size) // n_anchor
        keep.extend(spec)
        keep.extend(group_patches[pick].tolist())
    return np.sort(np.array(keep, dtype=np.int64))
