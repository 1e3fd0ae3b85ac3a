"""Merge step on the GPU: tcgen05 similarity GEMM with fused top-1 / top-4 epilogue against
the reference goldens and the oracle.  Indices must match bit-exactly up to exact ties: every
pick is the stable top-k of the bf16 score matrix under some admissible fp32 accumulation
order (helpers.check_topk_contract), and the returned values equal the reference's."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import admissible_bf16, check_topk_contract, to_np

pytestmark = pytest.mark.gpu


def _bf16(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev, torch.bfloat16)


def _check_topk(oracle, q, b, got_v, got_i, k, groups=None):
    """The top-k contract of helpers.check_topk_contract: every pick is the stable top-k of an
    admissible bf16 score matrix (exact ties under some fp32 accumulation order), every value
    an admissible rounding of its own score.  ``groups``: ((q0, q1), (b0, b1)) pairs; a row
    may only pick basis rows of its own group.  Returns the share of rows whose picks equal
    the oracle's exact-score ranking."""
    _, lo, hi = admissible_bf16(q, b)
    valid = None
    if groups is not None:
        valid = np.zeros(lo.shape, bool)
        for (q0, q1), (b0, b1) in groups:
            valid[q0:q1, b0:b1] = True
    check_topk_contract(lo, hi, got_v, got_i, valid)
    scores = oracle.topk_scores(q, b)
    if valid is not None:
        scores = np.where(valid, scores, -np.inf)
    ref_order = np.argsort(-scores, axis=1, kind="stable")[:, :k]
    rows = np.isfinite(np.take_along_axis(scores, ref_order[:, :1], 1)[:, 0])
    exact = np.all(got_i[rows] == ref_order[rows], axis=1)
    assert exact.mean() > 0.9, f"only {exact.mean():.4f} of the rows match the exact-score ranking"
    return exact.mean()


def test_golden_top4_and_argmax(pkg, golden, oracle, cuda_device):
    q, b = golden["topk_q"], golden["topk_b"]
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 4)
    v, i = to_np(v), i.cpu().numpy()
    scores = oracle.topk_scores(q, b)
    ref_i = golden["topk_indices"].astype(np.int64)
    np.testing.assert_array_equal(v, golden["topk_values"])
    np.testing.assert_array_equal(np.take_along_axis(scores, i, 1), np.take_along_axis(scores, ref_i, 1))
    _check_topk(oracle, q, b, v, i, 4)
    best, target = pkg.merge_argmax(_bf16(q, cuda_device), _bf16(b, cuda_device))
    np.testing.assert_array_equal(to_np(best), golden["topk_max_values"])
    np.testing.assert_array_equal(scores[np.arange(len(q)), target.cpu().numpy()], golden["topk_max_values"])


@pytest.mark.parametrize("k", [1, 4])
@pytest.mark.parametrize("shape", [(1, 4, 64), (130, 300, 128), (1000, 2100, 1024), (257, 513, 192)],
                         ids=lambda s: "x".join(map(str, s)))
def test_against_oracle(pkg, oracle, cuda_device, k, shape):
    R, Nb, D = shape
    rng = np.random.default_rng(R + Nb + D)
    q = rng.standard_normal((R, D)).astype(np.float32)
    b = rng.standard_normal((Nb, D)).astype(np.float32)
    q = oracle.round_bf16(q / np.linalg.norm(q, axis=1, keepdims=True))
    b = oracle.round_bf16(b / np.linalg.norm(b, axis=1, keepdims=True))
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), k)
    _check_topk(oracle, q, b, to_np(v), i.cpu().numpy(), k)
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("shape", [(130, 300, 128), (1000, 2100, 1024), (257, 513, 192)],
                         ids=lambda s: "x".join(map(str, s)))
def test_shortlist16_against_oracle(pkg, oracle, cuda_device, shape):
    """k = 16, the geometry-guarded route's shortlist (sparse_convex.py:263-266, 506-508)."""
    R, Nb, D = shape
    rng = np.random.default_rng(R * 3 + Nb + D)
    q = rng.standard_normal((R, D)).astype(np.float32)
    b = rng.standard_normal((Nb, D)).astype(np.float32)
    q = oracle.round_bf16(q / np.linalg.norm(q, axis=1, keepdims=True))
    b = oracle.round_bf16(b / np.linalg.norm(b, axis=1, keepdims=True))
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 16)
    assert v.shape == (R, 16) and i.shape == (R, 16)
    _check_topk(oracle, q, b, to_np(v), i.cpu().numpy(), 16)
    # the first four are the top-4 search's picks
    v4, i4 = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 4)
    assert torch.equal(i[:, :4], i4) and torch.equal(v[:, :4], v4)
    assert pkg.device_error_flags() == 0


def test_shortlist16_small_basis_and_groups(pkg, oracle, cuda_device):
    """Groups with fewer than 16 basis rows leave the remaining slots -inf / -1."""
    rng = np.random.default_rng(11)
    D = 128
    qb, bb = [0, 40, 100], [0, 5, 300]
    q = oracle.round_bf16(rng.standard_normal((100, D)).astype(np.float32) / 11)
    b = oracle.round_bf16(rng.standard_normal((300, D)).astype(np.float32) / 11)
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 16,
                               query_begin=torch.tensor(qb), basis_begin=torch.tensor(bb))
    v, i = to_np(v), i.cpu().numpy()
    assert np.all(i[:40, 5:] == -1) and np.all(np.isneginf(v[:40, 5:]))
    assert np.all((i[:40, :5] >= 0) & (i[:40, :5] < 5)) and np.all((i[40:] >= 5) & (i[40:] < 300))
    scores = oracle.topk_scores(q, b)
    np.testing.assert_array_equal(np.sort(i[:40, :5], axis=1), np.tile(np.arange(5), (40, 1)))
    _check_topk(oracle, q[40:], b[5:], v[40:], i[40:] - 5, 16)
    assert np.all(np.diff(v[:40, :5], axis=1) <= 0) and np.all(np.isfinite(scores))
    assert pkg.device_error_flags() == 0


def test_groups(pkg, oracle, cuda_device):
    rng = np.random.default_rng(7)
    D = 256
    qb = [0, 300, 300, 700, 1000]   # group 1 has no query rows
    bb = [0, 500, 600, 600, 1200]   # group 2 has no basis rows
    q = oracle.round_bf16(rng.standard_normal((1000, D)).astype(np.float32) / 16)
    b = oracle.round_bf16(rng.standard_normal((1200, D)).astype(np.float32) / 16)
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 4,
                               query_begin=torch.tensor(qb), basis_begin=torch.tensor(bb))
    v, i = to_np(v), i.cpu().numpy()
    groups = [((qb[g], qb[g + 1]), (bb[g], bb[g + 1])) for g in range(4)]
    _check_topk(oracle, q, b, v, i, 4, groups=groups)
    # rows of the group without basis rows: -inf / -1
    assert np.all(i[300:700] == -1) and np.all(np.isneginf(v[300:700]))


def test_streaming_top4_transposed_basis(pkg, oracle, cuda_device):
    rng = np.random.default_rng(3)
    q = oracle.round_bf16(rng.standard_normal((200, 128)).astype(np.float32) / 11)
    b = oracle.round_bf16(rng.standard_normal((64, 128)).astype(np.float32) / 11)
    bt = _bf16(b, cuda_device).t()  # [D, N] view, as the reference passes it
    v, i = pkg.streaming_top4(_bf16(q, cuda_device), bt)
    assert i.dtype == torch.int64 and v.dtype == torch.float32
    _check_topk(oracle, q, b, to_np(v), i.cpu().numpy(), 4)
    with pytest.raises(ValueError, match="at least four"):
        pkg.streaming_top4(_bf16(q, cuda_device), bt[:, :3])


@pytest.mark.parametrize("half", [100, 300])  # 300: the copies fall in a different basis tile
def test_exact_ties_prefer_lower_index(pkg, oracle, cuda_device, half):
    """Basis rows duplicated (row c and row c + half are identical), so every score appears
    twice and ties are exact in any accumulation order: the top-4 must list equal scores with
    the lower index first (the strict-> running top-k and the stable sort of the reference).
    Some queries are exact negatives of a basis row, so negative and zero scores occur too."""
    rng = np.random.default_rng(11)
    D = 64
    b1 = oracle.round_bf16(rng.standard_normal((half, D)).astype(np.float32) / 8)
    b = np.concatenate([b1, b1])
    q = oracle.round_bf16(rng.standard_normal((260, D)).astype(np.float32) / 8)
    q[:20] = -b1[:20]
    q[20:30] = 0.0
    v, i = pkg.similarity_topk(_bf16(q, cuda_device), _bf16(b, cuda_device), 4)
    v, i = to_np(v), i.cpu().numpy()
    for r in range(len(q)):
        pairs = list(zip(-v[r], i[r]))
        assert pairs == sorted(pairs), f"row {r}: not ordered by (score desc, index asc): {pairs}"
        for c in i[r]:
            if c >= half:  # the later copy may only appear after its earlier twin
                assert c - half in i[r] and list(i[r]).index(c - half) < list(i[r]).index(c), (r, i[r])
    assert np.all(i[20:30] == np.arange(4))  # all scores 0: the four lowest indices
    _check_topk(oracle, q, b, v, i, 4)
