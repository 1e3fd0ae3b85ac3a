"""The torch restatement of the reference's CPU call sequence (oracle/torch_path.py, the timed
CPU baseline of bench.py) against the numpy oracle, on CPU: plan parents up to bf16 ties,
projected-gradient weights, masses, and the block output on the same plan."""
from __future__ import annotations

import numpy as np
import torch

from helpers import admissible_bf16, assert_close, check_topk_contract


def _params(rng, dim):
    return {
        "qkv.weight": (rng.standard_normal((3 * dim, dim)) * 0.05).astype(np.float32),
        "qkv.bias": (rng.standard_normal(3 * dim) * 0.05).astype(np.float32),
        "qkv.bias_mask": np.concatenate([np.ones(dim), np.zeros(dim), np.ones(dim)]).astype(np.float32),
        "q_norm.weight": (1 + 0.1 * rng.standard_normal(64)).astype(np.float32),
        "q_norm.bias": (0.1 * rng.standard_normal(64)).astype(np.float32),
        "k_norm.weight": (1 + 0.1 * rng.standard_normal(64)).astype(np.float32),
        "k_norm.bias": (0.1 * rng.standard_normal(64)).astype(np.float32),
        "proj.weight": (rng.standard_normal((dim, dim)) * 0.05).astype(np.float32),
        "proj.bias": (rng.standard_normal(dim) * 0.05).astype(np.float32),
    }


def test_torch_path_matches_oracle(oracle):
    from oracle import torch_path as tp
    rng = np.random.default_rng(0)
    frames, tpf, special, dim, heads = 8, 69, 5, 256, 4
    lay = oracle.pipeline.uniform_layout(frames, tpf, special, 4, 4)
    keep, src, qb, bb = lay
    x = rng.standard_normal((frames * tpf, dim)).astype(np.float32)
    params = _params(rng, dim)
    plan = tp.build_plan(torch.from_numpy(x), lay)
    np.testing.assert_array_equal(plan.keep.numpy(), keep)
    np.testing.assert_array_equal(plan.source.numpy(), src)
    # parents: stable top-4 within each frame group, up to bf16 ties
    feat = torch.nn.functional.normalize(torch.from_numpy(x), dim=-1).to(torch.bfloat16).float().numpy()
    sf, bf = feat[src], feat[keep]
    exact, lo, hi = admissible_bf16(sf, bf)
    valid = np.zeros(lo.shape, bool)
    for g in range(len(qb) - 1):
        valid[qb[g]:qb[g + 1], bb[g]:bb[g + 1]] = True
    parent = plan.parent.numpy()
    # the path's own bf16 scores (same per-group GEMM calls); torch.topk picks among equal
    # scores in its own order, which the reference leaves unspecified
    tf = torch.nn.functional.normalize(torch.from_numpy(x), dim=-1).to(torch.bfloat16)
    ts, tb = tf[torch.from_numpy(src)], tf[torch.from_numpy(keep)]
    v = np.empty(parent.shape, np.float32)
    for g in range(len(qb) - 1):
        sc = (ts[qb[g]:qb[g + 1]] @ tb[bb[g]:bb[g + 1]].T).float().numpy()
        v[qb[g]:qb[g + 1]] = np.take_along_axis(sc, parent[qb[g]:qb[g + 1]] - bb[g], 1)
    check_topk_contract(lo, hi, v, parent, valid, stable=False)
    # weights: the projected gradient on the fp32 Gram of those supports
    sup = bf[parent].astype(np.float64)
    gram = np.einsum("sid,sjd->sij", sup, sup).astype(np.float32)
    rhs = np.einsum("sid,sd->si", sup, sf.astype(np.float64)).astype(np.float32)
    np.testing.assert_allclose(plan.weights.numpy(), oracle.projected_gradient(gram, rhs, 32), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(plan.normalizer.numpy(), oracle.normalizer(parent, plan.weights.numpy(), keep.size),
                               rtol=1e-6)
    # the block on the same plan
    pd = dict(keep=keep, source=src, parent=parent, weights=plan.weights.numpy(), normalizer=plan.normalizer.numpy(),
              special=np.zeros(0, np.int64), special_compact=np.zeros(0, np.int64))
    ref = oracle.global_attention_forward(x, params, pd, heads=heads, preserve_queries=False, dense_special=False)
    got = tp.block_forward(torch.from_numpy(x), tp.params_to_torch(params), plan, heads).numpy()
    assert_close(got, ref, "f32", tol=1e-5)


def test_torch_plan_ops_match_oracle(oracle):
    """compact / restore / normalizer on a random plan (bf16 values: fp32 accumulation,
    value-dtype restore)."""
    from oracle import torch_path as tp
    rng = np.random.default_rng(1)
    N, M, C = 700, 150, 96
    keep, src, parent, w = oracle.random_plan(rng, N, M)
    mass = tp.normalizer(torch.from_numpy(parent), torch.from_numpy(w), M)
    np.testing.assert_array_equal(mass.numpy(), oracle.normalizer(parent, w, M))
    orders, lengths = tp._corner_orders(torch.from_numpy(parent), M)
    plan = tp.TorchPlan(torch.from_numpy(keep), torch.from_numpy(src), torch.from_numpy(parent), torch.from_numpy(w),
                        mass, mass.log(), orders, lengths, N)
    x = oracle.round_bf16(rng.standard_normal((N, C)).astype(np.float32))
    got = tp.compact(plan, torch.from_numpy(x).to(torch.bfloat16)).float().numpy()
    ref = oracle.compact(x, keep, src, parent, w, mass.numpy(), dtype="bf16")
    assert np.abs(got - ref).max() <= 2 ** -7 * np.abs(ref).max()
    y = oracle.round_bf16(rng.standard_normal((M, C)).astype(np.float32))
    got = tp.restore(plan, torch.from_numpy(y).to(torch.bfloat16)).float().numpy()
    np.testing.assert_array_equal(got, oracle.restore(y, keep, src, parent, w, N, dtype="bf16"))
