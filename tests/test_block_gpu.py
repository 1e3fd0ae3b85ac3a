"""The global-attention call site end to end on the GPU: GlobalAttention.forward with a token
plan against the reference's own SelfAttention.forward (golden vectors, fp32) and, in bf16
under autocast, against the oracle; plus the device planners."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import admissible_bf16, assert_close, check_topk_contract, to_np

pytestmark = pytest.mark.gpu


def _module(pkg, golden, tag, dev):
    params = {k[len(tag) + 3:]: v for k, v in golden.items() if k.startswith(f"{tag}_p_")}
    dim = params["qkv.weight"].shape[1]
    m = pkg.GlobalAttention(dim, 2, device=dev)
    m.load_reference_state({k: torch.from_numpy(v).to(dev) for k, v in params.items()})
    return m, params


def _plan(pkg, golden, tag, dev, preserve):
    t = lambda k, dt=torch.long: torch.from_numpy(golden[f"{tag}_{k}"]).to(dev, dt)
    norm = t("normalizer", torch.float32).view(1, -1, 1)
    return pkg.WeightedBilinearTokenPlan(
        keep=t("keep")[None], source_original=t("source")[None], source_parent_compact=t("parent")[None],
        source_pool_weights=t("weights", torch.float32)[None], source_restore_weights=t("weights", torch.float32)[None],
        original_tokens=golden[f"{tag}_x"].shape[1], normalizer=norm, preserve_queries=preserve,
        preserve_destination_keys=preserve, dense_special_queries=True, special_query_original=t("special"),
        special_query_compact=t("special_compact"), key_log_mass=norm[..., 0].log())


@pytest.mark.parametrize("tag,preserve", [("block_compact_q", False), ("block_preserve_q", True)])
def test_block_fp32_matches_reference(pkg, golden, cuda_device, tag, preserve):
    m, _ = _module(pkg, golden, tag, cuda_device)
    plan = _plan(pkg, golden, tag, cuda_device, preserve)
    x = torch.from_numpy(golden[f"{tag}_x"]).to(cuda_device)
    torch.backends.cuda.matmul.allow_tf32 = False
    with torch.no_grad():
        y = m(x, token_plan=plan)
    assert_close(to_np(y), golden[f"{tag}_y"], "f32", tol=2e-5)


@pytest.mark.parametrize("tag,preserve", [("block_compact_q", False), ("block_preserve_q", True)])
def test_block_bf16_autocast(pkg, golden, oracle, cuda_device, tag, preserve):
    m, params = _module(pkg, golden, tag, cuda_device)
    plan = _plan(pkg, golden, tag, cuda_device, preserve)
    x = torch.from_numpy(golden[f"{tag}_x"]).to(cuda_device)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x, token_plan=plan)
    assert y.dtype == torch.bfloat16
    pd = {k: golden[f"{tag}_{k}"] for k in ("keep", "source", "parent", "weights", "normalizer", "special",
                                            "special_compact")}
    ref = oracle.global_attention_forward(golden[f"{tag}_x"][0], params, pd, heads=2, preserve_queries=preserve)
    assert_close(to_np(y[0]), ref, "bf16")


def test_fastvggt_plan_matches_reference(pkg, golden, cuda_device):
    tokens = torch.from_numpy(golden["fast_tokens"]).to(cuda_device)
    plan = pkg.build_fastvggt_plan(tokens, frames=3, tokens_per_frame=69, patch_token_start=5, patch_hw=(8, 8),
                                   merge_ratio=0.5, protect_ratio=0.1, seed=3)
    np.testing.assert_array_equal(plan.keep[0].cpu().numpy(), golden["fast_keep"])
    np.testing.assert_array_equal(plan.inverse[0].cpu().numpy(), golden["fast_inverse"])
    assert pkg.device_error_flags() == 0


def _bf16_ulps(a, b):
    """Distance in bf16 ulps between two arrays of bf16-valued floats (same sign assumed)."""
    ia = np.asarray(a, np.float32).view(np.int32) >> 16
    ib = np.asarray(b, np.float32).view(np.int32) >> 16
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


@pytest.mark.parametrize("frames", [4, 8])
def test_fastvggt_plan_large(pkg, oracle, cuda_device, frames):
    """frames x 1029 tokens, D = 1024, against the oracle restatement of build_fastvggt_plan.

    Contract (bit-exact up to exact ties): the device features are F.normalize(x).bf16 up to
    one bf16 ulp where the fp32 norm's summation order lands on a rounding boundary; each
    source's (best, target) is the stable argmax of an admissible bf16 score row
    (helpers.check_topk_contract); keep / inverse equal, bit for bit, the reference's ranking
    (stable descending sort, token_merging.py:1112-1121) applied to the device scores; and where
    the plan differs from the oracle's exact-score plan, the differing choices are ties: both
    targets have overlapping admissible score ranges, and every source merged by one plan but
    not the other has an admissible best score at the merge boundary."""
    rng = np.random.default_rng(2 + frames)
    tpf, pts, hw, ratio = 1029, 5, (32, 32), 0.5
    total = frames * tpf
    tok = rng.standard_normal((total, 1024)).astype(np.float32)
    x = torch.from_numpy(tok).to(cuda_device)
    plan = pkg.build_fastvggt_plan(x[None], frames=frames, tokens_per_frame=tpf, patch_token_start=pts,
                                   patch_hw=hw, merge_ratio=ratio)
    _, _, _, _, src_o, dst_o = oracle.fastvggt_plan(
        tok, frames=frames, tokens_per_frame=tpf, patch_token_start=pts, patch_hw=hw, merge_ratio=ratio)
    src_t, dst_t, removed = pkg.planners.fastvggt_tables(frames, tpf, pts, hw, ratio, 0.10, 0)
    np.testing.assert_array_equal(src_t.numpy(), src_o)
    np.testing.assert_array_equal(dst_t.numpy(), dst_o)
    assert removed == oracle.fastvggt_removed(total, ratio, src_o.size)
    # device features vs F.normalize(x).bf16
    sf = pkg.row_normalize_bf16(x, src_t.to(cuda_device))
    df = pkg.row_normalize_bf16(x, dst_t.to(cuda_device))
    sf_h, df_h = to_np(sf), to_np(df)
    for got, ref in ((sf_h, oracle.normalize_bf16(tok[src_o])), (df_h, oracle.normalize_bf16(tok[dst_o]))):
        ulps = _bf16_ulps(got, ref)
        assert ulps.max() <= 1 and np.mean(ulps > 0) < 1e-3, (ulps.max(), np.mean(ulps > 0))
    # (best, target) on the device features: admissible stable argmax per source
    best, target = pkg.similarity_topk(sf, df, 1)
    best_h, target_h = to_np(best)[:, 0], target.cpu().numpy()[:, 0]
    _, lo, hi = admissible_bf16(sf_h, df_h)
    check_topk_contract(lo, hi, best_h[:, None], target_h[:, None])
    # the device ranking, bit for bit
    keep_r, inv_r = oracle.fastvggt_assign(best_h, target_h, src_o, dst_o, total, removed)
    got_keep, got_inv = plan.keep[0].cpu().numpy(), plan.inverse[0].cpu().numpy()
    np.testing.assert_array_equal(got_keep, keep_r)
    np.testing.assert_array_equal(got_inv, inv_r)
    # differences from the exact-score plan on the same features are ties
    best_o, tgt_o = (a[:, 0] for a in oracle.similarity_topk(sf_h, df_h, 1))
    merged_g = np.zeros(total, bool)
    merged_g[src_o[np.argsort(-best_h, kind="stable")[:removed]]] = True
    merged_o = np.zeros(total, bool)
    merged_o[src_o[np.argsort(-best_o, kind="stable")[:removed]]] = True
    both = np.nonzero(merged_g[src_o] & merged_o[src_o])[0]     # rows (source order) merged by both
    diff_t = both[target_h[both] != tgt_o[both]]
    s_lo, s_hi = lo[diff_t], hi[diff_t]
    a, b = target_h[diff_t], tgt_o[diff_t]
    r = np.arange(diff_t.size)
    assert np.all((s_hi[r, a] >= s_lo[r, b]) & (s_hi[r, b] >= s_lo[r, a])), "a differing target is not a tie"
    flip = np.nonzero(merged_g[src_o] != merged_o[src_o])[0]
    vb_g = np.sort(best_h)[::-1][removed - 1]
    vb_o = np.sort(best_o)[::-1][removed - 1]
    lo_max, hi_max = lo.max(axis=1), hi.max(axis=1)
    assert np.all((lo_max[flip] <= max(vb_g, vb_o)) & (hi_max[flip] >= min(vb_g, vb_o))), \
        "a source merged by only one plan does not tie the merge boundary"
    assert flip.size <= 0.01 * removed and diff_t.size <= 0.01 * both.size, (flip.size, diff_t.size)
    assert pkg.device_error_flags() == 0


def test_uniform_convex_plan(pkg, oracle, cuda_device):
    rng = np.random.default_rng(4)
    frames, tpf = 8, 1029
    tok = torch.from_numpy(rng.standard_normal((1, frames * tpf, 1024)).astype(np.float32)).to(cuda_device)
    plan = pkg.build_uniform_convex_plan(tok.bfloat16(), frames=frames, tokens_per_frame=tpf, patch_token_start=5,
                                         merge_factor=4, group_frames=4)
    N = frames * tpf
    assert plan.kept_tokens == N // 4
    w = plan.source_pool_weights[0]
    assert torch.all(w >= 0) and torch.allclose(w.sum(-1), torch.ones_like(w[:, 0]), atol=1e-5)
    mass = plan.normalizer[0, :, 0]
    assert abs(float(mass.sum()) - N) < 1.0  # convex weights: masses sum to N
    np.testing.assert_allclose(to_np(mass), oracle.normalizer(plan.source_parent_compact[0].cpu().numpy(),
                                                              to_np(w), plan.kept_tokens), rtol=1e-5)
    # supports stay inside the source's frame group
    keep = plan.keep[0].cpu().numpy()
    src = plan.source_original[0].cpu().numpy()
    par = keep[plan.source_parent_compact[0].cpu().numpy()]
    assert np.all(par // (4 * tpf) == (src // (4 * tpf))[:, None])
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("preserve,special", [(False, False), (False, True), (True, True), (True, False)])
def test_fused_qkv_path_bf16(pkg, oracle, cuda_device, preserve, special):
    """dim 256 / 4 heads in bf16: compute_attention takes the fused LayerNorm + Q||K||V
    compaction kernel; compared with the oracle restatement of the reference call site."""
    rng = np.random.default_rng(5 + 2 * preserve + special)
    dim, heads, frames, tpf, n_special = 256, 4, 3, 90, 5
    N = frames * tpf
    K = 80
    m = pkg.GlobalAttention(dim, heads, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.from_numpy(rng.standard_normal(p.shape).astype(np.float32) * (0.1 if p.ndim > 1 else 0.5)))
    params = {k: to_np(v) for k, v in m.state_dict().items()}
    params["qkv.bias_mask"] = params.pop("bias_mask")
    special_ids = np.concatenate([np.arange(f * tpf, f * tpf + n_special) for f in range(frames)])
    others = np.setdiff1d(np.arange(N), special_ids)
    keep = np.sort(np.concatenate([special_ids, rng.choice(others, K - special_ids.size, replace=False)]))
    src = np.setdiff1d(np.arange(N), keep)
    parent = np.stack([rng.choice(K, 4, replace=False) for _ in src])
    w = rng.dirichlet(np.ones(4), size=src.size).astype(np.float32)
    norm = oracle.normalizer(parent, w, K)
    o2c = np.full(N, -1)
    o2c[keep] = np.arange(K)
    t = lambda a, dt=torch.long: torch.as_tensor(a, device=cuda_device, dtype=dt)
    nt = t(norm, torch.float32).view(1, -1, 1)
    plan = pkg.WeightedBilinearTokenPlan(
        keep=t(keep)[None], source_original=t(src)[None], source_parent_compact=t(parent)[None],
        source_pool_weights=t(w, torch.float32)[None], source_restore_weights=t(w, torch.float32)[None],
        original_tokens=N, normalizer=nt, preserve_queries=preserve, preserve_destination_keys=preserve,
        dense_special_queries=special, special_query_original=t(special_ids), special_query_compact=t(o2c[special_ids]),
        key_log_mass=nt[..., 0].log())
    x = oracle.round_bf16(rng.standard_normal((N, dim)).astype(np.float32))
    with torch.no_grad():
        y = m(t(x, torch.bfloat16)[None], token_plan=plan)
    pd = dict(keep=keep, source=src, parent=parent, weights=w, normalizer=norm, special=special_ids,
              special_compact=o2c[special_ids])
    ref = oracle.global_attention_forward(x, params, pd, heads=heads, preserve_queries=preserve, dense_special=special)
    assert_close(to_np(y[0]), ref, "bf16")
    assert pkg.device_error_flags() == 0


def test_step_graph_replay_matches_eager(pkg, cuda_device):
    """ShardedGlobalBlock (one rank, 8 frames, dim 1024) recorded as a CUDA graph: a replay
    gives the eager step's output bit for bit, and refilling the input buffer between replays
    gives the eager output of the new input."""
    torch.manual_seed(0)
    dev = cuda_device
    attn = pkg.GlobalAttention(1024, 16, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in attn.parameters():
            p.normal_(0.0, 0.02)
        attn.q_norm.weight.fill_(1.0)
        attn.k_norm.weight.fill_(1.0)
    block = pkg.parallel.ShardedGlobalBlock(attn, frames=8, tokens_per_frame=1029, patch_token_start=5,
                                            merge_factor=4, group_frames=4)
    gen = torch.Generator(device="cpu").manual_seed(1)
    x0 = torch.randn(1, 8 * 1029, 1024, generator=gen).to(dev, torch.bfloat16)
    x1 = torch.randn(1, 8 * 1029, 1024, generator=gen).to(dev, torch.bfloat16)
    ref0 = block.step(x0).clone()
    ref1 = block.step(x1).clone()
    buf = x0.clone()
    g = pkg.parallel.StepGraph(block, buf)
    assert g.launches > 0
    out = g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref0)
    buf.copy_(x1)
    out = g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref1)
    g.release()
    assert pkg.device_error_flags() == 0
