"""Top-4 projection, normalizer and hard-merge plans on the GPU against the reference's
golden vectors and the oracle, through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import TORCH_DTYPE, assert_close, to_np

pytestmark = pytest.mark.gpu


def _plan(pkg, keep, src, parent, w, N, normalizer=None, dev="cuda"):
    keep_t = torch.as_tensor(keep, dtype=torch.long, device=dev)[None]
    src_t = torch.as_tensor(src, dtype=torch.long, device=dev)[None]
    par_t = torch.as_tensor(parent, dtype=torch.long, device=dev)[None]
    w_t = torch.as_tensor(w, dtype=torch.float32, device=dev)[None]
    if normalizer is None:
        normalizer = pkg.deterministic_weighted_normalizer(par_t, w_t, keep_t.shape[1])
    else:
        normalizer = torch.as_tensor(normalizer, dtype=torch.float32, device=dev).view(1, -1, 1)
    return pkg.WeightedBilinearTokenPlan(
        keep=keep_t, source_original=src_t, source_parent_compact=par_t, source_pool_weights=w_t,
        source_restore_weights=w_t, original_tokens=N, normalizer=normalizer,
        key_log_mass=normalizer[..., 0].log())


def test_golden_plan_ops(pkg, golden, cuda_device):
    g = golden
    plan = _plan(pkg, g["plan_keep"], g["plan_source"], g["plan_parent"], g["plan_weights"],
                 g["plan_value"].shape[1], dev=cuda_device)
    np.testing.assert_allclose(to_np(plan.normalizer[0, :, 0]), g["plan_normalizer"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(to_np(plan.csr.mass), g["plan_normalizer"], rtol=1e-6, atol=1e-6)
    v = torch.from_numpy(g["plan_value"]).to(cuda_device)
    np.testing.assert_allclose(to_np(plan.compact(v)), g["plan_compact_f32"], rtol=1e-5, atol=1e-6)
    cb = to_np(plan.compact(v.bfloat16()))
    np.testing.assert_allclose(cb, g["plan_compact_bf16"], rtol=2 ** -7, atol=1e-6)
    assert np.mean(cb == g["plan_compact_bf16"]) > 0.99
    y = torch.from_numpy(g["plan_y"]).to(cuda_device)
    np.testing.assert_allclose(to_np(plan.restore(y)), g["plan_restore_f32"], rtol=1e-6, atol=1e-6)
    # value-dtype restore arithmetic is reproduced exactly
    np.testing.assert_array_equal(to_np(plan.restore(y.bfloat16())), g["plan_restore_bf16"])


def test_golden_config1_and_config5(pkg, oracle, golden, cuda_device):
    """The reference-generated goldens at size: config 1's restore of 1,029 merged rows to 4,116
    tokens (the golden's channels of head 5) and config 5 scaled to 8,192 tokens / 512 merged rows
    with Zipf parents (compact and restore), fp32."""
    dev = cuda_device
    c1 = oracle.c1_inputs(seed=0)
    plan = _plan(pkg, c1["keep"], c1["src"], c1["parent"], c1["weights"], c1["N"], dev=dev)
    np.testing.assert_allclose(to_np(plan.normalizer[0, :, 0]), golden["c1_normalizer"], rtol=1e-6)
    merged = torch.from_numpy(golden["c1_attention"][0][: c1["M"]]).to(dev)
    np.testing.assert_allclose(to_np(plan.restore(merged[None])[0]), golden["c1_restore_cols"], rtol=1e-6, atol=1e-7)
    keep, src, parent, w = oracle.zipf_plan(5, 8192, 512)
    plan5 = _plan(pkg, keep, src, parent, w, 8192, dev=dev)
    np.testing.assert_allclose(to_np(plan5.normalizer[0, :, 0]), golden["c5_normalizer"], rtol=1e-6)
    g = torch.Generator().manual_seed(55)
    x = torch.randn(1, 8192, 16, generator=g).to(dev)
    y = torch.randn(1, 512, 16, generator=g).to(dev)
    np.testing.assert_allclose(to_np(plan5.compact(x)), golden["c5_compact"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_np(plan5.restore(y)), golden["c5_restore"], rtol=1e-6, atol=1e-6)
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("C", [64, 1024, 3072])
def test_random_plans(pkg, oracle, cuda_device, dtype, C):
    rng = np.random.default_rng(C)
    N, M = 900, 230
    keep, src, parent, w = oracle.random_plan(rng, N, M)
    plan = _plan(pkg, keep, src, parent, w, N, dev=cuda_device)
    x = oracle.round_to(rng.standard_normal((N, C)).astype(np.float32), dtype)
    xt = torch.from_numpy(x).to(cuda_device, TORCH_DTYPE[dtype])[None]
    norm = oracle.normalizer(parent, w, M)
    ref_c = oracle.compact(x, keep, src, parent, w, norm, dtype=dtype)
    got_c = to_np(plan.compact(xt)[0])
    assert_close(got_c, ref_c, dtype, tol=1e-5 if dtype == "f32" else 8e-3)
    y = oracle.round_to(rng.standard_normal((M, C)).astype(np.float32), dtype)
    yt = torch.from_numpy(y).to(cuda_device, TORCH_DTYPE[dtype])[None]
    ref_r = oracle.restore(y, keep, src, parent, w, N, dtype=dtype)
    got_r = to_np(plan.restore(yt)[0])
    if dtype == "f32":
        np.testing.assert_allclose(got_r, ref_r, rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(got_r, ref_r)
    # deterministic: a second compaction is bitwise identical
    assert torch.equal(plan.compact(xt), plan.compact(xt))
    assert pkg.device_error_flags() == 0


def test_zipf_skewed_segments(pkg, oracle, cuda_device):
    """Config-5 distributions at reduced size: Zipf(1.1) parents (a few very long segments),
    Dirichlet(1,1,1,1) weights."""
    N, M, C = 16384, 1024, 256
    keep, src, parent, w = oracle.zipf_plan(5, N, M)
    plan = _plan(pkg, keep, src, parent, w, N, dev=cuda_device)
    norm = oracle.normalizer(parent, w, M)
    np.testing.assert_allclose(to_np(plan.normalizer[0, :, 0]), norm, rtol=2e-6)
    assert abs(float(plan.normalizer.sum()) - N) < 0.05 * 1  # masses sum to N (weights sum to 1)
    rng = np.random.default_rng(1)
    x = oracle.round_bf16(rng.standard_normal((N, C)).astype(np.float32))
    ref = oracle.compact(x, keep, src, parent, w, norm, dtype="bf16")
    got = to_np(plan.compact(torch.from_numpy(x).to(cuda_device, torch.bfloat16)[None])[0])
    assert_close(got, ref, "bf16", tol=8e-3)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_scatter_long_rows_chunked(pkg, oracle, cuda_device, dtype):
    """Every merged row owns thousands of entries (16 rows for 20,000 tokens), so the scatter
    splits rows into 128-entry chunks whose fp32 sums are added in chunk order.  Matches the
    oracle's sequential sum within the parity tolerance and is bit-repeatable."""
    N, M, C = 20000, 16, 96
    rng = np.random.default_rng(2)
    keep, src, parent, w = oracle.random_plan(rng, N, M)
    plan = _plan(pkg, keep, src, parent, w, N, dev=cuda_device)
    norm = oracle.normalizer(parent, w, M)
    x = rng.standard_normal((N, C)).astype(np.float32)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    if dtype == "bf16":
        x = oracle.round_bf16(x)
    xt = torch.from_numpy(x).to(cuda_device, tdt)[None]
    ref = oracle.compact(x, keep, src, parent, w, norm, dtype=dtype)
    got = plan.compact(xt)
    assert_close(to_np(got[0]), ref, dtype)
    assert torch.equal(got, plan.compact(xt))
    assert pkg.device_error_flags() == 0


def test_empty_sources_and_partial_cover(pkg, cuda_device):
    dev = cuda_device
    N, K, C = 50, 50, 64
    keep = torch.arange(K, device=dev)[None]
    empty = torch.zeros(1, 0, dtype=torch.long, device=dev)
    plan = pkg.WeightedBilinearTokenPlan(
        keep=keep, source_original=empty, source_parent_compact=torch.zeros(1, 0, 4, dtype=torch.long, device=dev),
        source_pool_weights=torch.zeros(1, 0, 4, device=dev), source_restore_weights=torch.zeros(1, 0, 4, device=dev),
        original_tokens=N, normalizer=torch.ones(1, K, 1, device=dev))
    x = torch.randn(1, N, C, device=dev, dtype=torch.bfloat16)
    assert torch.equal(plan.compact(x), x)
    assert torch.equal(plan.restore(x), x)
    # keep covering only part of the tokens: uncovered rows are zero (new_zeros semantics)
    plan2 = pkg.WeightedBilinearTokenPlan(
        keep=keep[:, :20], source_original=empty, source_parent_compact=torch.zeros(1, 0, 4, dtype=torch.long, device=dev),
        source_pool_weights=torch.zeros(1, 0, 4, device=dev), source_restore_weights=torch.zeros(1, 0, 4, device=dev),
        original_tokens=N, normalizer=torch.ones(1, 20, 1, device=dev))
    r = plan2.restore(x[:, :20])
    assert torch.equal(r[:, :20], x[:, :20]) and torch.count_nonzero(r[:, 20:]) == 0


def test_token_plan_golden(pkg, golden, cuda_device):
    dev = cuda_device
    keep = torch.from_numpy(golden["fast_keep"]).to(dev)[None]
    inverse = torch.from_numpy(golden["fast_inverse"]).to(dev)[None]
    plan = pkg.TokenPlan(keep, inverse, inverse.shape[1])
    value = torch.from_numpy(golden["fast_value"]).to(dev)
    comp = plan.compact(value)
    np.testing.assert_allclose(to_np(comp), golden["fast_compact"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(to_np(plan.restore(comp)), golden["fast_restore"])
    assert torch.equal(plan.compact(value), comp)  # deterministic, unlike scatter_add_
    np.testing.assert_array_equal(to_np(plan.compact(value, merge=False)), golden["fast_value"][:, golden["fast_keep"]])


def test_row_ops(pkg, oracle, cuda_device):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((300, 1024)).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda_device)
    rows = torch.from_numpy(rng.permutation(300)[:120]).to(cuda_device)
    nb = pkg.row_normalize_bf16(xt, rows)
    ref = x[to_np(rows).astype(int)]
    ref = oracle.round_bf16(ref / np.maximum(np.linalg.norm(ref.astype(np.float64), axis=1, keepdims=True), 1e-12))
    # within one bf16 ulp (the fp32 norm may differ in its last bit), almost always exact
    np.testing.assert_allclose(to_np(nb), ref, rtol=2 ** -7, atol=0)
    assert np.mean(to_np(nb) == ref) > 0.999
    g = pkg.row_gather(xt.bfloat16(), rows)
    assert torch.equal(g, xt.bfloat16()[rows])


@pytest.mark.parametrize("dtype,C", [("bf16", 1024), ("bf16", 256), ("f16", 256), ("f32", 256)])
def test_hot_row_gather_matches_plain(pkg, oracle, cuda_device, dtype, C, monkeypatch):
    """Zipf(1.1)-skewed plan: the gather that stages the most-referenced merged rows in shared
    memory (vb200_proj_gather_hot) gives the plain gather's output bit for bit (and, for 16-bit
    types, the oracle's value-dtype restore exactly); the staged rows are exactly the rows with
    the most references; plan.restore takes this path above HOT_GATHER_MIN_REFERENCES."""
    from importlib import import_module
    tp = import_module("4d_ttt_merging_b200.token_plan")
    N, M = 16384, 1024
    keep, src, parent, w = oracle.zipf_plan(7, N, M)
    plan = _plan(pkg, keep, src, parent, w, N, dev=cuda_device)
    lib = pkg.load_library()
    cap = lib.vb200_proj_gather_hot_capacity(pkg._clib.dtype_code(TORCH_DTYPE[dtype]), C)
    assert cap >= 64
    hot_rows, hot_slot, n_hot, max_hot = pkg.ops.plan_hot_rows(plan.csr, cap)
    n = int(n_hot)
    assert 0 < n <= max_hot
    counts = np.bincount(parent.ravel(), minlength=M)
    slots = hot_slot.cpu().numpy()
    staged = np.sort(hot_rows[:n].cpu().numpy())
    np.testing.assert_array_equal(staged, np.nonzero(slots >= 0)[0])
    np.testing.assert_array_equal(slots[staged][np.argsort(slots[staged])], np.arange(n))
    assert counts[slots >= 0].min() > counts[slots < 0].max()  # the most-referenced rows
    rng = np.random.default_rng(3)
    y = oracle.round_to(rng.standard_normal((M, C)).astype(np.float32), dtype)
    yt = torch.from_numpy(y).to(cuda_device, TORCH_DTYPE[dtype])
    args = (yt, plan._keep_flat, plan.source_original.reshape(-1), plan.source_parent_compact[0].contiguous(),
            plan.source_restore_weights[0].contiguous(), N, False)
    plain = tp._gather(*args)
    hot = tp._gather(*args, hot=(hot_rows, hot_slot, n_hot, max_hot))
    torch.cuda.synchronize()
    assert torch.equal(hot, plain)
    ref = oracle.restore(y, keep, src, parent, w, N, dtype=dtype)
    if dtype == "f32":
        np.testing.assert_allclose(to_np(hot), ref, rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(to_np(hot), ref)
    monkeypatch.setattr(tp, "HOT_GATHER_MIN_REFERENCES", 1)
    assert torch.equal(plan.restore(yt[None])[0], plain)
    assert plan._hot is not None
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("sizes", [[(3087, 1029)] * 3, [(500, 40), (0, 7), (1200, 300), (37, 5)], [(60, 20)] * 40,
                                   [(3601, 515)]],
                         ids=["frame_groups", "ragged", "many_groups", "one_group"])
def test_grouped_csr_equals_general(pkg, cuda_device, sizes):
    """vb200_plan_csr_build_grouped (up to eight CTAs per group, each owning a range of the
    group's merged rows) against the general radix-sort build:
    identical segment offsets, entries, masses and log-masses, for frame-group shapes and for
    ragged groups (one without sources, skewed parents giving long segments)."""
    rng = np.random.default_rng(len(sizes))
    parents, weights, qb, bb = [], [], [0], [0]
    for S_g, K_g in sizes:
        if S_g:
            pr = np.stack([rng.choice(K_g, 4, replace=False) for _ in range(S_g)])
            if K_g > 100:  # skew: a third of the sources share two popular parents
                pr[: S_g // 3, :2] = [0, 1]
            parents.append(pr + bb[-1])
            weights.append(rng.dirichlet(np.ones(4), size=S_g).astype(np.float32))
        qb.append(qb[-1] + S_g)
        bb.append(bb[-1] + K_g)
    parent = torch.as_tensor(np.concatenate(parents), device=cuda_device)
    w = torch.as_tensor(np.concatenate(weights), device=cuda_device)
    S, M = qb[-1], bb[-1]
    src_rows = torch.as_tensor(np.sort(rng.choice(4 * S, S, replace=False)), device=cuda_device)
    ref = pkg.build_plan_csr(parent, w, M, src_rows=src_rows)
    groups = (torch.as_tensor(qb, device=cuda_device), torch.as_tensor(bb, device=cuda_device),
              max(k for _, k in sizes), max(q for q, _ in sizes))
    got = pkg.build_plan_csr(parent, w, M, src_rows=src_rows, groups=groups)
    torch.cuda.synchronize()
    for name in ("seg_offsets", "entry_src", "entry_w", "mass", "log_mass"):
        assert torch.equal(getattr(got, name), getattr(ref, name)), name
    assert pkg.device_error_flags() == 0
