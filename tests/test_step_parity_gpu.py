"""The benchmarked step against the oracle at config-2 shapes.

``ShardedGlobalBlock.step`` (one rank) is what bench.py times: the uniform four-support convex
plan (row normalisation, tcgen05 top-4 retrieval inside the frame group, the fused Gram +
projected-gradient fit of vb200_support_fit, the plan CSR and masses), the qkv GEMM, the fused
q/k LayerNorm + Q||K||V compaction, mass-bias attention, the proj GEMM and the top-4 restore.
Here it runs on one 4-frame group of config 2 (4 x 1029 tokens, dim 1024, 16 heads, bf16,
merge 4x to 1029 keys; 3087 sources) and each stage is checked against the oracle
(oracle/pipeline.py, oracle/ref.py):

  (i)   the keep / source layout equals the oracle's;
  (ii)  the features are F.normalize(x).bf16 within one bf16 ulp (fp32 norm order);
  (iii) the parents are the stable top-4 of the group's bf16 scores, bit-exact up to exact
        ties (helpers.check_topk_contract);
  (iv)  the pool weights are the reference's 32-step projected gradient on the fp32 Gram of
        the chosen supports (sparse_convex.py:2308-2321), to 1e-4;
  (v)   the masses are deterministic_weighted_normalizer of those parents and weights;
  (vi)  the restored block output matches the oracle's block on the same plan (bf16 bar:
        max rel err <= 2e-2, cosine > 0.999), and the oracle's whole step (its own plan) too.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import admissible_bf16, assert_close, check_topk_contract, to_np

pytestmark = pytest.mark.gpu

FRAMES, TPF, SPECIAL, DIM, HEADS, MERGE, GROUP = 4, 1029, 5, 1024, 16, 4, 4


def _bf16_ulps(a, b):
    ia = np.asarray(a, np.float32).view(np.int32) >> 16
    ib = np.asarray(b, np.float32).view(np.int32) >> 16
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


@pytest.fixture(scope="module")
def case(pkg, cuda_device):
    dev = cuda_device
    torch.manual_seed(0)
    attn = pkg.GlobalAttention(DIM, HEADS, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in attn.parameters():
            p.normal_(0.0, 0.02)  # the bench's random init
        attn.q_norm.weight.fill_(1.0)
        attn.k_norm.weight.fill_(1.0)
    block = pkg.parallel.ShardedGlobalBlock(attn, frames=FRAMES, tokens_per_frame=TPF, patch_token_start=SPECIAL,
                                            merge_factor=MERGE, group_frames=GROUP)
    gen = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(1, FRAMES * TPF, DIM, generator=gen).to(dev, torch.bfloat16)
    plan = block.plan(x)
    out = block.step(x)
    lay = pkg.planners.uniform_keep_layout(FRAMES, TPF, SPECIAL, MERGE, GROUP)
    rows = torch.cat([lay["source"], lay["keep"]]).to(dev)
    feat = pkg.row_normalize_bf16(x[0], rows)  # the planner's feature rows: [sources; keeps]
    torch.cuda.synchronize()
    params = {k: to_np(v) for k, v in attn.state_dict().items()}
    params["qkv.bias_mask"] = params.pop("bias_mask")
    return dict(x=to_np(x[0]), plan=plan, out=to_np(out[0]), feat=feat, lay=lay, params=params)


def test_layout(case, oracle):
    keep, src, qb, bb = oracle.pipeline.uniform_layout(FRAMES, TPF, SPECIAL, MERGE, GROUP)
    plan = case["plan"]
    np.testing.assert_array_equal(plan.keep[0].cpu().numpy(), keep)
    np.testing.assert_array_equal(plan.source_original[0].cpu().numpy(), src)
    assert plan.kept_tokens == FRAMES * TPF // MERGE


def test_features(case, oracle):
    lay = case["lay"]
    ref = oracle.normalize_bf16(case["x"][np.concatenate([lay["source"].numpy(), lay["keep"].numpy()])])
    ulps = _bf16_ulps(to_np(case["feat"]), ref)
    assert ulps.max() <= 1 and np.mean(ulps > 0) < 1e-3, (ulps.max(), np.mean(ulps > 0))


def test_parents_are_top4_up_to_ties(pkg, case, oracle):
    plan, feat = case["plan"], case["feat"]
    S = plan.source_original.shape[1]
    v, i = pkg.similarity_topk(feat[:S], feat[S:], 4, query_begin=case["lay"]["q_begin"],
                               basis_begin=case["lay"]["b_begin"])
    parent = plan.source_parent_compact[0]
    assert torch.equal(i, parent)  # the plan's parents are that kernel's picks
    f = to_np(feat)
    _, lo, hi = admissible_bf16(f[:S], f[S:])
    amb = check_topk_contract(lo, hi, to_np(v), i.cpu().numpy())
    # and the exact-score ranking agrees on all but the candidate-tie rows
    _, ref = oracle.similarity_topk(f[:S], f[S:], 4)
    differ = np.any(i.cpu().numpy() != ref, axis=1).sum()
    assert differ <= amb, (differ, amb)


def test_weights_and_masses(case, oracle):
    plan, f = case["plan"], to_np(case["feat"]).astype(np.float64)
    S = plan.source_original.shape[1]
    parent = plan.source_parent_compact[0].cpu().numpy()
    sup = f[S:][parent]                                             # [S, 4, D]
    gram = np.einsum("sid,sjd->sij", sup, sup).astype(np.float32)
    rhs = np.einsum("sid,sd->si", sup, f[:S]).astype(np.float32)
    w_ref = oracle.projected_gradient(gram, rhs, 32)
    w = to_np(plan.source_pool_weights[0])
    np.testing.assert_allclose(w, w_ref, rtol=1e-4, atol=1e-4)
    assert np.all(w >= 0) and np.allclose(w.sum(axis=1), 1.0, atol=1e-5)
    assert torch.equal(plan.source_pool_weights, plan.source_restore_weights)
    mass = to_np(plan.normalizer[0, :, 0])
    np.testing.assert_allclose(mass, oracle.normalizer(parent, w, plan.kept_tokens), rtol=2e-6)
    np.testing.assert_allclose(to_np(plan.key_log_mass[0]), np.log(mass), rtol=1e-6, atol=1e-7)


def test_block_output(case, oracle):
    plan = case["plan"]
    pd = dict(keep=plan.keep[0].cpu().numpy(), source=plan.source_original[0].cpu().numpy(),
              parent=plan.source_parent_compact[0].cpu().numpy(), weights=to_np(plan.source_pool_weights[0]),
              normalizer=to_np(plan.normalizer[0, :, 0]), special=np.zeros(0, np.int64),
              special_compact=np.zeros(0, np.int64))
    ref = oracle.global_attention_forward(case["x"], case["params"], pd, heads=HEADS, preserve_queries=False,
                                          dense_special=False)
    assert_close(case["out"], ref, "bf16")
    # the oracle's whole step: its own plan (exact-score top-4, float64 Gram) and block
    lay = oracle.pipeline.uniform_layout(FRAMES, TPF, SPECIAL, MERGE, GROUP)
    ref_step = oracle.pipeline.block_step(case["x"], case["params"], lay, heads=HEADS)
    assert_close(case["out"], ref_step, "bf16")


def test_support_fit_direct(pkg, case, oracle, cuda_device):
    """vb200_support_fit on its own at the config-2 group size (3087 sources x 1029 basis rows,
    D = 1024): the Gram and rhs against float64 products within the fp32 summation bound, the
    weights against the oracle's solve of those Gram / rhs and of the exact ones."""
    plan, feat = case["plan"], case["feat"]
    S = plan.source_original.shape[1]
    parent_rows = (plan.source_parent_compact[0] + S).contiguous()
    gram = torch.empty((S, 4, 4), device=cuda_device, dtype=torch.float32)
    rhs = torch.empty((S, 4), device=cuda_device, dtype=torch.float32)
    alpha = torch.empty((S, 4), device=cuda_device, dtype=torch.float32)
    C = pkg._clib
    rc = C.lib().vb200_support_fit(C.BF16, feat.data_ptr(), feat.shape[0], feat.stride(0), None,
                                   parent_rows.data_ptr(), S, feat.shape[1], gram.data_ptr(), rhs.data_ptr(),
                                   alpha.data_ptr(), 32, C.stream_of(cuda_device))
    C.check(rc, "support_fit")
    torch.cuda.synchronize()
    f = to_np(feat).astype(np.float64)
    sup = f[parent_rows.cpu().numpy()]
    g64 = np.einsum("sid,sjd->sij", sup, sup)
    r64 = np.einsum("sid,sd->si", sup, f[:S])
    D = f.shape[1]
    gbound = np.einsum("sid,sjd->sij", np.abs(sup), np.abs(sup)) * D * 2.0 ** -24 + 1e-7
    rbound = np.einsum("sid,sd->si", np.abs(sup), np.abs(f[:S])) * D * 2.0 ** -24 + 1e-7
    g, r, a = to_np(gram), to_np(rhs), to_np(alpha)
    assert np.all(np.abs(g - g64) <= gbound) and np.all(np.abs(r - r64) <= rbound)
    np.testing.assert_array_equal(g, np.swapaxes(g, 1, 2))
    np.testing.assert_allclose(a, oracle.projected_gradient(g, r, 32), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(a, oracle.projected_gradient(g64.astype(np.float32), r64.astype(np.float32), 32),
                               rtol=1e-4, atol=1e-4)
    # the plan's weights are this kernel's
    np.testing.assert_array_equal(a, to_np(plan.source_pool_weights[0]))
    assert pkg.device_error_flags() == 0
