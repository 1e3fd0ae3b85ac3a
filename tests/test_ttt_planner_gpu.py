"""The released planner (build_ttt_protected_uniform_convex_plan) on the GPU against the oracle
restatement (oracle/ttt_planner.py, pinned to the reference's own output by the golden tests) and
the reference goldens.

Index decisions here rest on bf16 scores, fp32 certificates and fp32 pruning scores computed in
a different order than the oracle's float64, so a decision whose quantity lies within rounding
distance of its boundary (a bf16 rounding boundary, the certificate threshold, the 0.95 pruning
threshold) may go either way.  The tests therefore check: the skeleton and the event proposals
exactly; the keep set and sources up to a handful of such boundary cases; parents identical on
nearly every source, with the oracle's weights on the shared supports; the device certificate
against the oracle's on the device's own supports; masses consistent with the plan."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import to_np

pytestmark = pytest.mark.gpu


def _structured(seed, frames, hw, pts, dim, noise):
    """Tokens whose patches repeat across frames with noise, a region that changes content in
    later frames, TTT labels marking it (plus a few random), random sensitivity and geometry."""
    rng = np.random.default_rng(seed)
    patches = hw[0] * hw[1]
    tpf = pts + patches
    base = rng.standard_normal((patches, dim))
    tok = rng.standard_normal((frames, tpf, dim))
    tok[:, pts:] = base[None] + noise * rng.standard_normal((frames, patches, dim))
    moving = np.zeros((frames, patches), bool)
    moving[frames // 2:, patches // 6: patches // 6 + patches // 3] = True
    tok[:, pts:][moving] = rng.standard_normal((int(moving.sum()), dim))
    labels = (moving | (rng.random((frames, patches)) < 0.05)).astype(np.int64).ravel()
    labels[:patches] = 0
    return (tok.reshape(frames * tpf, dim).astype(np.float32), labels,
            rng.random(frames * patches).astype(np.float32),
            rng.standard_normal((frames * patches, 4)).astype(np.float32))


def _run(pkg, oracle, dev, tokens, labels, sens, geo, frames, hw, pts, prune, ratio, support_w=0.0):
    tpf = pts + hw[0] * hw[1]
    kw = dict(frames=frames, tokens_per_frame=tpf, patch_token_start=pts, patch_hw=hw, threshold=0.9,
              top1_prune_threshold=prune, sensitive_event_ratio=ratio)
    if support_w:
        kw.update(support_geometry_weight=support_w, support_geometry_guard_tolerance=0.0)
    plan = pkg.build_ttt_protected_uniform_convex_plan(
        torch.from_numpy(tokens)[None].to(dev), labels=torch.from_numpy(labels), sensitivity=torch.from_numpy(sens),
        geometry=torch.from_numpy(geo), **kw)
    ref = oracle.ttt_planner.build_plan(tokens, labels=labels, sensitivity=sens, geometry=geo, **kw)
    return plan, ref


def _compare(pkg, oracle, plan, ref, patches, tpf, pts, max_boundary):
    md = plan.metadata
    assert md["protected_uniform_bases"] == len(ref["stable_basis"])
    assert md["sensitive_event_proposals"] == len(ref["event_proposal"])
    assert abs(md["sensitive_event_bases"] - len(ref["event"])) <= max_boundary
    keep, src = plan.keep[0].cpu().numpy(), plan.source_original[0].cpu().numpy()
    assert len(np.setxor1d(keep, ref["keep"])) <= 2 * max_boundary
    assert len(np.setxor1d(src, ref["source"])) <= 2 * max_boundary
    parent = plan.source_parent_compact[0].cpu().numpy()
    w = to_np(plan.source_pool_weights[0])
    assert np.all(w >= 0) and np.allclose(w.sum(1), 1.0, atol=1e-5)
    # the device certificate and weights against the oracle's solve on the device's own supports
    patch = lambda tok: (tok // tpf) * patches + tok % tpf - pts
    feats = ref["features"]
    fw, fcos, fres, fnrm = oracle.ttt_planner.fit_supports(feats, patch(src), patch(keep[parent]))
    np.testing.assert_allclose(w, fw, rtol=1e-4, atol=1e-4)
    assert np.all(fcos >= 0.9 - 1e-4) and np.all(fres <= (2 * 0.1) ** 0.5 + 1e-4) and np.all(fnrm >= 0.8 - 1e-4)
    # the same sources mostly got the oracle's parents (compare by original token ids)
    common, ia, ib = np.intersect1d(src, ref["source"], return_indices=True)
    same = np.all(keep[parent[ia]] == ref["keep"][ref["parent"][ib]], axis=1)
    assert same.mean() > 0.9, same.mean()
    np.testing.assert_allclose(w[ia][same], ref["weights"][ib][same], rtol=1e-4, atol=1e-4)
    mass = to_np(plan.normalizer[0, :, 0])
    np.testing.assert_allclose(mass, oracle.normalizer(parent, w, len(keep)), rtol=1e-6)
    np.testing.assert_allclose(to_np(plan.key_log_mass[0]), np.log(mass), rtol=1e-6, atol=1e-7)
    special = (np.arange(plan.original_tokens // tpf)[:, None] * tpf + np.arange(pts)[None]).ravel()
    np.testing.assert_array_equal(plan.special_query_original.cpu().numpy(), special)
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("tag,prune,ratio,support_w", [("ttt_prune", 0.95, 0.02, 0.0), ("ttt_noprune", 2.0, 0.05, 0.0),
                                                       ("ttt_geo", 2.0, 0.01, 0.01)])
def test_golden_inputs(pkg, oracle, golden, cuda_device, tag, prune, ratio, support_w):
    """The reference's golden inputs (10 frames of 8 x 8 patches, D = 64): the device plan against
    the oracle, and its keep set against the reference's.  ttt_geo: the released configuration's
    geometry-guarded support route (weight 0.01, tolerance 0)."""
    g = lambda k: golden[f"{tag}_{k}"]
    plan, ref = _run(pkg, oracle, cuda_device, g("tokens"), g("labels"), g("sensitivity"), g("geometry"), 10, (8, 8),
                     5, prune, ratio, support_w)
    _compare(pkg, oracle, plan, ref, 64, 69, 5, max_boundary=2)
    assert len(np.setxor1d(plan.keep[0].cpu().numpy(), g("keep"))) <= 4
    if support_w:
        md = plan.metadata
        assert md["geometry_guard_enabled"]
        assert abs(md["geometry_guard_selected"] - ref["guard_selected"]) <= max(3, 0.05 * ref["guard_selected"])


@pytest.mark.parametrize("prune,ratio,support_w", [(0.95, 0.02, 0.0), (2.0, 0.01, 0.0), (2.0, 0.01, 0.01)])
def test_structured_clip(pkg, oracle, cuda_device, prune, ratio, support_w):
    """12 frames of 16 x 16 patches, D = 256 (two temporal-local frame groups, events, global
    fallbacks), feature route and geometry-guarded route; the plan then drives compact / restore
    without device errors."""
    frames, hw, pts, dim = 12, (16, 16), 5, 256
    tokens, labels, sens, geo = _structured(11, frames, hw, pts, dim, 0.2 if prune <= 1 else 0.4)
    plan, ref = _run(pkg, oracle, cuda_device, tokens, labels, sens, geo, frames, hw, pts, prune, ratio, support_w)
    if support_w:
        assert abs(plan.metadata["geometry_guard_selected"] - ref["guard_selected"]) <= max(
            4, 0.05 * ref["guard_selected"])
    _compare(pkg, oracle, plan, ref, 256, 5 + 256, pts, max_boundary=4)
    x = torch.from_numpy(tokens)[None].to(cuda_device, torch.bfloat16)
    y = plan.restore(plan.compact(x))
    assert y.shape == x.shape and bool(torch.isfinite(y.float()).all())
    keep = plan.keep[0]
    assert torch.equal(y[0, keep], plan.compact(x)[0])  # kept rows are restored as they were pooled
    assert pkg.device_error_flags() == 0


def test_rejects_unbuilt_routes(pkg, cuda_device):
    x = torch.zeros(1, 2 * 69, 64, device=cuda_device)
    z = torch.zeros(128)
    with pytest.raises(ValueError, match="joint-metric"):
        pkg.build_ttt_protected_uniform_convex_plan(
            x, frames=2, tokens_per_frame=69, patch_token_start=5, patch_hw=(8, 8), threshold=0.9, labels=z,
            sensitivity=z, geometry=torch.zeros(128, 4), support_geometry_weight=0.01)
    with pytest.raises(ValueError, match="one value per patch"):
        pkg.build_ttt_protected_uniform_convex_plan(
            x, frames=2, tokens_per_frame=69, patch_token_start=5, patch_hw=(8, 8), threshold=0.9, labels=z[:5],
            sensitivity=z, geometry=torch.zeros(128, 4))


def test_guard_kernels_against_oracle(pkg, oracle, cuda_device):
    """vb200_geometry_shortlist and vb200_geometry_guard on their own: random bf16 features and
    4-D geometry, the shortlist of vb200_sim_topk (k = 16), against oracle.ttt_planner's
    geometry_shortlist / guard_choose on the same inputs (ties in the bf16 shortlist may order
    differently: such rows are skipped, and must be few)."""
    dev = cuda_device
    rng = np.random.default_rng(21)
    n, nb, D = 600, 300, 128
    feats = oracle.round_bf16(rng.standard_normal((n + nb, D)).astype(np.float32) / np.sqrt(D) * 3)
    feats = oracle.round_bf16(feats / np.linalg.norm(feats, axis=1, keepdims=True))
    geo = rng.standard_normal((n + nb, 4)).astype(np.float32)
    src, basis = np.arange(n), np.arange(n, n + nb)
    f = torch.from_numpy(feats).to(dev, torch.bfloat16)
    g = torch.from_numpy(geo).to(dev)
    s_t, b_t = torch.from_numpy(src).to(dev), torch.from_numpy(basis).to(dev)
    from importlib import import_module
    planners = import_module("4d_ttt_merging_b200.planners")
    ids, w, cos, res, nrm, chosen = planners._guarded_fit(f, g, s_t, b_t, 0.05, 0.0)
    fids, jids = oracle.ttt_planner.geometry_shortlist(feats, geo, src, basis, 0.05)
    o = oracle.ttt_planner.guard_choose(feats, geo, src, fids, jids, 0.0)
    ids, chosen = ids.cpu().numpy(), chosen.cpu().numpy().astype(bool)
    same = np.all(ids == o[0], axis=1)
    assert same.mean() > 0.97, same.mean()
    assert 0.02 < o[5].mean() < 0.98 and abs(chosen.mean() - o[5].mean()) < 0.02  # both branches taken
    np.testing.assert_allclose(w.cpu().numpy()[same], o[1][same], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(cos.cpu().numpy()[same], o[2][same], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(res.cpu().numpy()[same], o[3][same], rtol=1e-4, atol=1e-5)
    assert pkg.device_error_flags() == 0
