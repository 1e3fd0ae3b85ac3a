"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Runs the reference's own PyTorch code (shuang-yang18/4D_TTT_merging, imported read-only from
the checkout named by --reference or REFERENCE_ROOT) on CPU with seeded inputs and stores inputs and
outputs in ``tests/golden/golden.npz``.  It is run once in the build container; the GPU box
never needs the reference.  Cases:

  block_compact_q / block_preserve_q
      SelfAttention.forward(x, token_plan=WeightedBilinearTokenPlan) — the global-attention
      call site (vggt_omega/models/layers/attention.py:264-439): qkv, q/k LayerNorm, compact,
      SDPA with the log-mass bias (the non-Triton branch, :400), dense special queries
      (:406-423), proj, restore.  Compact-query and query-preserving plans.
  plan_*     WeightedBilinearTokenPlan.compact / restore in fp32 and bf16 and
             deterministic_weighted_normalizer (vggt_omega/models/token_merging.py:40-59, 253-426).
  fast_*     build_fastvggt_plan + TokenPlan.compact / restore (token_merging.py:143-196, 1045-1122).
  topk_*     (q.bf16 @ basis.bf16).topk(4) and .max(-1) (vggt_omega/models/sparse_convex.py:264).
  pg_*       _adaptive_fit in "adaptive_convex" mode (sparse_convex.py:128-160): top-4 supports
             and 32 projected-gradient steps.
  as_*       _convex_fit (sparse_convex.py:2260-2305): exact 15-active-set solve.
  rand_*     torch.rand with a seeded CPU generator (the anchor draw of the planners).

Usage: python tests/golden/make_golden.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent / "golden.npz"


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


def make_plan(WeightedBilinearTokenPlan, deterministic_weighted_normalizer, gen, N, K, frames,
              special_per_frame, preserve_queries):
    tokens_per_frame = N // frames
    special = torch.cat([torch.arange(f * tokens_per_frame, f * tokens_per_frame + special_per_frame)
                         for f in range(frames)])
    others = torch.tensor([i for i in range(N) if i not in set(special.tolist())])
    perm = others[torch.randperm(others.numel(), generator=gen)]
    keep = torch.sort(torch.cat([special, perm[: K - special.numel()]])).values
    mask = torch.ones(N, dtype=torch.bool)
    mask[keep] = False
    source = torch.nonzero(mask).flatten()
    S = source.numel()
    parent = torch.stack([torch.randperm(K, generator=gen)[:4] for _ in range(S)])
    w = torch.softmax(torch.randn(S, 4, generator=gen), dim=-1)
    norm = deterministic_weighted_normalizer(parent[None], w[None], K)
    original_to_compact = torch.full((N,), -1, dtype=torch.long)
    original_to_compact[keep] = torch.arange(K)
    plan = WeightedBilinearTokenPlan(
        keep=keep[None], source_original=source[None], source_parent_compact=parent[None],
        source_pool_weights=w[None], source_restore_weights=w[None], original_tokens=N,
        normalizer=norm, preserve_queries=preserve_queries,
        preserve_destination_keys=preserve_queries, dense_special_queries=True,
        special_query_original=special, special_query_compact=original_to_compact[special],
        key_log_mass=norm[..., 0].log(),
    )
    return plan, dict(keep=keep, source=source, parent=parent, weights=w, normalizer=norm[0, :, 0],
                      special=special, special_compact=original_to_compact[special])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"),
                    help="reference checkout (default: $REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or REFERENCE_ROOT")
    sys.path.insert(0, args.reference)
    from vggt_omega.models.layers.attention import SelfAttention
    from vggt_omega.models.sparse_convex import _adaptive_fit, _convex_fit
    from vggt_omega.models.token_merging import (TokenPlan, WeightedBilinearTokenPlan,
                                                 build_fastvggt_plan,
                                                 deterministic_weighted_normalizer)

    torch.set_num_threads(1)  # fixed reduction order in the CPU kernels
    out: dict[str, np.ndarray] = {}

    # ---------------- block: the global-attention call site ----------------
    for tag, preserve in (("block_compact_q", False), ("block_preserve_q", True)):
        torch.manual_seed(1 if preserve else 0)
        gen = torch.Generator().manual_seed(11 if preserve else 10)
        dim, heads, frames, tpf, special = 128, 2, 2, 56, 5
        N, K = frames * tpf, 40
        attn = SelfAttention(dim, num_heads=heads, qkv_bias=True, proj_bias=True, mask_k_bias=True,
                             use_qk_norm=True).eval()
        with torch.no_grad():
            for p in attn.parameters():
                p.copy_(torch.randn(p.shape, generator=gen) * (0.2 if p.ndim > 1 else 0.5))
        plan, pd = make_plan(WeightedBilinearTokenPlan, deterministic_weighted_normalizer, gen, N, K,
                             frames, special, preserve)
        x = torch.randn(1, N, dim, generator=gen)
        with torch.no_grad():
            y = attn(x, token_plan=plan)
        out[f"{tag}_x"] = _np(x)
        out[f"{tag}_y"] = _np(y)
        for name, p in attn.named_parameters():
            out[f"{tag}_p_{name}"] = _np(p)
        out[f"{tag}_p_qkv.bias_mask"] = _np(attn.qkv.bias_mask)
        for k_, v_ in pd.items():
            out[f"{tag}_{k_}"] = _np(v_)

    # ---------------- plan ops ----------------
    gen = torch.Generator().manual_seed(20)
    N, K, Cc = 240, 64, 64
    plan, pd = make_plan(WeightedBilinearTokenPlan, deterministic_weighted_normalizer, gen, N, K, 3, 5, False)
    v32 = torch.randn(1, N, Cc, generator=gen)
    y32 = torch.randn(1, K, Cc, generator=gen)
    out["plan_value"] = _np(v32)
    out["plan_compact_f32"] = _np(plan.compact(v32))
    out["plan_compact_bf16"] = _np(plan.compact(v32.bfloat16()))
    out["plan_y"] = _np(y32)
    out["plan_restore_f32"] = _np(plan.restore(y32))
    out["plan_restore_bf16"] = _np(plan.restore(y32.bfloat16()))
    for k_, v_ in pd.items():
        out[f"plan_{k_}"] = _np(v_)

    # ---------------- FastVGGT plan + TokenPlan ----------------
    gen = torch.Generator().manual_seed(30)
    frames, hw, pts = 3, (8, 8), 5
    tpf = pts + hw[0] * hw[1]
    tokens = torch.randn(1, frames * tpf, 64, generator=gen)
    fplan = build_fastvggt_plan(tokens, frames=frames, tokens_per_frame=tpf, patch_token_start=pts,
                                patch_hw=hw, merge_ratio=0.5, protect_ratio=0.1, seed=3)
    value = torch.randn(1, frames * tpf, 32, generator=gen)
    compacted = fplan.compact(value)
    out["fast_tokens"] = _np(tokens)
    out["fast_keep"] = _np(fplan.keep[0])
    out["fast_inverse"] = _np(fplan.inverse[0])
    out["fast_value"] = _np(value)
    out["fast_compact"] = _np(compacted)
    out["fast_restore"] = _np(fplan.restore(compacted))

    # ---------------- bf16 top-4 / argmax ----------------
    gen = torch.Generator().manual_seed(40)
    q = F.normalize(torch.randn(96, 64, generator=gen), dim=-1).bfloat16()
    b = F.normalize(torch.randn(160, 64, generator=gen), dim=-1).bfloat16()
    score = q @ b.T
    tv, ti = score.topk(4, dim=-1)
    mv, mi = score.max(dim=-1)
    out["topk_q"] = _np(q)
    out["topk_b"] = _np(b)
    out["topk_values"] = _np(tv)
    out["topk_indices"] = _np(ti)
    out["topk_max_values"] = _np(mv)
    out["topk_max_indices"] = _np(mi)

    # ---------------- projected gradient (adaptive_convex) ----------------
    gen = torch.Generator().manual_seed(50)
    feats = F.normalize(torch.randn(160, 48, generator=gen), dim=-1)
    basis_ids = torch.randperm(160, generator=gen)[:40]
    fit = _adaptive_fit(feats, basis_ids, max_support=4, mode="adaptive_convex", coefficient_limit=1.0,
                        chunk=1024, steps=32)
    out["pg_features"] = _np(feats)
    out["pg_basis_ids"] = _np(basis_ids)
    for k_ in ("support_ids", "weights", "cosine"):
        if k_ in fit:
            out[f"pg_{k_}"] = _np(fit[k_])

    # ---------------- exact active set ----------------
    gen = torch.Generator().manual_seed(60)
    src = F.normalize(torch.randn(128, 32, generator=gen), dim=-1)
    sup = F.normalize(src[:, None, :] + 0.7 * torch.randn(128, 4, 32, generator=gen), dim=-1)
    cos, alpha = _convex_fit(src, sup)
    out["as_source"] = _np(src)
    out["as_supports"] = _np(sup)
    out["as_alpha"] = _np(alpha)
    out["as_cosine"] = _np(cos)

    # ---------------- released planner: build_ttt_protected_uniform_convex_plan ----------------
    # The Triton projected-gradient kernel cannot run on a CPU; its PyTorch restatement
    # (oracle/torch_path.py, itself checked against _adaptive_fit above) stands in for it.
    import vggt_omega.models.sparse_convex as sc
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from oracle.torch_path import projected_gradient as torch_pg
    sc.four_support_projected_gradient = lambda gram, rhs, *, steps=32: torch_pg(gram.float(), rhs.float(), steps)
    # ttt_geo: the released configuration's support route (geometry weight 0.01, guard
    # tolerance 0, top-1 pruning off, event ratio 0.01) on geometry that follows the content
    cases = (("ttt_prune", 0.95, 0.02, 0.15, 0.0, 70), ("ttt_noprune", 2.0, 0.05, 0.35, 0.0, 71),
             ("ttt_geo", 2.0, 0.01, 0.35, 0.01, 72))
    for tag, prune, ratio, noise, support_w, seed in cases:
        gen = torch.Generator().manual_seed(seed)
        frames, hw, pts, dim = 10, (8, 8), 5, 64
        patches = hw[0] * hw[1]
        tpf = pts + patches
        base = torch.randn(patches, dim, generator=gen)
        tok = torch.randn(frames, tpf, dim, generator=gen)
        tok[:, pts:] = base[None] + noise * torch.randn(frames, patches, dim, generator=gen)
        moving = torch.zeros(frames, patches, dtype=torch.bool)
        moving[5:, 10:30] = True  # a region whose content changes in later frames
        tok[:, pts:][moving] = torch.randn(int(moving.sum()), dim, generator=gen)
        labels = (moving | (torch.rand(frames, patches, generator=gen) < 0.05)).long().flatten()
        labels[:patches] = 0
        sensitivity = torch.rand(frames * patches, generator=gen)
        geometry = torch.randn(frames * patches, 4, generator=gen)
        if support_w:  # per-patch xyz of the base content plus noise, time in the fourth channel
            base_xyz = torch.randn(patches, 3, generator=gen)
            geometry = torch.cat([base_xyz[None].expand(frames, -1, -1) + 0.3 * torch.randn(frames, patches, 3, generator=gen),
                                  torch.linspace(-1, 1, frames)[:, None, None].expand(-1, patches, 1)], -1).reshape(-1, 4)
        tokens = tok.reshape(1, frames * tpf, dim)
        extra = dict(support_geometry_weight=support_w, support_geometry_guard_tolerance=0.0) if support_w else {}
        plan = sc.build_ttt_protected_uniform_convex_plan(
            tokens, frames=frames, tokens_per_frame=tpf, patch_token_start=pts, patch_hw=hw, threshold=0.9,
            labels=labels, sensitivity=sensitivity, geometry=geometry, top1_prune_threshold=prune,
            sensitive_event_ratio=ratio, **extra)
        out[f"{tag}_tokens"] = _np(tokens[0])
        out[f"{tag}_labels"] = _np(labels)
        out[f"{tag}_sensitivity"] = _np(sensitivity)
        out[f"{tag}_geometry"] = _np(geometry)
        out[f"{tag}_keep"] = _np(plan.keep[0])
        out[f"{tag}_source"] = _np(plan.source_original[0])
        out[f"{tag}_parent"] = _np(plan.source_parent_compact[0])
        out[f"{tag}_weights"] = _np(plan.source_pool_weights[0])
        out[f"{tag}_normalizer"] = _np(plan.normalizer[0, :, 0])
        out[f"{tag}_special_compact"] = _np(plan.special_query_compact)
        md = plan.metadata
        out[f"{tag}_counts"] = np.array([md["protected_uniform_bases"], md["top1_pruned_uniform_bases"],
                                         md["sensitive_event_budget"], md["sensitive_event_proposals"],
                                         md["sensitive_event_bases"], md["fit_failure_promotions"],
                                         md["global_fallback_candidates"]], np.int64)
        if support_w:
            out[f"{tag}_guard_selected"] = np.array([md["geometry_guard_selected"]], np.int64)
        print(tag, {k: md[k] for k in ("protected_uniform_bases", "top1_pruned_uniform_bases",
                                       "sensitive_event_budget", "sensitive_event_proposals", "sensitive_event_bases",
                                       "fit_failure_promotions", "global_fallback_candidates", "physical_patch_tokens")})

    # ---------------- TTT pre-pass: correspondences, warp, motion cues, sensitivity ----------------
    import vggt_omega.utils.token_matching as tm
    from vggt_omega.utils.ttt_4d import _flow_grid, _warp
    from vggt_omega.utils.ttt_kernels import normalize_rows as ref_normalize_rows
    gen = torch.Generator().manual_seed(80)
    T, H, W, Cd = 4, 6, 7, 32
    base = torch.randn(H + 6, W + 6, Cd, generator=gen)
    shifts = [(0, 0), (1, 0), (1, -1), (2, 1)]  # per-frame content shift (dy, dx)
    raw = torch.stack([base[3 + dy:3 + dy + H, 3 + dx:3 + dx + W] for dy, dx in shifts])
    raw = raw + 0.3 * torch.randn(T, H, W, Cd, generator=gen)
    desc = ref_normalize_rows(raw)
    fflow, bflow, fconf, bconf, _ = tm.adjacent_token_correspondences(desc, search_radius=2)
    out["ttt_raw"], out["ttt_desc"] = _np(raw), _np(desc)
    out["ttt_forward_flow"], out["ttt_backward_flow"] = _np(fflow), _np(bflow)
    out["ttt_forward_conf"], out["ttt_backward_conf"] = _np(fconf), _np(bconf)
    field = torch.randn(2, 5, 6, 3, generator=gen)
    flow = torch.randint(-3, 4, (2, 5, 6, 2), generator=gen).float()
    grid, _ = _flow_grid(flow)
    out["ttt_field"], out["ttt_flow"], out["ttt_warped"] = _np(field), _np(flow), _np(_warp(field, grid))
    # motion cues and sensitivity through the CPU path of adapt_token_motion_ttt: the adapter's
    # predicted motion is recorded from its eval-mode forward, the residual and boundary maps
    # from the two _robust_unit calls of the sensitivity formula
    seen = {"pred": [], "unit": []}
    fwd = tm.SequenceTokenMotionAdapter.forward

    def record_forward(self, inputs, motion_scale):
        f, b = fwd(self, inputs, motion_scale)
        if not self.training:
            seen["pred"].append(torch.cat((f, b), -1).detach().clone())
        return f, b

    unit = tm._robust_unit

    def record_unit(value, mask):
        seen["unit"].append(value.detach().clone())
        return unit(value, mask)

    tm.SequenceTokenMotionAdapter.forward, tm._robust_unit = record_forward, record_unit
    try:
        anchors = torch.randn(2, H, W, 3, generator=gen)
        _, labels, sens, md = tm.adapt_token_motion_ttt(anchors, (0, T - 1), desc, fflow, bflow, fconf, bconf,
                                                        steps=4, uncertain_confidence=0.10)
    finally:
        tm.SequenceTokenMotionAdapter.forward, tm._robust_unit = fwd, unit
    out["ttt_predicted"] = _np(torch.cat(seen["pred"]).reshape(T, H, W, 4))
    out["ttt_residual"], out["ttt_boundary"] = _np(seen["unit"][0]), _np(seen["unit"][1])
    out["ttt_sensitivity"], out["ttt_labels"] = _np(sens), _np(labels)
    out["ttt_cue_stats"] = np.array([md["motion_residual_threshold"], md["motion_boundary_threshold"],
                                     md["confidence_mean"], md["motion_residual_mean"], md["motion_boundary_mean"]],
                                    np.float64)

    # ---------------- config 1 at its full size, and config 5 scaled down ----------------
    # Inputs from the oracle's seeded numpy generators (oracle/synth.py); outputs from the
    # reference's own CPU path: the SDPA call with the log-mass mask of layers/attention.py:386-400
    # and WeightedBilinearTokenPlan.compact / restore.  To keep the fixture small only some heads
    # and channels of the large outputs are stored (they are exact slices of the full results).
    from oracle import synth
    c1 = synth.c1_inputs(seed=0)
    q, k, v = (torch.from_numpy(c1[n]) for n in ("q", "k", "v"))
    log_m = torch.from_numpy(c1["log_mass"])
    att = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=log_m[None, None, None, :])
    out["c1_heads"] = np.array([5], np.int64)
    out["c1_attention"] = _np(att[0, out["c1_heads"]])
    N1, M1 = c1["N"], c1["M"]
    parent1 = torch.from_numpy(c1["parent"])[None]
    w1 = torch.from_numpy(c1["weights"])[None]
    norm1 = deterministic_weighted_normalizer(parent1, w1, M1)
    plan1 = WeightedBilinearTokenPlan(
        keep=torch.from_numpy(c1["keep"])[None], source_original=torch.from_numpy(c1["src"])[None],
        source_parent_compact=parent1, source_pool_weights=w1, source_restore_weights=w1, original_tokens=N1,
        normalizer=norm1, key_log_mass=norm1[..., 0].log())
    merged = att[0].transpose(0, 1)[:M1].reshape(1, M1, -1)  # [1, M, 16 x 64]: the first M query rows
    restored = plan1.restore(merged)
    out["c1_restore_cols"] = _np(restored[0, :, 320:384])  # head 5's 64 channels
    out["c1_normalizer"] = _np(norm1[0, :, 0])
    N5, M5, D5 = 8192, 512, 16
    keep5, src5, parent5, w5 = synth.zipf_plan(5, N5, M5)
    p5, ww5 = torch.from_numpy(parent5)[None], torch.from_numpy(w5)[None]
    norm5 = deterministic_weighted_normalizer(p5, ww5, M5)
    plan5 = WeightedBilinearTokenPlan(
        keep=torch.from_numpy(keep5)[None], source_original=torch.from_numpy(src5)[None], source_parent_compact=p5,
        source_pool_weights=ww5, source_restore_weights=ww5, original_tokens=N5, normalizer=norm5,
        key_log_mass=norm5[..., 0].log())
    g5 = torch.Generator().manual_seed(55)
    x5 = torch.randn(1, N5, D5, generator=g5)
    y5 = torch.randn(1, M5, D5, generator=g5)
    # x5 / y5 are regenerated by the tests from torch.Generator().manual_seed(55) (randn, CPU)
    out["c5_normalizer"] = _np(norm5[0, :, 0])
    out["c5_compact"] = _np(plan5.compact(x5))
    out["c5_restore"] = _np(plan5.restore(y5))

    # ---------------- CPU generator stream ----------------
    out["rand_seed3"] = _np(torch.rand(2, 4, 4, 2, generator=torch.Generator(device="cpu").manual_seed(3)))

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KB, {len(out)} arrays)")
    print("adaptive fit keys:", sorted(fit.keys()))


if __name__ == "__main__":
    main()
