"""install() inside the reference's own model: VGGTOmega() from the pip-installed reference
(baseline/_ref, skipped when absent) with random weights, bf16 autocast and the released
merging configuration (configs/ttt_best.py: the released planner with geometry-guarded supports,
compact Q/K/V on all global layers but 8, 10, 11, 12), run stock (the reference's Triton
kernels) and with install() routing every global layer's planner, compaction, mass-bias
attention and restore through this library.  On a static scene (one image repeated with 2%
noise) the planner merges; the two forwards must agree to the bf16 bar (max relative error
<= 2e-2, cosine > 0.999) on the final tokens, depth and pose, with the same number of kept
tokens per layer up to a few boundary decisions."""
from __future__ import annotations

import os
import sys

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu

REF = REPO / "baseline" / "_ref"
ENV = {"VGGT_TTT_REUSE_PLAN": "0", "VGGT_TTT_FIXED_TOPOLOGY": "0", "VGGT_TTT_LOCAL_SUPPORT_SEARCH": "1",
       "VGGT_TTT_FIT_CHUNK": "4096", "VGGT_TTT_LOCAL_SOLVER": "projected", "VGGT_TRITON_ACTIVE_SET": "0",
       "VGGT_TRITON_MASS_BIAS_ATTENTION": "1"}


@pytest.mark.skipif(not (REF / "vggt_omega").exists(), reason="the reference is not installed under baseline/_ref")
def test_installed_forward_matches_stock(pkg, cuda_device):
    dev = cuda_device
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    for k, v in ENV.items():
        os.environ.setdefault(k, v)
    from vggt_omega.models.vggt_omega import VGGTOmega
    frames, size = 6, 192
    torch.manual_seed(0)
    with torch.device(dev):
        model = VGGTOmega().eval()
    model.to(dev)
    agg = model.aggregator
    ph = size // 16
    patches = frames * ph * ph
    gen = torch.Generator().manual_seed(3)
    labels = (torch.rand(patches, generator=gen) < 0.08).long()
    labels[: ph * ph] = 0
    sens = torch.rand(patches, generator=gen)
    xyz = torch.randn(ph * ph, 3, generator=gen)[None] + 0.3 * torch.randn(frames, ph * ph, 3, generator=gen)
    geo = torch.cat([xyz, torch.linspace(-1, 1, frames)[:, None, None].expand(-1, ph * ph, 1)], -1).reshape(-1, 4)
    agg.set_sparse_convex(enabled=True, threshold=0.90, planner="ttt_protected_uniform_convex", max_support=4,
                          qkv_global_layers=tuple(l for l in range(19) if l not in {8, 10, 11, 12}),
                          dense_global_layers=())
    agg.set_sparse_convex_ttt_top1_pruning(False)
    agg.set_sparse_convex_ttt_sensitive_event_ratio(0.01)
    agg.set_sparse_convex_4d(geo.to(dev), global_layers=tuple(range(19)), selection_weight=0.01, support_weight=0.01,
                             guard_tolerance=0.0)
    agg.set_sparse_convex_ttt_partition(labels.to(dev), sens.to(dev))
    g = torch.Generator(device=dev).manual_seed(4)
    images = (torch.rand(1, 1, 3, size, size, device=dev, generator=g)
              + 0.02 * torch.randn(1, frames, 3, size, size, device=dev, generator=g)).clamp(0, 1)
    with torch.no_grad():
        ref = model(images)
        ref_kept = [s["kept_tokens"] for s in agg.sparse_convex_last_plan_stats]
        n0 = pkg._clib.lib().vb200_launch_count()
        pkg.install()
        try:
            ours = model(images)
        finally:
            pkg.uninstall()
        launches = pkg._clib.lib().vb200_launch_count() - n0
        our_kept = [s["kept_tokens"] for s in agg.sparse_convex_last_plan_stats]
    torch.cuda.synchronize()
    assert launches > 19 * 10  # the global layers ran on this library
    assert len(ref_kept) == len(our_kept) == 19
    total = frames * (ph * ph + agg.patch_token_start)
    assert min(ref_kept) < 0.6 * total  # merging is active
    for a, b in zip(our_kept, ref_kept):
        assert abs(a - b) <= max(4, 0.01 * b), (our_kept, ref_kept)
    for key in ("camera_and_register_tokens", "depth", "pose_enc"):
        a, b = ours[key].float().flatten(), ref[key].float().flatten()
        err = ((a - b).abs().max() / b.abs().max()).item()
        cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
        assert err <= 2e-2 and cos > 0.999, (key, err, cos)
    assert pkg.device_error_flags() == 0
