"""install() rebinds the reference's hot-path names to the B200 operators (CPU check: the
reference is importable in the build container; nothing is computed)."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

# a reference checkout named by REFERENCE_ROOT, else the pip install under baseline/_ref
# (neither present: the test skips)
_INSTALLED = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
REFERENCE = (Path(os.environ["REFERENCE_ROOT"]) if os.environ.get("REFERENCE_ROOT")
             else _INSTALLED if (_INSTALLED / "vggt_omega").exists() else None)


@pytest.mark.skipif(REFERENCE is None or not (REFERENCE / "vggt_omega").exists(),
                    reason="REFERENCE_ROOT does not name a reference checkout")
def test_install_patches_reference(pkg):
    patched = pkg.install(str(REFERENCE))
    try:
        mba = sys.modules["vggt_omega.models.mass_bias_attention"]
        tm = sys.modules["vggt_omega.models.token_merging"]
        sc = sys.modules["vggt_omega.models.sparse_convex"]
        assert mba.mass_bias_attention is pkg.mass_bias_attention
        assert tm.WeightedBilinearTokenPlan is pkg.WeightedBilinearTokenPlan
        assert tm.build_fastvggt_plan is pkg.build_fastvggt_plan
        assert sc.WeightedBilinearTokenPlan is pkg.WeightedBilinearTokenPlan
        assert sc.four_support_projected_gradient is pkg.four_support_projected_gradient
        assert "vggt_omega.models.sparse_convex_kernels.streaming_top4" in patched
        agg = sys.modules["vggt_omega.models.aggregator"]
        assert sc.build_ttt_protected_uniform_convex_plan is pkg.build_ttt_protected_uniform_convex_plan
        assert agg.build_ttt_protected_uniform_convex_plan is pkg.build_ttt_protected_uniform_convex_plan
    finally:
        pkg.uninstall()
    assert sys.modules["vggt_omega.models.mass_bias_attention"].mass_bias_attention is not pkg.mass_bias_attention
