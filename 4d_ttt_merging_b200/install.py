"""Route a reference checkout (shuang-yang18/4D_TTT_merging) through the B200 operators.

``install()`` rebinds, in the already-imported reference modules, the names the global
blocks call, in the manner of the reference's own ``fast_affine.install``
(vggt_omega/models/fast_affine.py:738-745):

* ``vggt_omega.models.mass_bias_attention.mass_bias_attention`` (imported at call time by
  attention.py:397-398)
* ``vggt_omega.models.sparse_convex_kernels.streaming_top4`` /
  ``four_support_projected_gradient`` / ``four_support_active_set`` and their aliases in
  ``vggt_omega.models.sparse_convex``
* ``vggt_omega.models.sparse_convex.build_ttt_protected_uniform_convex_plan`` (the released
  planner, called by the aggregator's global branch, aggregator.py:922)
* ``vggt_omega.models.token_merging.TokenPlan`` / ``WeightedBilinearTokenPlan`` /
  ``deterministic_weighted_normalizer`` / ``build_fastvggt_plan`` and their aliases in the
  planner modules that imported them by name.

The attention layer then runs compaction, mass-bias attention and restore on the GPU kernels
unchanged.  ``uninstall()`` restores the originals.
"""
from __future__ import annotations

import importlib
import sys

from . import ops, planners, token_plan

__all__ = ["install", "uninstall", "REPLACEMENTS"]

REPLACEMENTS = {
    "vggt_omega.models.mass_bias_attention": {"mass_bias_attention": ops.mass_bias_attention},
    "vggt_omega.models.sparse_convex_kernels": {
        "streaming_top4": ops.streaming_top4,
        "four_support_projected_gradient": ops.four_support_projected_gradient,
        "four_support_active_set": ops.four_support_active_set,
    },
    "vggt_omega.models.sparse_convex": {
        "build_ttt_protected_uniform_convex_plan": planners.build_ttt_protected_uniform_convex_plan,
    },
    "vggt_omega.models.token_merging": {
        "TokenPlan": token_plan.TokenPlan,
        "WeightedBilinearTokenPlan": token_plan.WeightedBilinearTokenPlan,
        "deterministic_weighted_normalizer": ops.deterministic_weighted_normalizer,
        "build_fastvggt_plan": planners.build_fastvggt_plan,
    },
}
# modules that import the names above with ``from ... import name``
ALIAS_MODULES = ("vggt_omega.models.sparse_convex", "vggt_omega.models.fast_affine",
                 "vggt_omega.models.aggregator", "vggt_omega.models.layers.attention")

_saved: dict[tuple[str, str], object] = {}


def install(reference_root: str | None = None) -> list[str]:
    """Patch the reference modules; returns the list of patched ``module.name`` entries."""
    if reference_root is not None and reference_root not in sys.path:
        sys.path.insert(0, reference_root)
    patched = []
    names = {}
    for mod_name, table in REPLACEMENTS.items():
        mod = importlib.import_module(mod_name)
        for name, new in table.items():
            if hasattr(mod, name):
                _saved.setdefault((mod_name, name), getattr(mod, name))
                setattr(mod, name, new)
                patched.append(f"{mod_name}.{name}")
                names[name] = new
    for mod_name in ALIAS_MODULES:
        try:
            mod = importlib.import_module(mod_name)
        except Exception:  # optional modules of the reference
            continue
        for name, new in names.items():
            if hasattr(mod, name):
                _saved.setdefault((mod_name, name), getattr(mod, name))
                setattr(mod, name, new)
                patched.append(f"{mod_name}.{name}")
    return patched


def uninstall() -> None:
    for (mod_name, name), old in _saved.items():
        setattr(sys.modules[mod_name], name, old)
    _saved.clear()
