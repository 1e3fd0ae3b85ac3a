"""CPU checks of the planners' host tables: the uniform keep layout the product builds
(planners.uniform_keep_layout) equals the oracle's restatement for the benchmark layouts, and
the FastVGGT static tables reproduce the reference plan's keep set (via the oracle pinned to the
golden vectors).  No GPU involved: these tables are host data the kernels consume."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.mark.parametrize("frames,tpf,special,merge,group", [
    (32, 1029, 5, 4, 4),     # config 2
    (256, 1029, 5, 8, 4),    # config 4
    (8, 22, 2, 4, 2),        # the gloo test layout
    (12, 100, 5, 3, 4),      # uneven split of the keeps over groups
])
def test_uniform_layout_matches_oracle(pkg, oracle, frames, tpf, special, merge, group):
    from oracle import pipeline
    lay = pkg.planners.uniform_keep_layout(frames, tpf, special, merge, group)
    keep, src, qb, bb = pipeline.uniform_layout(frames, tpf, special, merge, group)
    np.testing.assert_array_equal(lay["keep"].numpy(), keep)
    np.testing.assert_array_equal(lay["source"].numpy(), src)
    np.testing.assert_array_equal(lay["q_begin"].numpy(), qb)
    np.testing.assert_array_equal(lay["b_begin"].numpy(), bb)
    total = frames * tpf
    assert keep.size == total // merge
    assert np.array_equal(np.sort(np.concatenate([keep, src])), np.arange(total))
    # every special token is kept, and its compact id points back at it
    spec = lay["special"].numpy()
    assert np.all(np.isin(spec, keep))
    np.testing.assert_array_equal(keep[lay["special_compact"].numpy()], spec)
    # sources and keeps of a group stay inside the group's frames
    for g in range(frames // group):
        lo, hi = g * group * tpf, (g + 1) * group * tpf
        assert np.all((keep[bb[g]:bb[g + 1]] >= lo) & (keep[bb[g]:bb[g + 1]] < hi))
        assert np.all((src[qb[g]:qb[g + 1]] >= lo) & (src[qb[g]:qb[g + 1]] < hi))


def test_uniform_layout_errors(pkg):
    with pytest.raises(ValueError, match="multiple of group_frames"):
        pkg.planners.uniform_keep_layout(10, 100, 5, 4, 4)
    with pytest.raises(ValueError, match="no room for patch anchors"):
        pkg.planners.uniform_keep_layout(4, 10, 8, 2, 4)  # the special tokens alone exceed the keeps


def test_uniform_layout_is_cached(pkg):
    a = pkg.planners.uniform_keep_layout(32, 1029, 5, 4, 4)
    b = pkg.planners.uniform_keep_layout(32, 1029, 5, 4, 4)
    assert a is b


@pytest.mark.parametrize("frames,hw,special,merge,protect,seed", [
    (3, (8, 8), 5, 0.9, 0.10, 0),
    (4, (7, 9), 5, 0.5, 0.05, 3),    # odd grid: the last 2x2 cells are clipped
    (2, (32, 32), 5, 0.9, 0.10, 1),  # 512 px frames: 1029 tokens each
])
def test_fastvggt_tables_match_oracle(pkg, oracle, frames, hw, special, merge, protect, seed):
    """The static FastVGGT tables (seeded destination choice, protected tokens, sources) equal
    the oracle's restatement of token_merging.py:1068-1096."""
    tpf = special + hw[0] * hw[1]
    src, dst, removed = pkg.planners.fastvggt_tables(frames, tpf, special, hw, merge, protect, seed)
    rng = np.random.default_rng(seed)
    tokens = rng.standard_normal((frames * tpf, 16)).astype(np.float32)
    _, _, _, _, src_o, dst_o = oracle.fastvggt_plan(tokens, frames=frames, tokens_per_frame=tpf,
                                                    patch_token_start=special, patch_hw=hw,
                                                    merge_ratio=merge, protect_ratio=protect, seed=seed)
    np.testing.assert_array_equal(src.numpy(), src_o)
    np.testing.assert_array_equal(dst.numpy(), dst_o)
    assert removed == min(int(frames * tpf * merge), src_o.size)
