"""CPU checks of the C ABI: the library loads, exports exactly the symbols that
include/vggt_b200.h declares, and rejects bad arguments on the host (before any launch) with
the reference's exception types."""
from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import REPO

HEADER = REPO / "include" / "vggt_b200.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"VB200_API\s+[\w\s\*]+?\b(vb200_\w+)\s*\(", text))


def test_header_declares_entry_points():
    names = _declared()
    assert "vb200_mass_bias_attention" in names and "vb200_proj_gather" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    for name in sorted(_declared()):
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_binding_covers_header(pkg):
    assert set(pkg._clib.EXPORTED_SYMBOLS) == _declared()


def test_version_and_error_text(pkg):
    lib = pkg.load_library()
    assert lib.vb200_version() >= 1
    # head_dim 32 is rejected on the host before any CUDA call
    strides = (ctypes.c_int64 * 3)(1, 1, 1)
    rc = lib.vb200_mass_bias_attention(1, 16, 16, 16, None, 0, 16, 1, 1, 1, 1, 32, strides, strides,
                                       strides, strides, 16, 1 << 20, None)
    assert rc == pkg._clib.EINVAL
    assert b"head_dim=64" in lib.vb200_last_error()
    with pytest.raises(ValueError, match="head_dim"):
        pkg._clib.check(rc, "mass_bias_attention")


def test_reference_exceptions_without_gpu(pkg):
    q = torch.zeros(1, 2, 4, 32)
    with pytest.raises(ValueError, match="head_dim=64"):
        pkg.mass_bias_attention(q, q, q, torch.zeros(4))
    with pytest.raises(ValueError, match="batch, heads"):
        pkg.mass_bias_attention(q[0], q[0], q[0], torch.zeros(4))
    q = torch.zeros(1, 2, 4, 64)
    with pytest.raises(ValueError, match="incompatible"):
        pkg.mass_bias_attention(q, q[:, :, :3], q, torch.zeros(3))
    # well-formed CPU tensors: no CPU fallback
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.mass_bias_attention(q, q, q, torch.zeros(4))
    with pytest.raises(ValueError, match="Gram"):
        pkg.four_support_projected_gradient(torch.zeros(3, 3, 3), torch.zeros(3, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.four_support_projected_gradient(torch.zeros(3, 4, 4), torch.zeros(3, 4))
    with pytest.raises(RuntimeError):
        pkg.streaming_top4(torch.zeros(4, 64), torch.zeros(64, 8))


def test_host_side_size_checks(pkg):
    lib = pkg.load_library()
    assert lib.vb200_mass_bias_attention_workspace_size(1) == 4096
    assert lib.vb200_mass_bias_attention_workspace_size(129) == 8192
    rc = lib.vb200_proj_gather(1, None, 0, None, 0, None, None, None, 0, 9, None, 0, 0, 8, 0, None)
    assert rc == pkg._clib.EINVAL and b"corners" in lib.vb200_last_error()
    rc = lib.vb200_sim_topk(None, 0, None, 0, 4, 4, 64, 3, None, None, 1, None, None, None)
    assert rc != 0


def test_peer_exchange_argument_checks(pkg):
    lib = pkg.load_library()
    one = (ctypes.c_uint64 * 1)(16)
    rc = lib.vb200_peer_gather(one, 17, 1, 16, 16, None, 16, None)
    assert rc == pkg._clib.EINVAL and b"world" in lib.vb200_last_error()
    rc = lib.vb200_peer_gather(one, 1, 1, 16, 6, 16, 16, None)
    assert rc == pkg._clib.EINVAL and b"multiples of 4" in lib.vb200_last_error()
    rc = lib.vb200_peer_push(8, 1, 16, 16, one, 1, 0, 16, None)  # source not 16-byte aligned
    assert rc == pkg._clib.EINVAL and b"16-byte" in lib.vb200_last_error()


def _attention_plan(lib, B, H, Nq, Nk, sms):
    out = (ctypes.c_int64 * 5)()
    assert lib.vb200_mass_bias_attention_plan(B, H, Nq, Nk, sms, out) == 0
    return list(out)


def test_attention_launch_plan(pkg):
    """The last-wave key split of the attention launch (host arithmetic, no GPU)."""
    lib = pkg.load_library()
    # config 2: 33 query blocks x 16 heads = 528 items on 148 SMs -> 3 whole waves + 84 split
    items, n_full, n_tail, split, extra = _attention_plan(lib, 1, 16, 8232, 8232, 148)
    assert (items, n_full, n_tail) == (528, 444, 84) and 2 <= split <= 4 and extra > 0
    # the split is what the cost model says: ceil(tail * s / SMs) rounds of (1/s + 3/65)
    cost = lambda s: -(-84 * s // 148) * (1 / s + 3 / 65)  # noqa: E731
    assert cost(split) == min(cost(s) for s in range(1, 5))
    # a whole number of waves, or a single key tile: nothing to split
    assert _attention_plan(lib, 1, 148, 256, 8232, 148)[3] == 1
    assert _attention_plan(lib, 1, 16, 8232, 100, 148)[3] == 1
    # N = 8 shard of config 2: 5 query blocks x 16 heads = 80 items, fewer than the SMs
    items, n_full, n_tail, split, _ = _attention_plan(lib, 1, 16, 1029, 8232, 148)
    assert (items, n_full, n_tail) == (80, 0, 80) and split > 1
    # the workspace query agrees with the plan
    assert lib.vb200_mass_bias_attention_split_workspace_size(1, 16, 8232, 8232) == \
        lib.vb200_mass_bias_attention_workspace_size(8232) + _attention_plan(lib, 1, 16, 8232, 8232, 148)[4] \
        or lib.vb200_mass_bias_attention_split_workspace_size(1, 16, 8232, 8232) == \
        lib.vb200_mass_bias_attention_workspace_size(8232)  # no device here: SM count unknown -> unsplit


def test_topk_split_choice(pkg):
    lib = pkg.load_library()
    assert lib.vb200_sim_topk_split(200, 5, 148) == 1   # config 2, 8 frame groups: enough CTAs
    assert lib.vb200_sim_topk_split(25, 5, 148) == 3    # one frame group (N = 8 shard)
    assert lib.vb200_sim_topk_split(25, 1, 148) == 1    # a single basis tile cannot split
    assert lib.vb200_sim_topk_split(25, 2, 148) == 1    # halving 2 tiles does not pay for the merge launch
    assert lib.vb200_sim_topk_split(25, 3, 148) == 3
    assert lib.vb200_sim_topk_split(10, 5, 0) == 1      # unknown SM count
