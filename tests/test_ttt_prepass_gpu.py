"""The TTT pre-pass kernels (ttt_kernels.py wrappers over vb200_row_l2_normalize ...
vb200_sensitivity_labels) against the oracle (oracle/ttt_prepass.py, pinned to the reference's
CPU outputs) and the reference goldens.

Bars: normalisation to fp32 rounding; local top-2 best / second scores to fp32 summation order
(rtol 1e-5), and where a best offset differs from the oracle's the two candidates' exact scores
tie within 1e-6 (a different summation order may order near-equal candidates differently);
the flows of the golden clip exactly; the integer warp bit-exact against the oracle (a gather);
motion cues to 1e-5; sensitivity to 1e-5 and the int8 predicates exactly away from their
thresholds."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _check_matches(oracle, src, tgt, ry, rx, reverse, got):
    best, second, dy, dx = (t.cpu().numpy() for t in got)
    rb, rs, rdy, rdx = oracle.ttt_prepass.local_top2_match(src, tgt, ry, rx, reverse_order=reverse)
    np.testing.assert_allclose(best, rb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(second, rs, rtol=1e-5, atol=1e-6)
    diff = (dy != rdy) | (dx != rdx)
    if diff.any():
        P, H, W, _ = src.shape
        p, y, x = np.nonzero(diff)
        s = src[p, y, x].astype(np.float64)
        ours = np.einsum("nc,nc->n", s, tgt[p, y + dy[diff], x + dx[diff]].astype(np.float64))
        theirs = np.einsum("nc,nc->n", s, tgt[p, y + rdy[diff], x + rdx[diff]].astype(np.float64))
        np.testing.assert_allclose(ours, theirs, atol=1e-6)
    return diff.sum()


def test_golden_descriptors(pkg, oracle, golden, cuda_device):
    tk = pkg.ttt_kernels
    raw = torch.from_numpy(golden["ttt_raw"]).to(cuda_device)
    desc = tk.normalize_rows(raw)
    assert desc.dtype == torch.float32 and desc.shape == raw.shape
    np.testing.assert_allclose(desc.cpu().numpy(), golden["ttt_desc"], rtol=1e-6, atol=1e-7)
    d = golden["ttt_desc"]
    dd = torch.from_numpy(d).to(cuda_device)
    fwd = tk.local_top2_match(dd[:-1], dd[1:], 2, 2)
    bwd = tk.local_top2_match(dd[1:], dd[:-1], 2, 2, reverse_order=True)
    assert fwd[2].dtype == torch.int64 and fwd[0].shape == (3, 6, 7)
    assert _check_matches(oracle, d[:-1], d[1:], 2, 2, False, fwd) == 0
    assert _check_matches(oracle, d[1:], d[:-1], 2, 2, True, bwd) == 0
    # the reference's flows are (dx, dy) of these matches
    np.testing.assert_array_equal(torch.stack([fwd[3], fwd[2]], -1).float().cpu().numpy(), golden["ttt_forward_flow"])
    np.testing.assert_array_equal(torch.stack([bwd[3], bwd[2]], -1).float().cpu().numpy(), golden["ttt_backward_flow"])
    field = torch.from_numpy(golden["ttt_field"]).to(cuda_device)
    flow = torch.from_numpy(golden["ttt_flow"]).to(cuda_device)
    warped = tk.integer_gather_warp(field, flow).cpu().numpy()
    np.testing.assert_array_equal(warped, oracle.ttt_prepass.integer_warp(golden["ttt_field"], golden["ttt_flow"]))
    np.testing.assert_allclose(warped, golden["ttt_warped"], rtol=1e-6, atol=1e-6)  # grid_sample rounding
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_local_match_realistic(pkg, oracle, cuda_device, dtype):
    """8 frames of 32 x 32 patches, 64-channel descriptors, radius 4 (81 candidates), both
    directions; bf16 descriptors are compared with the oracle on the same rounded values."""
    gen = torch.Generator().manual_seed(3)
    base = torch.randn(40, 40, 64, generator=gen)
    frames = [base[4 + k // 2:36 + k // 2, 4 + k % 3:36 + k % 3] for k in range(8)]
    raw = torch.stack(frames) + 0.5 * torch.randn(8, 32, 32, 64, generator=gen)
    desc = pkg.ttt_kernels.normalize_rows(raw.to(cuda_device)).to(dtype)
    d = desc.float().cpu().numpy()
    fwd = pkg.ttt_kernels.local_top2_match(desc[:-1], desc[1:], 4, 4)
    bwd = pkg.ttt_kernels.local_top2_match(desc[1:], desc[:-1], 4, 4, reverse_order=True)
    n = _check_matches(oracle, d[:-1], d[1:], 4, 4, False, fwd) + _check_matches(oracle, d[1:], d[:-1], 4, 4, True,
                                                                                  bwd)
    assert n <= 4, n
    # a radius clipped by the grid (H - 1) still works
    small = desc[:2, :3, :5]
    got = pkg.ttt_kernels.local_top2_match(small[:1].contiguous(), small[1:].contiguous(), 2, 4)
    _check_matches(oracle, d[:1, :3, :5], d[1:2, :3, :5], 2, 4, False, got)
    assert pkg.device_error_flags() == 0


def test_motion_cues_and_sensitivity(pkg, oracle, golden, cuda_device):
    tk, tp = pkg.ttt_kernels, oracle.ttt_prepass
    dev = cuda_device
    g = lambda k: golden[f"ttt_{k}"]
    # the golden clip: the reference's recorded prediction
    args = [g("forward_flow"), g("backward_flow"), g("predicted"), g("forward_conf"), g("backward_conf")]
    got = tk.fused_motion_cues(*(torch.from_numpy(a).to(dev) for a in args))
    for a, b in zip(got, tp.motion_cues(*args)):
        np.testing.assert_allclose(a.cpu().numpy(), b, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got[0].cpu().numpy(), g("residual"), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got[2].cpu().numpy(), g("boundary"), rtol=1e-5, atol=1e-6)
    # a larger random clip: integer flows, random predictions and confidences
    rng = np.random.default_rng(7)
    F, H, W = 5, 12, 9
    ff = rng.integers(-3, 4, (F - 1, H, W, 2)).astype(np.float32)
    bf = rng.integers(-3, 4, (F - 1, H, W, 2)).astype(np.float32)
    pred = rng.standard_normal((F, H, W, 4)).astype(np.float32)
    fc = rng.random((F - 1, H, W)).astype(np.float32)
    bc = rng.random((F - 1, H, W)).astype(np.float32)
    got = tk.fused_motion_cues(*(torch.from_numpy(a).to(dev) for a in (ff, bf, pred, fc, bc)))
    ref = tp.motion_cues(ff, bf, pred, fc, bc)
    for a, b in zip(got, ref):
        np.testing.assert_allclose(a.cpu().numpy(), b, rtol=1e-5, atol=1e-6)
    res, conf, bnd = ref
    kw = dict(uncertain_confidence=0.25, residual_scale=np.float32(np.quantile(res[1:], .9)),
              boundary_scale=np.float32(np.quantile(bnd[1:], .9)), residual_threshold=np.float32(np.median(res[1:])),
              boundary_threshold=np.float32(np.median(bnd[1:])))
    sens, low, event = tk.fused_sensitivity_labels(
        *(torch.from_numpy(a).to(dev) for a in ref),
        **{k: (torch.tensor(v, device=dev) if k != "uncertain_confidence" else v) for k, v in kw.items()})
    rs, rl, re = tp.sensitivity_labels(res, conf, bnd, **kw)
    np.testing.assert_allclose(sens.cpu().numpy(), rs, rtol=1e-5, atol=1e-6)
    assert low.dtype == torch.bool and event.dtype == torch.bool
    np.testing.assert_array_equal(low.cpu().numpy(), rl)
    np.testing.assert_array_equal(event.cpu().numpy(), re)
    assert rl.any() and re.any() and not re[0].any()
    assert pkg.device_error_flags() == 0


def test_argument_errors(pkg, cuda_device):
    tk = pkg.ttt_kernels
    a = torch.zeros(2, 4, 4, 8, device=cuda_device)
    with pytest.raises(ValueError, match="share"):
        tk.local_top2_match(a, a[:, :3], 1, 1)
    with pytest.raises(ValueError):
        tk.local_top2_match(torch.zeros(1, 4, 4, 300, device=cuda_device), torch.zeros(1, 4, 4, 300,
                                                                                     device=cuda_device), 1, 1)
    with pytest.raises(ValueError, match="field/flow"):
        tk.integer_gather_warp(a, torch.zeros(2, 4, 4, 3, device=cuda_device))
    with pytest.raises(ValueError, match="four channels"):
        tk.fused_motion_cues(a, a, torch.zeros(2, 4, 4, 3, device=cuda_device), a[..., 0], a[..., 0])
    with pytest.raises(RuntimeError, match="CUDA"):
        tk.local_top2_match(a.cpu(), a.cpu(), 1, 1)


@pytest.mark.parametrize("shape,dtype", [((5, 37), torch.float32), ((7, 64), torch.bfloat16), ((3, 1024), torch.float32),
                                         ((9, 8), torch.float16)])
def test_normalize_rows_paths(pkg, oracle, cuda_device, shape, dtype):
    """Both launch forms of vb200_row_l2_normalize: 16-byte vectors with 1-32 lanes per row, and
    the scalar fallback (a row that is not a whole number of vectors)."""
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape))).to(cuda_device, dtype)
    got = pkg.ttt_kernels.normalize_rows(x)
    ref = oracle.ttt_prepass.normalize_rows(x.float().cpu().numpy())
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-6, atol=1e-7)
