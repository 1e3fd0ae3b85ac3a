"""Comparison helpers shared by the GPU parity tests.

Tolerances follow the contract of the path: float outputs within a max relative error of
2e-2 (bf16 / fp16) or 1e-5 (fp32), measured normwise as max|out - ref| / max|ref|, plus a
cosine similarity above 0.999; integer / index outputs bit-exact up to exact ties."""
from __future__ import annotations

import numpy as np
import torch

TOL = {"bf16": 2e-2, "f16": 2e-2, "f32": 1e-5}
TORCH_DTYPE = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def max_rel_err(out, ref) -> float:
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = np.abs(ref).max()
    return float(np.abs(out - ref).max() / (scale if scale > 0 else 1.0))


def cosine(out, ref) -> float:
    a = np.asarray(out, dtype=np.float64).ravel()
    b = np.asarray(ref, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(out, ref, dtype: str, tol: float | None = None) -> None:
    tol = TOL[dtype] if tol is None else tol
    err = max_rel_err(out, ref)
    cs = cosine(out, ref)
    assert err <= tol, f"max relative error {err:.3e} > {tol:.1e}"
    assert cs > 0.999, f"cosine similarity {cs:.6f} <= 0.999"


# ------------------------------------------------------------------------------------------
# Index parity: "bit-exact up to exact ties"
# ------------------------------------------------------------------------------------------
# A similarity score is round_bf16(fp32 dot product of two bf16 rows).  Its fp32 value depends
# on the accumulation order (cuBLAS, the reference's Triton kernel and this library's tcgen05
# kernel each use their own), so a score whose exact value lies within the fp32 accumulation
# error of a bf16 rounding boundary can round to either neighbour.  The contract the tests
# enforce: every index the kernel returns is the stable (ties to the lower index) top-k of
# SOME admissible score matrix — each score being the bf16 rounding of a value within
# gamma = D * 2^-24 * sum_i |a_i b_i| (the standard fp32 summation bound) of the exact dot
# product — and every value it returns is an admissible rounding of its own exact score.
# Where the kernel and the oracle pick differently, the two candidates are therefore exact
# bf16 ties under some admissible accumulation order.

def _bf16(x) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


def admissible_bf16(a_bf16, b_bf16):
    """Exact scores a @ b.T (float64) of bf16-valued rows and the [lo, hi] range of their
    admissible bf16 roundings (see above)."""
    a = np.asarray(a_bf16, dtype=np.float64)
    b = np.asarray(b_bf16, dtype=np.float64)
    exact = a @ b.T
    gamma = np.abs(a) @ np.abs(b).T * (a.shape[1] * 2.0 ** -24)
    lo = _bf16(np.nextafter((exact - gamma).astype(np.float32), -np.inf))
    hi = _bf16(np.nextafter((exact + gamma).astype(np.float32), np.inf))
    return exact, lo, hi


def check_topk_contract(lo, hi, got_v, got_i, valid=None, stable=True):
    """Assert the top-k contract above.  lo/hi [R, Nb] admissible bf16 range per score;
    got_v [R, k] (fp32) and got_i [R, k] the kernel's values and column indices; ``valid``
    [R, Nb] marks the columns a row may pick (frame groups), default all.  A row with fewer
    than k valid columns reports index -1 in the slots beyond them.  Returns the number of
    rows where an unpicked column's admissible range reaches the k-th pick (candidate ties).
    ``stable=False`` lets equal scores come in any order (torch.topk's unspecified tie order)."""
    lo = np.asarray(lo, np.float32)
    hi = np.asarray(hi, np.float32)
    R, Nb = lo.shape
    got_v = np.asarray(got_v, np.float32).reshape(R, -1)
    got_i = np.asarray(got_i, np.int64).reshape(R, -1)
    k = got_i.shape[1]
    if valid is None:
        valid = np.ones((R, Nb), bool)
    kk = np.minimum(k, valid.sum(axis=1))                      # picks per row
    pick = np.arange(k)[None, :] < kk[:, None]                 # [R, k]
    assert np.all(got_i[~pick] < 0), "a row reports more columns than it has valid ones"
    assert np.all((got_i[pick] >= 0) & (got_i[pick] < Nb)), "column index out of range"
    gi = np.where(pick, got_i, 0)
    rows = np.arange(R)[:, None]
    assert np.all(valid[rows, gi][pick]), "a pick lies outside the row's valid columns"
    srt = np.sort(np.where(pick, gi, -1 - np.arange(k)[None, :]), axis=1)
    assert np.all(srt[:, 1:] != srt[:, :-1]), "a row picks the same column twice"
    # each value is an admissible rounding of its own exact score
    inside = (lo[rows, gi] <= got_v) & (got_v <= hi[rows, gi])
    bad = np.nonzero(pick & ~inside)
    assert bad[0].size == 0, f"values outside their admissible range at rows {bad[0][:5]}"
    # stable descending order among the picks
    a, b = got_v[:, :-1], got_v[:, 1:]
    order_ok = (a > b) | ((a == b) & ((gi[:, :-1] < gi[:, 1:]) | (not stable))) | ~pick[:, 1:]
    assert np.all(order_ok), f"picks out of stable order at rows {np.nonzero(~order_ok.all(1))[0][:5]}"
    # no unpicked valid column can rank above the last pick under any admissible score
    picked = np.zeros((R, Nb), bool)
    picked[rows, gi] = pick
    has = kk > 0
    last = np.maximum(kk - 1, 0)
    vk = got_v[np.arange(R), last][:, None]
    ik = gi[np.arange(R), last][:, None]
    cols = np.arange(Nb)[None, :]
    rest = valid & ~picked & has[:, None]
    outrank = rest & ((lo > vk) | ((lo == vk) & (cols < ik) & stable))
    assert not outrank.any(), f"an unpicked column outranks the last pick at rows {np.nonzero(outrank.any(1))[0][:5]}"
    return int(np.sum((rest & (hi >= vk)).any(axis=1)))
