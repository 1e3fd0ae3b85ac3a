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
