"""Four-support simplex solvers on the GPU against the oracle and the reference goldens."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import to_np

pytestmark = pytest.mark.gpu


def _gram_rhs(sup, src):
    gram = np.einsum("rid,rjd->rij", sup, sup).astype(np.float32)
    rhs = np.einsum("rid,rd->ri", sup, src).astype(np.float32)
    return gram, rhs


def test_projected_gradient_golden(pkg, golden, oracle, cuda_device):
    feats = golden["pg_features"].astype(np.float64)
    ids = golden["pg_support_ids"].astype(np.int64)
    gram, rhs = _gram_rhs(feats[ids], feats)
    out = pkg.four_support_projected_gradient(torch.from_numpy(gram).to(cuda_device),
                                              torch.from_numpy(rhs).to(cuda_device), steps=32)
    np.testing.assert_allclose(to_np(out), golden["pg_weights"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(to_np(out), oracle.projected_gradient(gram, rhs, 32), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_np(out).sum(axis=1), 1.0, atol=1e-5)
    assert (to_np(out) >= 0).all()


def test_active_set_golden(pkg, golden, oracle, cuda_device):
    src = golden["as_source"].astype(np.float64)
    sup = golden["as_supports"].astype(np.float64)
    gram, rhs = _gram_rhs(sup, src)
    out = to_np(pkg.four_support_active_set(torch.from_numpy(gram).to(cuda_device),
                                            torch.from_numpy(rhs).to(cuda_device), ridge=1e-4))
    np.testing.assert_allclose(out, golden["as_alpha"], rtol=1e-3, atol=2e-4)
    np.testing.assert_allclose(out, oracle.active_set(gram, rhs, 1e-4), rtol=1e-3, atol=1e-4)


def test_random_rows(pkg, oracle, cuda_device):
    rng = np.random.default_rng(4)
    src = rng.standard_normal((5000, 32))
    src /= np.linalg.norm(src, axis=1, keepdims=True)
    sup = src[:, None] + 0.5 * rng.standard_normal((5000, 4, 32))
    sup /= np.linalg.norm(sup, axis=2, keepdims=True)
    gram, rhs = _gram_rhs(sup, src)
    out = to_np(pkg.four_support_projected_gradient(torch.from_numpy(gram).to(cuda_device),
                                                    torch.from_numpy(rhs).to(cuda_device)))
    np.testing.assert_allclose(out, oracle.projected_gradient(gram, rhs, 32), rtol=1e-5, atol=1e-6)
