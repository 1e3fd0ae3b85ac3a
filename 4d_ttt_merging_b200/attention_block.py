"""Global-attention block with a token plan, on the B200 operators.

``GlobalAttention`` holds the parameters of the reference's ``SelfAttention`` as used by the
aggregator's global blocks (vggt_omega/models/layers/attention.py:210-241 with qkv_bias,
proj_bias, mask_k_bias and use_qk_norm, as vggt_omega/models/aggregator.py:96-110 builds them)
and runs ``forward(x, token_plan=...)`` with the reference's semantics
(attention.py:264-314, 328-439):

    qkv = qkv(x)  (cuBLAS)  ->  q/k LayerNorm over the head dim
    compact:  compact-query plans compact Q, K and V; query-preserving plans keep all
              queries, physical keys (compact_key) and pooled values
    mass-bias attention over the compact keys with bias key_log_mass  (tcgen05 kernel)
    dense special queries: exact attention of the camera / register queries over the dense
              K/V (the same kernel without bias), written over their compact rows
    proj  (cuBLAS)  ->  restore  (top-4 gather kernel)

Tensors stay token-major throughout: Q/K/V are [B, T, H, 64] views of the qkv buffer and
the attention output is written token-major, so no transposes are materialised.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .ops import head_layernorm, mass_bias_attention, row_gather
from .token_plan import WeightedBilinearTokenPlan

__all__ = ["GlobalAttention", "compute_attention"]


def _bhtd(x: torch.Tensor, heads: int) -> torch.Tensor:
    """[B, T, C] -> [B, H, T, d] view."""
    B, T, C = x.shape
    return x.view(B, T, heads, C // heads).transpose(1, 2)


def _ln_params(q_norm, k_norm):
    if q_norm is None or k_norm is None:
        return None, None, 1e-5
    w = torch.stack([q_norm.weight.detach(), k_norm.weight.detach()]).float()
    b = torch.stack([q_norm.bias.detach(), k_norm.bias.detach()]).float()
    return w, b, float(q_norm.eps)


def _fused_ok(qkv: torch.Tensor, token_plan, q_norm, k_norm) -> bool:
    """The one-kernel LayerNorm + Q||K||V compaction applies to 16-bit qkv buffers with a
    WeightedBilinearTokenPlan without a separate query plan."""
    if not isinstance(token_plan, WeightedBilinearTokenPlan) or token_plan.query_keep is not None:
        return False
    if qkv.dtype not in (torch.bfloat16, torch.float16) or qkv.shape[0] != 1 or (qkv.shape[2] // 3) % 256:
        return False
    if (q_norm is None) != (k_norm is None):
        return False
    return q_norm is None or (q_norm.elementwise_affine and tuple(q_norm.normalized_shape) == (64,))


def _compute_attention_fused(qkv, num_heads, plan, q_norm, k_norm):
    B, N, C3 = qkv.shape
    C = C3 // 3
    x = qkv[0]
    lw, lb, eps = _ln_params(q_norm, k_norm)
    preserve = plan.preserve_queries
    if preserve:
        mask = 0b100 | (0 if plan.preserve_destination_keys else 0b010)
    else:
        mask = 0b111
    packed = plan.compact_qkv(x, lw, lb, eps, pool_mask=mask)  # [M, 3C]
    M = packed.shape[0]
    view = lambda t, T: t.view(1, T, num_heads, C // num_heads).transpose(1, 2)
    if preserve:
        q = head_layernorm(x[:, :C], lw[0], lb[0], eps) if lw is not None else x[:, :C]
        qv = view(q, N)
    else:
        qv = view(packed[:, :C], M)
    o = mass_bias_attention(qv, view(packed[:, C:2 * C], M), view(packed[:, 2 * C:], M), plan.key_log_mass)
    if plan.dense_special_queries:
        original, out_index = plan.special_query_original, (
            plan.special_query_original if preserve else plan.special_query_compact)
        if original is None or out_index is None:
            raise RuntimeError("dense-special attention plan has no special-token mapping")
        qs = row_gather(x[:, :C], original)
        if lw is not None:
            qs = head_layernorm(qs, lw[0], lb[0], eps)
            kd = head_layernorm(x[:, C:2 * C], lw[1], lb[1], eps)
        else:
            kd = x[:, C:2 * C]
        exact = mass_bias_attention(view(qs, qs.shape[0]), view(kd, N), view(x[:, 2 * C:], N), None)
        o.index_copy_(2, out_index, exact)
    return o.transpose(1, 2).reshape(B, o.shape[2], C)


def compute_attention(qkv: torch.Tensor, num_heads: int, token_plan, q_norm: nn.Module | None = None,
                      k_norm: nn.Module | None = None) -> torch.Tensor:
    """Attention part of SelfAttention.compute_attention (attention.py:328-439) for a global
    block with a token plan; returns [B, Nq, C] (Nq = compact query count or N).

    16-bit qkv buffers with a WeightedBilinearTokenPlan take the fused path: one kernel
    LayerNorms q/k per head and compacts Q||K||V (``vb200_compact_qkv``).  Other inputs
    (fp32, hard-merge TokenPlan, separate query plans) compose the individual operators."""
    if token_plan is not None and _fused_ok(qkv, token_plan, q_norm, k_norm):
        return _compute_attention_fused(qkv, num_heads, token_plan, q_norm, k_norm)
    B, N, C3 = qkv.shape
    C = C3 // 3
    hd = C // num_heads
    q, k, v = qkv.view(B, N, 3, num_heads, hd).unbind(2)  # [B, N, H, hd] views
    if q_norm is not None:
        q = q_norm(q)
    if k_norm is not None:
        k = k_norm(k)
    flat = lambda t: t.reshape(B, N, C)
    dense_q, dense_k, dense_v = q, k, v
    if token_plan is None:
        x = mass_bias_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None)
        return x.transpose(1, 2).reshape(B, N, C)
    if getattr(token_plan, "preserve_queries", False):
        key = token_plan.compact_key(flat(k)) if hasattr(token_plan, "compact_key") else token_plan.compact(flat(k))
        qc, kc, vc = flat(q), key, token_plan.compact(flat(v))
    else:
        qc = token_plan.compact_query(flat(q)) if hasattr(token_plan, "compact_query") else token_plan.compact(flat(q))
        kc, vc = token_plan.compact(flat(k)), token_plan.compact(flat(v))
    bias = getattr(token_plan, "key_log_mass", None)  # None: plain softmax attention
    x = mass_bias_attention(_bhtd(qc, num_heads), _bhtd(kc, num_heads), _bhtd(vc, num_heads), bias)
    if getattr(token_plan, "dense_special_queries", False):
        original = token_plan.special_query_original
        out_index = original if getattr(token_plan, "preserve_queries", False) else token_plan.special_query_compact
        if original is None or out_index is None:
            raise RuntimeError("dense-special attention plan has no special-token mapping")
        exact = mass_bias_attention(dense_q.index_select(1, original).transpose(1, 2), dense_k.transpose(1, 2),
                                    dense_v.transpose(1, 2), None)
        x.index_copy_(2, out_index, exact.to(x.dtype))
    return x.transpose(1, 2).reshape(B, x.shape[2], C)


class GlobalAttention(nn.Module):
    """Parameters and forward of a global-block SelfAttention (dim, heads, qkv / proj bias,
    masked k bias, q/k LayerNorm)."""

    def __init__(self, dim: int, num_heads: int, qkv_bias: bool = True, proj_bias: bool = True,
                 mask_k_bias: bool = True, use_qk_norm: bool = True, device=None, dtype=None) -> None:
        super().__init__()
        self.num_heads = num_heads
        head_dim = dim // num_heads
        factory = dict(device=device, dtype=dtype)
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias, **factory)
        self.proj = nn.Linear(dim, dim, bias=proj_bias, **factory)
        self.use_qk_norm = use_qk_norm
        self.q_norm = nn.LayerNorm(head_dim, eps=1e-5, **factory) if use_qk_norm else None
        self.k_norm = nn.LayerNorm(head_dim, eps=1e-5, **factory) if use_qk_norm else None
        mask = torch.ones(dim * 3, device=device, dtype=dtype or torch.float32)
        if mask_k_bias:
            mask[dim: 2 * dim] = 0
        self.register_buffer("bias_mask", mask)

    def load_reference_state(self, state: dict) -> None:
        """Load a state dict of the reference SelfAttention (names qkv.*, proj.*, q_norm.*,
        k_norm.*, qkv.bias_mask)."""
        own = {k: v for k, v in state.items() if k != "qkv.bias_mask"}
        self.load_state_dict({**own, "bias_mask": state.get("qkv.bias_mask", self.bias_mask)}, strict=True)

    def _masked_qkv_bias(self):
        """qkv bias with the key part zeroed (the reference's LinearKMaskedBias,
        layers/attention.py:195-207), cached until either tensor is modified in place (torch's
        version counters), so a step does not recompute it."""
        b = self.qkv.bias
        if b is None:
            return None
        key = (b.data_ptr(), b._version, self.bias_mask.data_ptr(), self.bias_mask._version, b.dtype)
        cached = getattr(self, "_bias_cache", None)
        if cached is None or cached[0] != key:
            cached = (key, b * self.bias_mask.to(b.dtype))
            self._bias_cache = cached
        return cached[1]

    def qkv_projection(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.qkv.weight, self._masked_qkv_bias())

    def forward(self, x: torch.Tensor, token_plan=None) -> torch.Tensor:
        qkv = (token_plan.precomputed_qkv
               if token_plan is not None and getattr(token_plan, "precomputed_qkv", None) is not None
               else self.qkv_projection(x))
        attn = compute_attention(qkv, self.num_heads, token_plan, self.q_norm, self.k_norm)
        y = self.proj(attn)
        if token_plan is None:
            return y
        return token_plan.restore(y)
