"""The reference's own PyTorch call sequence for one benchmark step, on CPU (CPU baseline and
test infrastructure: the timed CPU baseline and reference arm of bench.py; never a product path).

The reference (shuang-yang18/4D_TTT_merging) is a PyTorch program whose GPU kernels are Triton;
on a CPU it runs the PyTorch operators below.  This module restates that sequence with the
same torch operators, in the same order and dtypes, so that timing it on the host cores times
the reference's CPU path for the configuration the GPU bench runs:

* plan (sparse-convex, uniform keep set; the support search of sparse_convex.py:546-552):
  ``F.normalize(x.float()).to(bf16)`` features (:1791-1793); per frame group the bf16 score
  GEMM ``source.bf16 @ basis.bf16.T`` and ``topk(4)``; the fp32 Gram / rhs of the chosen
  supports (``supports.float() @ supports.T``, :2312-2316) and the 32-step projected gradient
  of four_support_projected_gradient (sparse_convex_kernels.py:214-296, restated with torch
  tensor ops because the Triton kernel cannot run on a CPU); the plan's stable argsort +
  bincount per corner (token_merging.py:323-333) and deterministic_weighted_normalizer
  (:40-59); key_log_mass = log(mass).
* block (SelfAttention.forward with the plan, layers/attention.py:264-439): the k-masked qkv
  Linear (:195-207), q/k LayerNorm over the head dim, WeightedBilinearTokenPlan.compact of
  Q, K and V (token_merging.py:343-370: gather, fp32 accumulation, per-corner index_select +
  segment_reduce, divide by the normaliser), SDPA with ``attn_mask = key_log_mass``
  (attention.py:386-400), the proj Linear and WeightedBilinearTokenPlan.restore
  (token_merging.py:387-414: zeros, kept rows, value-dtype weighted sum of the four parents).

The keep layout is 4d_ttt_merging_b200.planners.uniform_keep_layout (restated in
oracle.pipeline.uniform_layout).  tests/test_torch_path.py checks this module against the numpy
oracle, which the golden vectors pin to the reference.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

__all__ = ["TorchPlan", "normalizer", "projected_gradient", "build_plan", "compact", "restore",
           "block_forward", "step", "params_to_torch"]


@dataclass
class TorchPlan:
    keep: torch.Tensor            # [K] int64 token ids
    source: torch.Tensor          # [S] int64 token ids
    parent: torch.Tensor          # [S, 4] int64 compact ids
    weights: torch.Tensor         # [S, 4] fp32 (pool = restore weights)
    normalizer: torch.Tensor      # [K] fp32 mass
    key_log_mass: torch.Tensor    # [K] fp32
    orders: tuple                 # per corner: stable argsort of the parents
    lengths: tuple                # per corner: bincount of the parents
    original_tokens: int


def _corner_orders(parent: torch.Tensor, kept: int):
    orders, lengths = [], []
    for c in range(parent.shape[1]):
        dest = parent[:, c]
        orders.append(dest.argsort(stable=True))
        lengths.append(torch.bincount(dest, minlength=kept))
    return tuple(orders), tuple(lengths)


def normalizer(parent: torch.Tensor, weights: torch.Tensor, kept: int) -> torch.Tensor:
    """mass = 1 + per-corner segment sums of the weights in stable source order
    (token_merging.py:40-59).  parent/weights [S, 4]; returns fp32 [K]."""
    mass = torch.ones(kept, dtype=torch.float32)
    for c in range(parent.shape[1]):
        dest = parent[:, c]
        order = dest.argsort(stable=True)
        lengths = torch.bincount(dest, minlength=kept)
        mass = mass + torch.segment_reduce(weights[:, c].index_select(0, order).float(), "sum", lengths=lengths)
    return mass


def _simplex_project(v: torch.Tensor) -> torch.Tensor:
    s = v.sort(dim=-1, descending=True).values
    cssv = s.cumsum(dim=-1) - 1.0
    ranks = torch.arange(1, v.shape[-1] + 1, dtype=v.dtype)
    active = s > cssv / ranks
    rho = active.sum(dim=-1).clamp_min(1) - 1
    theta = cssv.gather(-1, rho[..., None]) / (rho[..., None].to(v.dtype) + 1)
    return (v - theta).clamp_min(0)


def projected_gradient(gram: torch.Tensor, rhs: torch.Tensor, steps: int = 32) -> torch.Tensor:
    """alpha_0 = e_0; step = 0.95 / max(max row abs-sum, 1e-4); ``steps`` projected-gradient
    iterations on the simplex (sparse_convex_kernels.py:244-280).  gram [R,4,4], rhs [R,4]."""
    step = 0.95 / gram.abs().sum(dim=-1).amax(dim=-1).clamp_min(1e-4)
    alpha = torch.zeros_like(rhs)
    alpha[:, 0] = 1
    for _ in range(steps):
        grad = torch.bmm(gram, alpha[..., None])[..., 0] - rhs
        alpha = _simplex_project(alpha - step[:, None] * grad)
    return alpha


def build_plan(tokens: torch.Tensor, layout, steps: int = 32) -> TorchPlan:
    """tokens [N, D] (float); layout = (keep, source, query group begins, basis group begins)."""
    keep, src, qb, bb = (torch.as_tensor(a, dtype=torch.int64) for a in layout)
    features = F.normalize(tokens.float(), dim=-1).to(torch.bfloat16)
    src_feat = features.index_select(0, src)
    basis_feat = features.index_select(0, keep)
    parent = torch.empty((src.numel(), 4), dtype=torch.int64)
    for g in range(qb.numel() - 1):
        q0, q1, b0, b1 = int(qb[g]), int(qb[g + 1]), int(bb[g]), int(bb[g + 1])
        score = src_feat[q0:q1] @ basis_feat[b0:b1].T   # bf16 GEMM, fp32 accumulation
        parent[q0:q1] = score.topk(4, dim=-1).indices + b0
    supports = basis_feat.index_select(0, parent.reshape(-1)).reshape(src.numel(), 4, -1).float()
    gram = supports @ supports.transpose(1, 2)
    rhs = (supports @ src_feat.float().unsqueeze(-1)).squeeze(-1)
    alpha = projected_gradient(gram, rhs, steps)
    mass = normalizer(parent, alpha, keep.numel())
    orders, lengths = _corner_orders(parent, keep.numel())
    return TorchPlan(keep, src, parent, alpha, mass, mass.log(), orders, lengths, tokens.shape[0])


def compact(plan: TorchPlan, value: torch.Tensor) -> torch.Tensor:
    """WeightedBilinearTokenPlan.compact for value [N, C] (token_merging.py:343-370)."""
    acc_dtype = torch.float32 if value.dtype in (torch.float16, torch.bfloat16) else value.dtype
    out = value.index_select(0, plan.keep).to(acc_dtype)
    if plan.source.numel() == 0:
        return out.to(value.dtype)
    source = value.index_select(0, plan.source).to(acc_dtype)
    for c in range(plan.parent.shape[1]):
        order = plan.orders[c]
        w = plan.weights[:, c].index_select(0, order).to(acc_dtype)[:, None]
        out = out + torch.segment_reduce(source.index_select(0, order) * w, "sum", lengths=plan.lengths[c])
    return (out / plan.normalizer.to(acc_dtype)[:, None]).to(value.dtype)


def restore(plan: TorchPlan, value: torch.Tensor) -> torch.Tensor:
    """WeightedBilinearTokenPlan.restore for value [K, C] (token_merging.py:387-414)."""
    out = value.new_zeros((plan.original_tokens, value.shape[-1]))
    out[plan.keep] = value
    if plan.source.numel():
        parents = value[plan.parent]                                  # [S, 4, C]
        out[plan.source] = (parents * plan.weights[..., None].to(value.dtype)).sum(dim=1).to(value.dtype)
    return out


def params_to_torch(params: dict) -> dict:
    return {k: torch.as_tensor(v, dtype=torch.float32) for k, v in params.items()}


def block_forward(tokens: torch.Tensor, params: dict, plan: TorchPlan, heads: int) -> torch.Tensor:
    """SelfAttention.forward with a compact-query WeightedBilinearTokenPlan (no dense special
    queries), fp32 on CPU.  tokens [N, dim]; params: fp32 tensors by module name."""
    N, dim = tokens.shape
    hd = dim // heads
    qkv = F.linear(tokens, params["qkv.weight"], params["qkv.bias"] * params["qkv.bias_mask"])
    q, k, v = qkv.reshape(N, 3, heads, hd).unbind(1)                   # [N, H, hd]
    q = F.layer_norm(q, (hd,), params["q_norm.weight"], params["q_norm.bias"])
    k = F.layer_norm(k, (hd,), params["k_norm.weight"], params["k_norm.bias"])
    K = plan.keep.numel()
    pack = lambda t: compact(plan, t.reshape(N, dim)).reshape(1, K, heads, hd).transpose(1, 2)
    qc, kc, vc = pack(q), pack(k), pack(v)
    bias = plan.key_log_mass[None, None, None, :].to(qc.dtype)
    o = F.scaled_dot_product_attention(qc, kc, vc, attn_mask=bias)       # [1, H, K, hd]
    o = o.transpose(1, 2).reshape(K, dim)
    y = F.linear(o, params["proj.weight"], params["proj.bias"])
    return restore(plan, y)


@torch.no_grad()
def step(tokens: torch.Tensor, params: dict, layout, heads: int = 16) -> torch.Tensor:
    """One benchmark step: plan + block.  tokens [N, dim] fp32."""
    plan = build_plan(tokens, layout)
    return block_forward(tokens, params, plan, heads)
