"""Reference-shaped operators of the token-merged global-attention path, backed by the
sm_100a kernels of ``libvggt_b200.so``.

Each function keeps the signature, argument meaning and exception types of the reference
function it replaces (paths inside shuang-yang18/4D_TTT_merging):

* ``mass_bias_attention``            vggt_omega/models/mass_bias_attention.py:85-129
* ``streaming_top4``                 vggt_omega/models/sparse_convex_kernels.py:309-329
* ``four_support_projected_gradient`` sparse_convex_kernels.py:283-296
* ``four_support_active_set``        sparse_convex_kernels.py:332-353
* ``deterministic_weighted_normalizer`` vggt_omega/models/token_merging.py:40-59

plus the internal operators the plans and planners use (row normalisation, similarity top-k,
plan CSR).  Nothing here computes on the CPU: every function raises ``RuntimeError`` for
non-CUDA tensors.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _clib as C

__all__ = [
    "mass_bias_attention",
    "mass_bias_attention_into",
    "streaming_top4",
    "similarity_topk",
    "merge_argmax",
    "four_support_projected_gradient",
    "four_support_active_set",
    "deterministic_weighted_normalizer",
    "row_normalize_bf16",
    "row_gather",
    "head_layernorm",
    "qkv_head_stats",
    "PlanCSR",
    "build_plan_csr",
]


def _tma_ready(t: torch.Tensor) -> bool:
    """TMA needs a unit channel stride, 16-byte aligned base and 16-byte multiple strides."""
    if t.stride(-1) != 1:
        return False
    es = t.element_size()
    if t.data_ptr() % 16:
        return False
    return all((s * es) % 16 == 0 for s, n in zip(t.stride()[:-1], t.shape[:-1]) if n > 1)


def mass_bias_attention_into(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             log_key_mass: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
    """Write softmax(q k^T / sqrt(64) + log_key_mass) v into ``out`` (same dtype as q, any
    [B,H,Nq,64] strides with unit channel stride).  q, k, v share one dtype; no casting."""
    B, H, Nq, D = q.shape
    Nk = k.shape[-2]
    dt = C.dtype_code(q.dtype)
    if dt != C.F32:
        q = q if _tma_ready(q) else q.contiguous()
        k = k if _tma_ready(k) else k.contiguous()
        v = v if _tma_ready(v) else v.contiguous()
    else:
        q, k, v = (t if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(s % 4 == 0 for s in t.stride()[:-1])
                   else t.contiguous() for t in (q, k, v))
    bias = None
    bias_dt = C.F32
    if log_key_mass is not None:
        bias = log_key_mass.reshape(-1)
        if bias.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            bias = bias.float()
        bias = bias.contiguous()
        bias_dt = C.dtype_code(bias.dtype)
    lib = C.lib()
    ws_bytes = lib.vb200_mass_bias_attention_split_workspace_size(B, H, Nq, Nk)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    rc = lib.vb200_mass_bias_attention(
        dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), C.ptr(bias), bias_dt, out.data_ptr(),
        B, H, Nq, Nk, D, C.strides3(q), C.strides3(k), C.strides3(v), C.strides3(out),
        ws.data_ptr(), ws_bytes, C.stream_of(q.device),
    )
    C.check(rc, "mass_bias_attention")
    return out


def mass_bias_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        log_key_mass: torch.Tensor) -> torch.Tensor:
    """Compute softmax(QK^T/sqrt(d) + log_key_mass)V exactly (head_dim 64).

    Same contract as the reference: 4-D [batch, heads, tokens, 64] inputs, ``log_key_mass``
    with one entry per key (rounded to q's dtype), fp32 q/k/v cast to bf16 under bf16
    autocast, output in q's (possibly cast) dtype.  The output is returned as a
    [B, H, Nq, 64] view of a token-major [B, Nq, H, 64] buffer, so the caller's
    ``transpose(1, 2).reshape(B, Nq, H*64)`` is free.
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k and v must be [batch, heads, tokens, channels]")
    if q.shape[-1] != 64 or k.shape[-1] != 64 or v.shape[-1] != 64:
        raise ValueError("the initial fused kernel supports head_dim=64 only")
    if k.shape != v.shape or q.shape[:2] != k.shape[:2]:
        raise ValueError("incompatible q/k/v shapes")
    C.require_cuda(q, "mass_bias_attention")
    autocast_bf16 = bool(
        torch.is_autocast_enabled("cuda") and q.dtype == torch.float32
        and torch.get_autocast_dtype("cuda") == torch.bfloat16
    )
    if autocast_bf16:
        q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
    if q.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported dtype {q.dtype}")
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    if log_key_mass is None:
        bias = None
    else:
        bias = log_key_mass.reshape(-1)
        if bias.numel() != k.shape[-2]:
            raise ValueError("log_key_mass length does not match key tokens")
        if bias.device != q.device:
            bias = bias.to(q.device)
    B, H, Nq, D = q.shape
    out = torch.empty((B, Nq, H, D), device=q.device, dtype=q.dtype).transpose(1, 2)
    return mass_bias_attention_into(q, k, v, bias, out)


def similarity_topk(query: torch.Tensor, basis: torch.Tensor, k: int, *,
                    query_begin: torch.Tensor | None = None,
                    basis_begin: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Row top-k (k = 1, 4 or 16) of bf16_round(query @ basis.T) on tcgen05, ties to the lower
    index.  query [R, D] and basis [Nb, D] are bf16 with D % 64 == 0.  With group tables
    (host int64 [G+1] each) query rows [qb[g], qb[g+1]) are ranked only against basis rows
    [bb[g], bb[g+1]).  Returns (values fp32 [R, k], indices int64 [R, k])."""
    C.require_cuda(query, "similarity_topk")
    if k not in (1, 4, 16):
        raise ValueError("k must be 1, 4 or 16")
    if query.ndim != 2 or basis.ndim != 2 or query.shape[1] != basis.shape[1]:
        raise ValueError("query [R,D] and basis [N,D] are required")
    query = query.to(torch.bfloat16)
    basis = basis.to(torch.bfloat16)
    if not _tma_ready(query):
        query = query.contiguous()
    if not _tma_ready(basis):
        basis = basis.contiguous()
    R, D = query.shape
    Nb = basis.shape[0]
    values = torch.empty((R, k), device=query.device, dtype=torch.float32)
    indices = torch.empty((R, k), device=query.device, dtype=torch.int64)
    groups = 1
    if query_begin is not None:
        groups = query_begin.numel() - 1
        query_begin = torch.as_tensor(query_begin, dtype=torch.int64, device="cpu").contiguous()
        basis_begin = torch.as_tensor(basis_begin, dtype=torch.int64, device="cpu").contiguous()
    rc = C.lib().vb200_sim_topk(
        query.data_ptr(), query.stride(0), basis.data_ptr(), basis.stride(0), R, Nb, D, k,
        C.ptr(query_begin), C.ptr(basis_begin), groups, values.data_ptr(), indices.data_ptr(),
        C.stream_of(query.device),
    )
    C.check(rc, "similarity_topk")
    return values, indices


def streaming_top4(query: torch.Tensor, basis_t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Memory-bounded BF16 Top-4 without materializing ``query @ basis``.

    ``basis_t`` is the transposed basis [D, N] as in the reference; a transposed view of a
    row-major [N, D] basis is used without a copy."""
    if not query.is_cuda:
        raise RuntimeError("streaming_top4 requires CUDA")
    if query.ndim != 2 or basis_t.ndim != 2 or query.shape[1] != basis_t.shape[0]:
        raise ValueError("query [M,D] and transposed basis [D,N] are required")
    if basis_t.shape[1] < 4:
        raise ValueError("streaming Top-4 requires at least four bases")
    return similarity_topk(query, basis_t.t(), 4)


def merge_argmax(source_bf16: torch.Tensor, dest_bf16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(best fp32 [S], target int64 [S]) = (source @ dest.T).max(-1) over bf16-rounded scores
    (build_fastvggt_plan's bmm + max, token_merging.py:1106-1111)."""
    v, i = similarity_topk(source_bf16, dest_bf16, 1)
    return v[:, 0], i[:, 0]


def four_support_projected_gradient(gram: torch.Tensor, rhs: torch.Tensor, *, steps: int = 32) -> torch.Tensor:
    """Run the four-way simplex projected-gradient iterations (one thread per row)."""
    if gram.ndim != 3 or gram.shape[1:] != (4, 4) or rhs.shape != (len(gram), 4):
        raise ValueError("the fused convex solver requires [N,4,4] Gram and [N,4] rhs")
    if not gram.is_cuda:
        raise RuntimeError("four_support_projected_gradient requires CUDA")
    gram, rhs = gram.contiguous().float(), rhs.contiguous().float()
    out = torch.empty_like(rhs)
    rc = C.lib().vb200_four_support_projected_gradient(
        gram.data_ptr(), rhs.data_ptr(), out.data_ptr(), len(gram), int(steps), C.stream_of(gram.device))
    C.check(rc, "four_support_projected_gradient")
    return out


def four_support_active_set(gram: torch.Tensor, rhs: torch.Tensor, *, ridge: float = 1e-4) -> torch.Tensor:
    """Exact 15-active-set simplex least-squares solve (one thread per row)."""
    if not gram.is_cuda:
        raise RuntimeError("four_support_active_set requires CUDA")
    if gram.ndim != 3 or gram.shape[1:] != (4, 4) or rhs.shape != (len(gram), 4):
        raise ValueError("active-set solver requires [N,4,4] Gram and [N,4] rhs")
    gram, rhs = gram.contiguous().float(), rhs.contiguous().float()
    out = torch.empty_like(rhs)
    rc = C.lib().vb200_four_support_active_set(
        gram.data_ptr(), rhs.data_ptr(), out.data_ptr(), len(gram), float(ridge), C.stream_of(gram.device))
    C.check(rc, "four_support_active_set")
    return out


@dataclass
class PlanCSR:
    """Parent-grouped view of a weighted plan (see ``vb200_plan_csr_build``)."""

    seg_offsets: torch.Tensor  # int32 [M*corners+1]
    entry_src: torch.Tensor    # int32 [S*corners], token rows
    entry_w: torch.Tensor      # fp32 [S*corners]
    mass: torch.Tensor         # fp32 [M]
    log_mass: torch.Tensor     # fp32 [M]
    corners: int
    kept: int


def build_plan_csr(parent: torch.Tensor, weights: torch.Tensor, kept: int,
                   src_rows: torch.Tensor | None = None, groups=None) -> PlanCSR:
    """Group (source, corner) pairs by compact parent; parent/weights are [S, corners]
    (a leading batch dim of 1 is accepted).  ``groups`` = (q_begin, b_begin, max_rows): device
    int64 group tables of a plan whose sources [q_begin[g], q_begin[g+1]) only take parents in
    merged rows [b_begin[g], b_begin[g+1]); the CSR is then built in one launch
    (``vb200_plan_csr_build_grouped``), with the same result."""
    C.require_cuda(parent, "build_plan_csr")
    if parent.ndim == 3:
        parent, weights = parent[0], weights[0]
    if parent.shape != weights.shape:
        raise ValueError("parent ids and weights must have matching shapes")
    S, corners = parent.shape
    dev = parent.device
    parent = parent.to(torch.int64).contiguous()
    weights = weights.to(torch.float32).contiguous()
    if src_rows is not None:
        src_rows = src_rows.reshape(-1).to(torch.int64).contiguous()
    seg = torch.empty(kept * corners + 1, device=dev, dtype=torch.int32)
    esrc = torch.empty(max(S * corners, 1), device=dev, dtype=torch.int32)
    ew = torch.empty(max(S * corners, 1), device=dev, dtype=torch.float32)
    mass = torch.empty(max(kept, 1), device=dev, dtype=torch.float32)
    log_mass = torch.empty(max(kept, 1), device=dev, dtype=torch.float32)
    lib = C.lib()
    if groups is not None:
        q_begin, b_begin, max_rows, max_sources = groups
        rc = lib.vb200_plan_csr_build_grouped(
            parent.data_ptr(), weights.data_ptr(), C.ptr(src_rows), S, corners, kept, q_begin.data_ptr(),
            b_begin.data_ptr(), q_begin.numel() - 1, int(max_rows), int(max_sources), seg.data_ptr(),
            esrc.data_ptr(), ew.data_ptr(), mass.data_ptr(), log_mass.data_ptr(), C.stream_of(dev))
        C.check(rc, "build_plan_csr (grouped)")
    else:
        ws_bytes = lib.vb200_plan_csr_workspace_size(S, corners, kept)
        ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
        rc = lib.vb200_plan_csr_build(
            parent.data_ptr(), weights.data_ptr(), C.ptr(src_rows), S, corners, kept, seg.data_ptr(),
            esrc.data_ptr(), ew.data_ptr(), mass.data_ptr(), log_mass.data_ptr(), ws.data_ptr(), ws_bytes,
            C.stream_of(dev),
        )
        C.check(rc, "build_plan_csr")
    return PlanCSR(seg, esrc[: S * corners], ew[: S * corners], mass[:kept], log_mass[:kept], corners, kept)


def plan_hot_rows(csr: PlanCSR, max_hot: int):
    """The plan's most-referenced merged rows (at most ``max_hot``), chosen on the device from
    the CSR lengths (``vb200_plan_hot_rows``): -> (hot_rows int32 [max_hot], hot_slot int32 [M],
    n_hot int32 [1], max_hot), the staging table of ``vb200_proj_gather_hot``."""
    dev = csr.seg_offsets.device
    hot_rows = torch.empty(max(max_hot, 1), device=dev, dtype=torch.int32)
    hot_slot = torch.empty(max(csr.kept, 1), device=dev, dtype=torch.int32)
    n_hot = torch.empty(1, device=dev, dtype=torch.int32)
    rc = C.lib().vb200_plan_hot_rows(csr.seg_offsets.data_ptr(), csr.kept, csr.corners, int(max_hot),
                                     hot_rows.data_ptr(), hot_slot.data_ptr(), n_hot.data_ptr(), C.stream_of(dev))
    C.check(rc, "plan_hot_rows")
    return hot_rows, hot_slot, n_hot, int(max_hot)


def deterministic_weighted_normalizer(parent_compact: torch.Tensor, weights: torch.Tensor,
                                      kept_tokens: int) -> torch.Tensor:
    """Return physical-plus-source mass [1, K, 1] without atomic additions."""
    if parent_compact.shape != weights.shape or parent_compact.shape[0] != 1:
        raise ValueError("parent ids and weights must have matching [1,M,S] shapes")
    csr = build_plan_csr(parent_compact, weights, kept_tokens)
    return csr.mass.view(1, kept_tokens, 1)


def row_normalize_bf16(x: torch.Tensor, rows: torch.Tensor | None = None, eps: float = 1e-12,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """F.normalize(x[rows].float(), dim=-1, eps=eps).to(bfloat16) for a 2-D x; written into
    ``out`` ([len(rows), C] bf16, unit channel stride, 16-byte aligned rows) when given."""
    C.require_cuda(x, "row_normalize_bf16")
    if x.ndim != 2:
        raise ValueError("row_normalize_bf16 expects a 2-D tensor")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or (x.stride(0) * x.element_size()) % 16:
        x = x.contiguous()
    R = x.shape[0] if rows is None else rows.numel()
    if rows is not None:
        rows = rows.reshape(-1).to(device=x.device, dtype=torch.int64).contiguous()
    if out is None:
        out = torch.empty((R, x.shape[1]), device=x.device, dtype=torch.bfloat16)
    elif out.shape != (R, x.shape[1]) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError(f"row_normalize_bf16: out must be [{R}, {x.shape[1]}] bf16 with unit channel stride")
    rc = C.lib().vb200_row_normalize_bf16(
        C.dtype_code(x.dtype), x.data_ptr(), x.shape[0], x.stride(0), C.ptr(rows), R, x.shape[1], float(eps),
        out.data_ptr(), out.stride(0), C.stream_of(x.device))
    C.check(rc, "row_normalize_bf16")
    return out


def qkv_head_stats(qkv: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Per-head LayerNorm statistics of the q and k blocks of a [N, 3C] (or [1, N, 3C]) qkv
    buffer (``vb200_qkv_head_stats``), as a workspace for ``compact_qkv(..., stats=...)``."""
    x = qkv[0] if qkv.ndim == 3 else qkv
    C.require_cuda(x, "qkv_head_stats")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or (x.stride(0) * x.element_size()) % 16:
        x = x.contiguous()
    c = x.shape[1] // 3
    lib = C.lib()
    ws_bytes = lib.vb200_compact_qkv_workspace_size(x.shape[0], c)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    C.check(lib.vb200_qkv_head_stats(C.dtype_code(x.dtype), x.data_ptr(), x.shape[0], x.stride(0), c, float(eps),
                                     ws.data_ptr(), ws_bytes, C.stream_of(x.device)), "qkv_head_stats")
    return ws


def head_layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm over every 64-channel head of the rows of a 2-D bf16 / fp16 tensor
    (nn.LayerNorm(64) applied to [N, H, 64]); weight / bias [64]."""
    C.require_cuda(x, "head_layernorm")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or (x.stride(0) * x.element_size()) % 16:
        x = x.contiguous()
    w = weight.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    b = bias.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    rc = C.lib().vb200_head_layernorm(C.dtype_code(x.dtype), x.data_ptr(), x.shape[0], x.stride(0), x.shape[1],
                                      w.data_ptr(), b.data_ptr(), float(eps), out.data_ptr(), out.stride(0),
                                      C.stream_of(x.device))
    C.check(rc, "head_layernorm")
    return out


def row_gather(x: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = x[index[i]] for a 2-D x (rows of 16-byte multiples)."""
    C.require_cuda(x, "row_gather")
    if x.stride(-1) != 1 or x.data_ptr() % 16 or (x.stride(0) * x.element_size()) % 16:
        x = x.contiguous()
    index = index.reshape(-1).to(device=x.device, dtype=torch.int64).contiguous()
    if out is None:
        out = torch.empty((index.numel(), x.shape[1]), device=x.device, dtype=x.dtype)
    rc = C.lib().vb200_row_gather(
        C.dtype_code(x.dtype), x.data_ptr(), x.shape[0], x.stride(0), index.data_ptr(), index.numel(),
        out.data_ptr(), out.stride(0), x.shape[1], C.stream_of(x.device))
    C.check(rc, "row_gather")
    return out
