"""Token-plan types of the token-merged global attention, with the reductions on B200.

``TokenPlan`` mirrors vggt_omega/models/token_merging.py:143-196 (hard merge: mean pooling by
``inverse`` and gather restore) and ``WeightedBilinearTokenPlan`` mirrors
token_merging.py:253-426 (four-parent convex pooling, ``key_log_mass``, bilinear restore).
Field names, defaults and method signatures are the reference's, so the aggregator and the
attention layer use them unchanged.

What changes is how the reductions run: at construction each plan builds, on the device, a
parent-grouped CSR of its (source, corner) pairs (``vb200_plan_csr_build``).  ``compact`` is
then one segmented kernel per call (one warp per compact row, fixed summation order, no
atomics), ``restore`` one vectorised gather kernel.  ``TokenPlan.compact`` is therefore
deterministic, unlike the reference's atomic ``scatter_add_``.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _clib as C
from .ops import PlanCSR, build_plan_csr

__all__ = ["TokenPlan", "WeightedBilinearTokenPlan"]


def _rows_ready(t: torch.Tensor) -> bool:
    return (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
            and (t.stride(-2) * t.element_size()) % 16 == 0)


def _as_rows(value: torch.Tensor) -> torch.Tensor:
    """2-D [N, C] view of a [1, N, C] tensor with unit channel stride and aligned rows."""
    x = value[0]
    return x if _rows_ready(x) else x.contiguous()


def _scatter(x2d: torch.Tensor, keep: torch.Tensor | None, csr: PlanCSR, normalizer: torch.Tensor,
             rows_out: int) -> torch.Tensor:
    out = torch.empty((rows_out, x2d.shape[1]), device=x2d.device, dtype=x2d.dtype)
    lib = C.lib()
    n_entries = csr.entry_src.numel()
    ws_bytes = lib.vb200_proj_scatter_workspace_size(rows_out, n_entries, x2d.shape[1])
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x2d.device)
    rc = lib.vb200_proj_scatter(
        C.dtype_code(x2d.dtype), x2d.data_ptr(), x2d.shape[0], x2d.stride(0), C.ptr(keep), rows_out, csr.corners,
        csr.seg_offsets.data_ptr(), csr.entry_src.data_ptr(), csr.entry_w.data_ptr(),
        normalizer.data_ptr(), out.data_ptr(), out.stride(0), x2d.shape[1], n_entries, ws.data_ptr(), ws_bytes,
        C.stream_of(x2d.device),
    )
    C.check(rc, "proj_scatter")
    return out


# Restores with at least this many (source, corner) references stage the plan's most-referenced
# merged rows in shared memory (vb200_proj_gather_hot); smaller ones read every parent from
# global memory, where the merged table fits in L2 anyway.
HOT_GATHER_MIN_REFERENCES = 1 << 19


def _gather(y2d: torch.Tensor, keep: torch.Tensor, src: torch.Tensor | None, parent: torch.Tensor | None,
            weights: torch.Tensor | None, n_out: int, zero_fill: bool, hot=None) -> torch.Tensor:
    out = torch.empty((n_out, y2d.shape[1]), device=y2d.device, dtype=y2d.dtype)
    S = 0 if src is None else src.numel()
    corners = 4 if parent is None else parent.shape[-1]
    lib, stream = C.lib(), C.stream_of(y2d.device)
    if hot is None:
        rc = lib.vb200_proj_gather(
            C.dtype_code(y2d.dtype), y2d.data_ptr(), y2d.stride(0), keep.data_ptr(), keep.numel(),
            C.ptr(src), C.ptr(parent), C.ptr(weights), S, corners, out.data_ptr(), out.stride(0), n_out,
            y2d.shape[1], int(zero_fill), stream,
        )
        C.check(rc, "proj_gather")
        return out
    if zero_fill:
        out.zero_()
    hot_rows, hot_slot, n_hot, max_hot = hot
    rc = lib.vb200_proj_gather_hot(
        C.dtype_code(y2d.dtype), y2d.data_ptr(), y2d.stride(0), keep.data_ptr(), keep.numel(),
        C.ptr(src), C.ptr(parent), C.ptr(weights), S, corners, out.data_ptr(), out.stride(0), n_out,
        y2d.shape[1], hot_rows.data_ptr(), hot_slot.data_ptr(), n_hot.data_ptr(), max_hot, stream,
    )
    C.check(rc, "proj_gather_hot")
    return out


def _idx(t: torch.Tensor | None) -> torch.Tensor | None:
    return None if t is None else t.reshape(-1).to(torch.int64).contiguous()


@dataclass
class TokenPlan:
    """A compact-token map for one attention operation (hard merge).

    ``keep`` [B, K] original ids of the compact tokens, ``inverse`` [B, N] original -> compact
    index.  ``compact`` mean-pools every original token into ``inverse`` (only tokens whose
    ``pool_mask`` is set contribute); ``restore`` broadcasts a compact update back through
    ``inverse``."""

    keep: torch.Tensor
    inverse: torch.Tensor
    original_tokens: int
    pool_sources: bool = True
    pool_mask: torch.Tensor | None = None
    metadata: dict[str, float | int] = field(default_factory=dict)
    precomputed_qkv: torch.Tensor | None = None
    _csr: list = field(default=None, init=False, repr=False)
    _counts: list = field(default=None, init=False, repr=False)

    @property
    def kept_tokens(self) -> int:
        return self.keep.shape[1]

    @property
    def keep_ratio(self) -> float:
        return self.kept_tokens / self.original_tokens

    def _ensure_csr(self) -> None:
        if self._csr is not None:
            return
        csrs, counts = [], []
        for b in range(self.inverse.shape[0]):
            inverse = self.inverse[b].to(torch.int64).reshape(-1, 1)
            if self.pool_mask is None:
                contribution = torch.ones_like(inverse, dtype=torch.float32)
            else:
                contribution = self.pool_mask[b].reshape(-1, 1).to(torch.float32)
            csr = build_plan_csr(inverse, contribution, self.kept_tokens)
            csrs.append(csr)
            # mass = 1 + count for 0/1 contributions, exact in fp32
            counts.append(csr.mass - 1.0)
        self._csr, self._counts = csrs, counts

    def compact(self, value: torch.Tensor, *, merge: bool = True) -> torch.Tensor:
        if self.kept_tokens == self.original_tokens:
            return value
        C.require_cuda(value, "TokenPlan.compact")
        if not merge and self.pool_mask is None:
            return torch.stack([self._gather_rows(value[b], self.keep[b]) for b in range(value.shape[0])])
        self._ensure_csr()
        outs = []
        for b in range(value.shape[0]):
            x = value[b]
            x = x if _rows_ready(x) else x.contiguous()
            outs.append(_scatter(x, None, self._csr[b], self._counts[b], self.kept_tokens))
        return torch.stack(outs)

    def restore(self, value: torch.Tensor) -> torch.Tensor:
        if self.kept_tokens == self.original_tokens:
            return value
        C.require_cuda(value, "TokenPlan.restore")
        return torch.stack([self._gather_rows(value[b], self.inverse[b]) for b in range(value.shape[0])])

    @staticmethod
    def _gather_rows(x: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
        from .ops import row_gather
        return row_gather(x, index)


@dataclass
class WeightedBilinearTokenPlan:
    """Compact attention plan with four-way, information-preserving pooling.

    Each removed source contributes its Q/K/V to its four physical parents with
    ``source_pool_weights`` and recovers its post-attention update from them with
    ``source_restore_weights``.  ``normalizer`` [1, K, 1] is the physical-plus-source mass and
    ``key_log_mass`` its log, the per-key attention bias."""

    keep: torch.Tensor
    source_original: torch.Tensor
    source_parent_compact: torch.Tensor
    source_pool_weights: torch.Tensor
    source_restore_weights: torch.Tensor
    original_tokens: int
    normalizer: torch.Tensor
    pool_sources: bool = True
    preserve_queries: bool = False
    preserve_destination_keys: bool = False
    dense_special_queries: bool = False
    special_query_original: torch.Tensor | None = None
    special_query_compact: torch.Tensor | None = None
    pool_source_content: bool = True
    precomputed_qkv: torch.Tensor | None = None
    source_query_correction: bool = False
    source_attention_output: torch.Tensor | None = None
    key_log_mass: torch.Tensor | None = None
    query_keep: torch.Tensor | None = None
    query_source_original: torch.Tensor | None = None
    query_source_parent_compact: torch.Tensor | None = None
    query_restore_weights: torch.Tensor | None = None
    compact_mlp: bool = False
    metadata: dict[str, float | int] = field(default_factory=dict)
    # Optional prebuilt parent-grouped CSR of (source_parent_compact, source_pool_weights)
    # with token rows from source_original; built at construction when absent.
    csr: PlanCSR | None = field(default=None, repr=False)
    _keep_flat: torch.Tensor | None = field(default=None, init=False, repr=False)
    _normalizer_flat: torch.Tensor | None = field(default=None, init=False, repr=False)

    def __post_init__(self) -> None:
        if self.source_parent_compact.shape[0] != 1:
            raise ValueError("weighted bilinear plans require one shared inference mapping")
        C.require_cuda(self.keep, "WeightedBilinearTokenPlan")
        self._keep_flat = _idx(self.keep)
        self._normalizer_flat = self.normalizer.reshape(-1).to(torch.float32).contiguous()
        self._hot = None
        if self.csr is None:
            self.csr = build_plan_csr(
                self.source_parent_compact[0], self.source_pool_weights[0], self.kept_tokens,
                src_rows=self.source_original.reshape(-1),
            )

    @property
    def kept_tokens(self) -> int:
        return self.keep.shape[1]

    @property
    def keep_ratio(self) -> float:
        return self.kept_tokens / self.original_tokens

    def compact(self, value: torch.Tensor, *, merge: bool = True) -> torch.Tensor:
        """Pool source Q/K/V mass into its four retained bilinear parents."""
        del merge
        C.require_cuda(value, "WeightedBilinearTokenPlan.compact")
        if value.shape[0] != 1:
            raise RuntimeError("weighted bilinear compaction currently supports inference batch size one")
        x = _as_rows(value)
        if self.source_original.shape[1] == 0 or not self.pool_source_content:
            from .ops import row_gather
            return row_gather(x, self._keep_flat).unsqueeze(0)
        return _scatter(x, self._keep_flat, self.csr, self._normalizer_flat, self.kept_tokens).unsqueeze(0)

    def compact_qkv(self, qkv: torch.Tensor, ln_weight: torch.Tensor | None = None,
                    ln_bias: torch.Tensor | None = None, eps: float = 1e-5,
                    pool_mask: int = 0b111, out: torch.Tensor | None = None, kv_peers=None,
                    stats: torch.Tensor | None = None) -> torch.Tensor:
        """Fused q/k LayerNorm + Q||K||V compaction of a [N, 3C] (or [1, N, 3C]) qkv buffer in
        one kernel (``vb200_compact_qkv``); returns [M, 3C].  ``ln_weight`` / ``ln_bias`` are
        [2, 64] fp32 (q then k) or None.  Bit t of ``pool_mask`` pools tensor t (q, k, v);
        a clear bit keeps the physical row only (compact_key semantics).  ``out``: an optional
        [M, 3C] destination (rows 16-byte aligned, unit channel stride), e.g. a buffer that other
        GPUs read.  ``kv_peers`` = (pointer array, world, row0, row_stride[, multicast]): also
        store the k|v part of every merged row into those peer-mapped [rows, 2C] buffers at row
        row0 + j (``vb200_compact_qkv_peer``, the fused all-gather of the sharded layer); with
        multicast set the array holds one multicast address covering every rank's buffer.
        ``stats``: the q/k LayerNorm statistics of this qkv already computed by
        ``ops.qkv_head_stats`` (e.g. on the qkv GEMM's stream); the call then runs the compaction
        alone."""
        x = qkv[0] if qkv.ndim == 3 else qkv
        C.require_cuda(x, "compact_qkv")
        if x.stride(-1) != 1 or x.data_ptr() % 16 or (x.stride(0) * x.element_size()) % 16:
            x = x.contiguous()
        c = x.shape[1] // 3
        if out is None:
            out = torch.empty((self.kept_tokens, 3 * c), device=x.device, dtype=x.dtype)
        elif (out.shape != (self.kept_tokens, 3 * c) or out.dtype != x.dtype or out.device != x.device
              or out.stride(-1) != 1):
            raise ValueError(f"compact_qkv: out must be [{self.kept_tokens}, {3 * c}] {x.dtype} on {x.device} "
                             f"with unit channel stride")
        if not self.pool_source_content or self.source_original.shape[1] == 0:
            pool_mask = 0
        lw = None if ln_weight is None else ln_weight.reshape(-1).to(torch.float32).contiguous()
        lb = None if ln_bias is None else ln_bias.reshape(-1).to(torch.float32).contiguous()
        csr = self.csr
        lib = C.lib()
        ws_bytes = lib.vb200_compact_qkv_workspace_size(x.shape[0], c) if lw is not None else 0
        if stats is not None and lw is not None:
            if stats.numel() * stats.element_size() < ws_bytes or stats.device != x.device:
                raise ValueError("compact_qkv: stats must come from ops.qkv_head_stats of this qkv")
            ws = stats
            pool_mask = int(pool_mask) | 8  # VB200_STATS_READY
        else:
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        args = (C.dtype_code(x.dtype), x.data_ptr(), x.shape[0], x.stride(0), c, C.ptr(lw), C.ptr(lb), float(eps),
                self._keep_flat.data_ptr(), self.kept_tokens, csr.corners, csr.seg_offsets.data_ptr(),
                csr.entry_src.data_ptr(), csr.entry_w.data_ptr(), self._normalizer_flat.data_ptr(), int(pool_mask),
                out.data_ptr(), out.stride(0))
        if kv_peers is None:
            rc = lib.vb200_compact_qkv(*args, ws.data_ptr(), ws_bytes, C.stream_of(x.device))
            C.check(rc, "compact_qkv")
        else:
            ptrs, world, row0, row_stride = kv_peers[:4]
            multicast = int(kv_peers[4]) if len(kv_peers) > 4 else 0
            rc = lib.vb200_compact_qkv_peer(*args, ptrs, int(world), multicast, int(row0), int(row_stride),
                                            ws.data_ptr(), ws_bytes, C.stream_of(x.device))
            C.check(rc, "compact_qkv_peer")
        return out

    def compact_key(self, value: torch.Tensor) -> torch.Tensor:
        """Keep physical keys unchanged for the Q-preserving KV-only path."""
        if not self.preserve_destination_keys:
            return self.compact(value)
        from .ops import row_gather
        return row_gather(_as_rows(value), self._keep_flat).unsqueeze(0)

    @property
    def query_kept_tokens(self) -> int:
        return self.kept_tokens if self.query_keep is None else self.query_keep.shape[1]

    def compact_query(self, value: torch.Tensor) -> torch.Tensor:
        if self.query_keep is None:
            return self.compact(value)
        from .ops import row_gather
        return row_gather(_as_rows(value), _idx(self.query_keep)).unsqueeze(0)

    def _hot_rows(self, value: torch.Tensor):
        """The staged-row table of the main restore (built once per plan and row width): the
        merged rows with the most references, chosen from the plan's CSR on the device."""
        c, dtype = value.shape[-1], value.dtype
        key = (c, dtype)
        if self._hot is None or self._hot[0] != key:
            from .ops import plan_hot_rows
            cap = C.lib().vb200_proj_gather_hot_capacity(C.dtype_code(dtype), c)
            self._hot = (key, plan_hot_rows(self.csr, cap))
        return self._hot[1]

    def _restore_with(self, value: torch.Tensor, keep: torch.Tensor, src: torch.Tensor | None,
                      parent: torch.Tensor | None, weights: torch.Tensor | None, main: bool = False) -> torch.Tensor:
        C.require_cuda(value, "WeightedBilinearTokenPlan.restore")
        y = _as_rows(value)
        keep = _idx(keep)
        has_src = src is not None and src.numel() > 0
        covered = keep.numel() + (src.numel() if has_src else 0)
        hot = None
        if main and has_src and parent.numel() >= HOT_GATHER_MIN_REFERENCES:
            hot = self._hot_rows(y)
        out = _gather(
            y, keep,
            _idx(src) if has_src else None,
            parent.reshape(-1, parent.shape[-1]).to(torch.int64).contiguous() if has_src else None,
            weights.reshape(-1, weights.shape[-1]).to(torch.float32).contiguous() if has_src else None,
            self.original_tokens,
            zero_fill=covered != self.original_tokens,
            hot=hot,
        )
        return out.unsqueeze(0)

    def restore(self, value: torch.Tensor) -> torch.Tensor:
        """Broadcast physical outputs and bilinearly recover source outputs."""
        if self.preserve_queries and value.shape[1] == self.original_tokens:
            return value
        if self.query_keep is not None:
            return self._restore_with(value, self.query_keep, self.query_source_original,
                                      self.query_source_parent_compact, self.query_restore_weights)
        if self.preserve_queries:
            if value.shape[1] != self.original_tokens:
                raise RuntimeError("Q-preserving KV compaction must produce one output per original query")
            return value
        if value.shape[0] != 1:
            raise RuntimeError("weighted bilinear compaction currently supports inference batch size one")
        return self._restore_with(value, self.keep, self.source_original, self.source_parent_compact,
                                  self.source_restore_weights, main=True)

    def restore_query(self, value: torch.Tensor) -> torch.Tensor:
        """Restore a tensor compacted with :meth:`compact_query`."""
        if self.query_keep is None:
            return self.restore(value)
        return self._restore_with(value, self.query_keep, self.query_source_original,
                                  self.query_source_parent_compact, self.query_restore_weights)
