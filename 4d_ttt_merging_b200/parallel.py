"""Query-row sharding of the token-merged global attention over the GPUs of one node.

Each rank owns a contiguous run of frames, aligned to the planner's frame groups, so the
merge plan of a rank is exactly the restriction of the single-GPU plan (sources only take
supports inside their own frame group).  Per global layer a rank

  1. builds its plan (merge step) and projects / compacts its own tokens (no exchange),
  2. all-gathers the merged K and V ([K_local, C] bf16 each) and the log-mass vector
     ([K_local] fp32) with NCCL — the only collective of the layer,
  3. runs mass-bias attention of its own compact queries over all merged keys,
  4. projects and restores its own tokens.

Ranks gather in rank order, which is the global compact order, so every rank attends over
the same key sequence as a single GPU would: results do not depend on the rank count.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["FrameShard", "frame_shard", "gather_merged", "ShardedGlobalBlock"]


@dataclass(frozen=True)
class FrameShard:
    rank: int
    world: int
    frame_begin: int
    frame_end: int
    tokens_per_frame: int

    @property
    def frames(self) -> int:
        return self.frame_end - self.frame_begin

    @property
    def token_begin(self) -> int:
        return self.frame_begin * self.tokens_per_frame

    @property
    def token_end(self) -> int:
        return self.frame_end * self.tokens_per_frame


def frame_shard(frames: int, tokens_per_frame: int, group_frames: int, world: int, rank: int) -> FrameShard:
    """Contiguous frame range of `rank`; every rank gets the same number of whole frame
    groups (so merged-token counts are equal across ranks and all-gathers are uniform)."""
    if frames % group_frames:
        raise ValueError("frames must be a multiple of group_frames")
    groups = frames // group_frames
    if groups % world:
        raise ValueError(f"{groups} frame groups cannot be split evenly over {world} ranks")
    per = groups // world * group_frames
    return FrameShard(rank, world, rank * per, (rank + 1) * per, tokens_per_frame)


def gather_merged(tensors: list[torch.Tensor], group=None) -> list[torch.Tensor]:
    """All-gather each [n, ...] tensor along dim 0 in rank order (one NCCL call each)."""
    world = dist.get_world_size(group)
    if world == 1:
        return tensors
    out = []
    for t in tensors:
        t = t.contiguous()
        full = torch.empty((world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(full, t, group=group)
        out.append(full)
    return out


class ShardedGlobalBlock:
    """One global-attention layer with a per-rank uniform convex plan (see module docstring).

    `attn` is a GlobalAttention; the tokens passed to `step` are this rank's frames,
    [1, frames_local * tokens_per_frame, dim]."""

    def __init__(self, attn, *, frames: int, tokens_per_frame: int, patch_token_start: int,
                 merge_factor: int = 4, group_frames: int = 4, world: int = 1, rank: int = 0, group=None):
        self.attn = attn
        self.shard = frame_shard(frames, tokens_per_frame, group_frames, world, rank)
        self.tokens_per_frame = tokens_per_frame
        self.patch_token_start = patch_token_start
        self.merge_factor = merge_factor
        self.group_frames = group_frames
        self.group = group
        self.world = world
        self.timers = None  # optional dict name -> list of (start, end) CUDA events
        self._ln = None     # fp32 q/k LayerNorm parameters, [2, 64] each

    def _ev(self, name):
        if self.timers is None:
            return None
        e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self.timers.setdefault(name, []).append(e)
        e[0].record()
        return e

    @staticmethod
    def _end(e):
        if e is not None:
            e[1].record()

    def plan(self, tokens: torch.Tensor):
        from .planners import build_uniform_convex_plan
        return build_uniform_convex_plan(tokens, frames=self.shard.frames, tokens_per_frame=self.tokens_per_frame,
                                         patch_token_start=self.patch_token_start, merge_factor=self.merge_factor,
                                         group_frames=self.group_frames)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        from .ops import mass_bias_attention
        attn = self.attn
        H = attn.num_heads
        e = self._ev("merge")
        plan = self.plan(tokens)
        self._end(e)
        e = self._ev("qkv_gemm")
        qkv = attn.qkv_projection(tokens)
        self._end(e)
        B, N, C3 = qkv.shape
        C = C3 // 3
        e = self._ev("compact")
        if self._ln is None and attn.q_norm is not None:
            from .attention_block import _ln_params
            self._ln = _ln_params(attn.q_norm, attn.k_norm)
        lw, lb, eps = self._ln if self._ln is not None else (None, None, 1e-5)
        packed = plan.compact_qkv(qkv[0], lw, lb, eps, pool_mask=0b111)  # [K_local, 3C]: q | k | v
        self._end(e)
        log_mass = plan.key_log_mass.reshape(-1)
        K_local = packed.shape[0]
        kv = packed[:, C:]
        if self.world > 1:
            e = self._ev("all_gather")
            kv, log_mass = gather_merged([kv, log_mass], self.group)
            self._end(e)
        e = self._ev("attention")
        view = lambda t: t.view(1, t.shape[0], H, C // H).transpose(1, 2)
        o = mass_bias_attention(view(packed[:, :C]), view(kv[:, :C]), view(kv[:, C:]), log_mass)
        self._end(e)
        e = self._ev("proj_gemm")
        y = attn.proj(o.transpose(1, 2).reshape(B, K_local, C))
        self._end(e)
        e = self._ev("restore")
        out = plan.restore(y)
        self._end(e)
        return out
