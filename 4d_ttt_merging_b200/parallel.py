"""Query-row sharding of the token-merged global attention over the GPUs of one node.

Each rank owns a contiguous run of frames, aligned to the planner's frame groups, so the
merge plan of a rank is exactly the restriction of the single-GPU plan (sources only take
supports inside their own frame group).  Per global layer a rank

  1. builds its plan (merge step) and projects its own tokens,
  2. compacts them and all-gathers the merged K and V ([K_local, C] bf16 each) and the
     log-mass vector ([K_local] fp32) — the only exchange of the layer.  With peer-mapped
     symmetric memory (PeerExchange) the compaction kernel itself stores every merged k|v
     row into all ranks' K|V buffers (posted NVLink writes overlapping the compaction)
     between two device barriers; otherwise the compaction is followed by an NCCL
     all_gather_into_tensor,
  3. runs mass-bias attention of its own compact queries over all merged keys,
  4. projects and restores its own tokens.

Ranks gather in rank order, which is the global compact order, so every rank attends over
the same key sequence as a single GPU would: results do not depend on the rank count.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["FrameShard", "frame_shard", "gather_merged", "agree_all", "PeerExchange", "ShardedGlobalBlock", "StepGraph",
           "shard_projection_plan", "ShardedProjection"]


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


def agree_all(ok: bool, group=None, device=None) -> bool:
    """True only when ``ok`` holds on every rank of the group (one MIN all-reduce), so that
    ranks whose local outcomes differ still take the same collective path."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(int(flag.item()))


class PeerExchange:
    """The merged-K/V and log-mass all-gather of the sharded block over peer-mapped memory.

    One symmetric allocation per GPU (PyTorch symmetric memory: the same-sized buffer on every
    GPU, mapped into every rank's address space) holds this rank's compacted q|k|v rows, its
    log-mass vector and the full rank-ordered K|V buffer.

    Fused form (what ShardedGlobalBlock uses): `begin` is a device barrier (every rank has
    finished reading its previous full buffer and published its log-mass); the compaction
    kernel then stores every merged k|v row into all ranks' full buffers itself (`kv_peers`:
    posted NVLink writes, or one multicast store per row part when opted in); `finish` reads
    every rank's log-mass with `vb200_peer_gather` and ends with a second barrier (all writes
    landed).  Unfused form: `exchange` pushes the finished rows with `vb200_peer_push` between
    the same two barriers.  Ranks must have the same number of merged rows.

    The barriers are this library's own (`vb200_peer_barrier`): each rank stores an epoch into
    its slot of every rank's signal pad (two pads, one per barrier, at the head of the
    allocation) and waits for every slot of its own pad.  A wait gives up after
    BARRIER_TIMEOUT_MS: the kernel sets device error bit 0 and returns, so a rank that never
    arrives leaves the others with an error the host reads (`device_error_flags`) and a usable
    CUDA context."""

    BARRIER_TIMEOUT_MS = 60_000
    CHANNELS = 2  # begin / finish

    def __init__(self, group, rows: int, C: int, dtype: torch.dtype, device: torch.device):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _clib
        self.rows, self.C = rows, C
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.es = es = torch.empty(0, dtype=dtype).element_size()
        up = lambda n: -(-n // 256) * 256
        pad_bytes = up(self.CHANNELS * self.world * 4)
        packed_bytes, lm_bytes = up(rows * 3 * C * es), up(rows * 4)
        kv_bytes = self.world * rows * 2 * C * es
        self.buf = symm_mem.empty(pad_bytes + packed_bytes + lm_bytes + kv_bytes, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.pads = self.buf[:pad_bytes].view(torch.int32)
        self.pads.zero_()
        self.epoch = torch.zeros(self.CHANNELS, dtype=torch.int32, device=device)
        p_off, lm_off = pad_bytes, pad_bytes + packed_bytes
        self.packed = self.buf[p_off:p_off + rows * 3 * C * es].view(dtype).view(rows, 3 * C)
        self.log_mass = self.buf[lm_off:lm_off + rows * 4].view(torch.float32)
        kv_off = lm_off + lm_bytes
        self.kv = self.buf[kv_off:kv_off + kv_bytes].view(dtype).view(self.world * rows, 2 * C)
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        u64 = ctypes.c_uint64 * self.world
        self._kv_dst = u64(*[p + kv_off for p in ptrs])
        self._lm_src = u64(*[p + lm_off for p in ptrs])
        self._pad = [u64(*[p + ch * self.world * 4 for p in ptrs]) for ch in range(self.CHANNELS)]
        # every rank's pads are zero before any rank signals
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self.log_mass_all = torch.empty(self.world * rows, dtype=torch.float32, device=device)
        self._lib, self._clib = _clib.lib(), _clib
        # multicast (NVLS) address of the K|V region when the allocation is bound to a multicast
        # object and VB200_PEER_MULTICAST=1.  Off by default: on 8 B200s one multimem store per
        # row part measured slower than one posted store per rank (0.54 vs 0.49 ms per config-2
        # step).
        mc = 0
        if os.environ.get("VB200_PEER_MULTICAST", "0") == "1":
            mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)  # 0: no multicast object
        self._kv_mc = (ctypes.c_uint64 * 1)(mc + kv_off) if mc else None

    @property
    def multicast(self) -> bool:
        return self._kv_mc is not None

    def kv_peers(self):
        """Destinations of this rank's merged k|v rows for `compact_qkv(kv_peers=...)`: every
        rank's full K|V buffer at this rank's row offset (through the multicast address when
        there is one, else one pointer per rank)."""
        if self._kv_mc is not None:
            return self._kv_mc, self.world, self.rank * self.rows, 2 * self.C, 1
        return self._kv_dst, self.world, self.rank * self.rows, 2 * self.C, 0

    def barrier(self, channel: int):
        """Cross-GPU barrier on the current stream (bounded; see the class docstring)."""
        stream = self._clib.stream_of(self.epoch.device)
        self._clib.check(self._lib.vb200_peer_barrier(self._pad[channel], self.world, self.rank,
                                                      self.epoch[channel:].data_ptr(),
                                                      self.BARRIER_TIMEOUT_MS * 1_000_000, stream), "peer_barrier")

    def begin(self):
        """Device barrier before the fused compaction writes into other ranks' buffers: every
        rank has finished reading its previous full K|V buffer and has published log_mass."""
        self.barrier(0)

    def finish(self):
        """After the fused compaction: gather every rank's log-mass, then a device barrier (all
        ranks' k|v writes have landed).  -> (kv, log_mass) in rank order."""
        stream = self._clib.stream_of(self.kv.device)
        rows = self.rows
        self._clib.check(self._lib.vb200_peer_gather(self._lm_src, self.world, 1, rows * 4, rows * 4,
                                                     self.log_mass_all.data_ptr(), rows * 4, stream), "peer_gather")
        self.barrier(1)
        return self.kv, self.log_mass_all

    def exchange(self):
        """Unfused form: -> (kv [world*rows, 2C], log_mass [world*rows]) in rank order, on the
        current stream, from this rank's compacted rows in `packed`."""
        C, es, rows = self.C, self.es, self.rows
        stream = self._clib.stream_of(self.kv.device)
        self.barrier(0)
        self._clib.check(self._lib.vb200_peer_push(self.packed.data_ptr() + C * es, rows, 3 * C * es, 2 * C * es,
                                                   self._kv_dst, self.world, self.rank * rows, 2 * C * es, stream),
                         "peer_push")
        self._clib.check(self._lib.vb200_peer_gather(self._lm_src, self.world, 1, rows * 4, rows * 4,
                                                     self.log_mass_all.data_ptr(), rows * 4, stream), "peer_gather")
        self.barrier(1)
        return self.kv, self.log_mass_all


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
        self._xchg = None   # PeerExchange (world > 1, CUDA), built on the first step
        self._xchg_failed = False
        self._side = None   # side stream of the qkv GEMM

    def _ev(self, name):
        """Start a phase timer on the current stream (phases on different streams overlap)."""
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

    def _exchange(self, rows: int, C: int, dtype: torch.dtype, device: torch.device):
        """The PeerExchange for this shape (built collectively on first use: every rank reaches
        this point with the same rows), or None where peer-mapped memory is unavailable (then
        the NCCL all-gather is used)."""
        if self._xchg_failed or device.type != "cuda":
            return None
        x = self._xchg
        if x is None or x.rows != rows or x.C != C or x.packed.dtype != dtype:
            group = self.group if self.group is not None else dist.group.WORLD
            err = None
            try:
                x = PeerExchange(group, rows, C, dtype, device)
            except (RuntimeError, ImportError) as e:  # e.g. no CUDA virtual-memory IPC on this system
                x, err = None, e
            # every rank takes the same path: peer memory only where it worked on all of them
            if not agree_all(x is not None, group, device):
                import warnings
                warnings.warn(f"peer-memory exchange unavailable ({err or 'on another rank'}); using NCCL all-gather")
                self._xchg_failed, self._xchg = True, None
                return None
            self._xchg = x
        return x

    def plan(self, tokens: torch.Tensor):
        from .planners import build_uniform_convex_plan
        return build_uniform_convex_plan(tokens, frames=self.shard.frames, tokens_per_frame=self.tokens_per_frame,
                                         patch_token_start=self.patch_token_start, merge_factor=self.merge_factor,
                                         group_frames=self.group_frames)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        from .ops import mass_bias_attention, qkv_head_stats
        attn = self.attn
        H = attn.num_heads
        if self._ln is None and attn.q_norm is not None:
            from .attention_block import _ln_params
            self._ln = _ln_params(attn.q_norm, attn.k_norm)
        lw, lb, eps = self._ln if self._ln is not None else (None, None, 1e-5)
        stats = None
        # The plan (a chain of small kernels) and the qkv GEMM both read only the tokens: the
        # GEMM runs on a side stream, concurrently with the plan, and joins before compaction.
        cur = torch.cuda.current_stream(tokens.device) if tokens.is_cuda else None
        if cur is not None:
            if self._side is None or self._side.device != tokens.device:
                self._side = torch.cuda.Stream(tokens.device)
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                e = self._ev("qkv_gemm")
                qkv = attn.qkv_projection(tokens)
                # the q/k LayerNorm statistics need only the GEMM's output: computed here, under
                # the plan's kernels, instead of at the head of the compaction
                if lw is not None:
                    stats = qkv_head_stats(qkv, eps)
                self._end(e)
        e = self._ev("merge")
        plan = self.plan(tokens)
        self._end(e)
        if cur is None:
            e = self._ev("qkv_gemm")
            qkv = attn.qkv_projection(tokens)
            self._end(e)
        else:
            cur.wait_stream(self._side)
            qkv.record_stream(cur)
            if stats is not None:
                stats.record_stream(cur)
        B, N, C3 = qkv.shape
        C = C3 // 3
        e = self._ev("compact")
        xchg = self._exchange(plan.kept_tokens, C, qkv.dtype, qkv.device) if self.world > 1 else None
        log_mass = plan.key_log_mass.reshape(-1)
        if xchg is not None:
            # fused all-gather: the compaction stores every merged k|v row into all ranks'
            # K|V buffers, between two device barriers
            xchg.log_mass.copy_(log_mass)
            xchg.begin()
            packed = plan.compact_qkv(qkv[0], lw, lb, eps, pool_mask=0b111, out=xchg.packed,
                                      kv_peers=xchg.kv_peers(), stats=stats)
            self._end(e)
            e = self._ev("all_gather")
            kv, log_mass = xchg.finish()
            self._end(e)
        else:
            packed = plan.compact_qkv(qkv[0], lw, lb, eps, pool_mask=0b111, stats=stats)  # [K_local, 3C]: q|k|v
            self._end(e)
            kv = packed[:, C:]
            if self.world > 1:
                e = self._ev("all_gather")
                kv, log_mass = gather_merged([kv, log_mass], self.group)
                self._end(e)
        K_local = packed.shape[0]
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


class StepGraph:
    """One `ShardedGlobalBlock.step` over a fixed input buffer, recorded as a CUDA graph.

    A step is some twenty kernels, several of them only a few microseconds long on a rank's
    share of the frames; launched one by one from Python the host becomes the bottleneck and
    the GPU idles between kernels.  Replaying the recorded graph submits the whole step at
    once.  The caller refills `tokens` (same shape, dtype and address) before each `replay()`;
    the result lands in `out`, a buffer owned by the graph that the next replay overwrites.

    Recording runs `warmup` eager steps first on a side stream (they create the cuBLAS handle,
    the peer-exchange buffers, cached plan tables), then records one step.  With world > 1
    every rank must construct its StepGraph at the same point: the recorded step contains the
    exchange's cross-GPU barriers.  `pool` lets several graphs that never run concurrently
    share one memory pool (`torch.cuda.graph_pool_handle()`).  `launches` is the number of
    this library's kernels in one replay."""

    def __init__(self, block: ShardedGlobalBlock, tokens: torch.Tensor, warmup: int = 2, pool=None):
        from . import _clib
        self.block, self.tokens = block, tokens
        dev = tokens.device
        timers, block.timers = block.timers, None
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    block.step(tokens)
            torch.cuda.current_stream(dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            n0 = _clib.lib().vb200_launch_count()
            with torch.cuda.graph(self.graph, pool=pool):
                self.out = block.step(tokens)
            self.launches = int(_clib.lib().vb200_launch_count() - n0)
        finally:
            block.timers = timers

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def release(self) -> None:
        """Drop the graph (do this before destroying the process group)."""
        self.graph = None
        self.out = None


def shard_projection_plan(keep: torch.Tensor, source: torch.Tensor, parent: torch.Tensor, weights: torch.Tensor,
                          N: int, world: int, rank: int) -> dict:
    """This rank's share of a one-GPU projection plan over N tokens: tokens [t0, t1) with
    t_r = r * N // world, the merged rows whose keep token lies there ([m0, m1)) and the sources
    that lie there ([s0, s1)); keep and source must be ascending original token ids (as the
    reference's plans are).  Returns the bounds, every rank's owned merged-row count, and the
    local keep / source ids (relative to t0) with the sources' GLOBAL parents and weights."""
    keep = keep.reshape(-1)
    source = source.reshape(-1)
    parent = parent.reshape(source.numel(), -1)
    weights = weights.reshape(source.numel(), -1)
    cuts = torch.tensor([r * N // world for r in range(world + 1)], dtype=keep.dtype, device=keep.device)
    mcut = torch.searchsorted(keep, cuts).tolist()
    scut = torch.searchsorted(source, cuts).tolist()
    t0, t1 = rank * N // world, (rank + 1) * N // world
    m0, m1, s0, s1 = mcut[rank], mcut[rank + 1], scut[rank], scut[rank + 1]
    return dict(t0=t0, t1=t1, m0=m0, m1=m1, s0=s0, s1=s1,
                owned_counts=[mcut[r + 1] - mcut[r] for r in range(world)],
                keep_local=(keep[m0:m1] - t0).contiguous(), source_local=(source[s0:s1] - t0).contiguous(),
                parent_local=parent[s0:s1].to(torch.int64).contiguous(),
                weights_local=weights[s0:s1].to(torch.float32).contiguous())


class ShardedProjection:
    """The top-4 projection of one large plan (config 5: a million tokens whose sources take
    parents anywhere among the merged rows) sharded by query rows over the ranks of `group`.

    Rank r holds tokens [r N / R, (r + 1) N / R) and owns the merged rows whose keep token lies
    there.  ``compact`` runs the deterministic scatter over the rank's own sources into fp32
    partial numerators of ALL merged rows (vb200_proj_scatter_numerators), sends each owner its
    rows with one NCCL all_to_all_single (data only; the partial sums are exact fp32 values of a
    fixed order), and the owner adds its keep row and the ranks' partials in rank order and
    divides by the global mass (vb200_rank_reduce_rows): the result does not depend on timing
    and equals the one-GPU compact up to the fp32 summation order of each merged row (the
    one-GPU kernel sums a row's entries in source order in one chain; here per rank, then
    across ranks).  ``restore`` all-gathers the merged rows (rank order = compact order) and
    runs the gather for the rank's own tokens.  ``normalizer`` is the global mass [M] (from the
    whole plan).  Reference: the one-GPU compact / restore of token_merging.py:343-370,
    :285-341; the reference has no multi-GPU form of them."""

    def __init__(self, keep: torch.Tensor, source: torch.Tensor, parent: torch.Tensor, weights: torch.Tensor,
                 normalizer: torch.Tensor, N: int, group=None):
        from .ops import build_plan_csr
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        sh = shard_projection_plan(keep, source, parent, weights, N, self.world, self.rank)
        self.__dict__.update(sh)
        self.M = keep.numel()
        self.tokens = self.t1 - self.t0
        self.normalizer = normalizer.reshape(-1)[self.m0:self.m1].to(torch.float32).contiguous()
        self.csr = build_plan_csr(self.parent_local, self.weights_local, self.M, src_rows=self.source_local)
        self._hot = None

    def compact(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local [tokens, C] (this rank's token rows) -> the owned merged rows [m1 - m0, C]."""
        from . import _clib as C
        C.require_cuda(x_local, "ShardedProjection.compact")
        if x_local.ndim != 2 or x_local.shape[0] != self.tokens or x_local.stride(-1) != 1:
            raise ValueError(f"x_local must be [{self.tokens}, C] with unit channel stride")
        Cd, dev = x_local.shape[1], x_local.device
        lib, stream = C.lib(), C.stream_of(dev)
        numer = torch.empty((self.M, Cd), device=dev, dtype=torch.float32)
        n_entries = self.csr.entry_src.numel()
        ws_bytes = lib.vb200_proj_scatter_workspace_size(self.M, n_entries, Cd)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        rc = lib.vb200_proj_scatter_numerators(
            C.dtype_code(x_local.dtype), x_local.data_ptr(), x_local.shape[0], x_local.stride(0), self.M,
            self.csr.corners, self.csr.seg_offsets.data_ptr(), self.csr.entry_src.data_ptr(),
            self.csr.entry_w.data_ptr(), numer.data_ptr(), Cd, n_entries, ws.data_ptr(), ws_bytes, stream)
        C.check(rc, "proj_scatter_numerators")
        owned = self.m1 - self.m0
        if self.world > 1:
            recv = torch.empty((self.world * owned, Cd), device=dev, dtype=torch.float32)
            dist.all_to_all_single(recv, numer, output_split_sizes=[owned] * self.world,
                                   input_split_sizes=self.owned_counts, group=self.group)
        else:
            recv = numer
        out = torch.empty((owned, Cd), device=dev, dtype=x_local.dtype)
        rc = lib.vb200_rank_reduce_rows(
            C.dtype_code(x_local.dtype), recv.data_ptr(), self.world, owned, Cd, x_local.data_ptr(),
            x_local.shape[0], x_local.stride(0), self.keep_local.data_ptr(), self.normalizer.data_ptr(),
            out.data_ptr(), out.stride(0), stream)
        C.check(rc, "rank_reduce_rows")
        return out

    def restore(self, y_owned: torch.Tensor) -> torch.Tensor:
        """y_owned [m1 - m0, C] (this rank's merged rows) -> this rank's token rows [tokens, C]."""
        from . import _clib as C
        from .token_plan import HOT_GATHER_MIN_REFERENCES
        C.require_cuda(y_owned, "ShardedProjection.restore")
        if len(set(self.owned_counts)) != 1:
            raise ValueError("restore needs the same number of merged rows on every rank")
        y_owned = y_owned.contiguous()
        (full,) = gather_merged([y_owned], self.group) if self.world > 1 else (y_owned,)
        Cd, dev = y_owned.shape[1], y_owned.device
        lib, stream = C.lib(), C.stream_of(dev)
        code = C.dtype_code(y_owned.dtype)
        out = torch.empty((self.tokens, Cd), device=dev, dtype=y_owned.dtype)
        S, corners = self.parent_local.shape
        if self.keep_local.numel() + S != self.tokens:
            out.zero_()
        # the rank's own kept tokens: straight copies of its merged rows
        rc = lib.vb200_proj_gather(code, full[self.m0:self.m1].data_ptr(), Cd, self.keep_local.data_ptr(),
                                   self.keep_local.numel(), None, None, None, 0, corners, out.data_ptr(), Cd,
                                   self.tokens, Cd, 0, stream)
        C.check(rc, "proj_gather (keep rows)")
        if S == 0:
            return out
        # its sources: weighted sums of merged rows of every rank
        args = (code, full.data_ptr(), Cd, None, self.M, self.source_local.data_ptr(), self.parent_local.data_ptr(),
                self.weights_local.data_ptr(), S, corners, out.data_ptr(), Cd, self.tokens, Cd)
        if self.parent_local.numel() >= HOT_GATHER_MIN_REFERENCES:
            if self._hot is None or self._hot[0] != (Cd, y_owned.dtype):
                from .ops import plan_hot_rows
                cap = lib.vb200_proj_gather_hot_capacity(code, Cd)
                self._hot = ((Cd, y_owned.dtype), plan_hot_rows(self.csr, cap))
            hot_rows, hot_slot, n_hot, max_hot = self._hot[1]
            rc = lib.vb200_proj_gather_hot(*args, hot_rows.data_ptr(), hot_slot.data_ptr(), n_hot.data_ptr(), max_hot,
                                           stream)
            C.check(rc, "proj_gather_hot (sources)")
        else:
            rc = lib.vb200_proj_gather(*args, 0, stream)
            C.check(rc, "proj_gather (sources)")
        return out
