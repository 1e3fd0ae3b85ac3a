"""Multi-rank host logic of the sharded global block on CPU (two `gloo` ranks).

The GPU path of `parallel.ShardedGlobalBlock.step` is: per rank, plan + compact its own frames,
all-gather the merged K, V and log-mass in rank order, attend with its own compact queries
over all merged keys, project and restore its own tokens.  These tests check the pieces that
make that equal to the single-GPU block, using the numpy oracle for the math:
  * frame_shard gives every rank whole, contiguous frame groups;
  * gather_merged concatenates in rank order over a real process group;
  * planning each shard alone gives exactly the restriction of the global plan, and the
    gathered merged keys are the global merged keys in the global order, so the sharded block
    reproduces the single-process block row for row;
  * a rank that exits between steps makes the others' next exchange end with an error
    instead of a hang (failure detection on the host, no GPU involved).
"""
from __future__ import annotations

import datetime
import importlib
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO

FRAMES, TPF, SPECIAL, MERGE, GROUP = 8, 22, 2, 4, 2  # 4 frame groups of 44 tokens, 11 kept each
DIM, HEADS = 64, 2


def _pkg():
    import sys
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    return importlib.import_module("4d_ttt_merging_b200")


def _inputs():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((FRAMES * TPF, DIM)).astype(np.float32)
    params = {
        "qkv.weight": (rng.standard_normal((3 * DIM, DIM)) / 8).astype(np.float32),
        "qkv.bias": (rng.standard_normal(3 * DIM) / 8).astype(np.float32),
        "qkv.bias_mask": np.concatenate([np.ones(DIM), np.zeros(DIM), np.ones(DIM)]).astype(np.float32),
        "q_norm.weight": (1 + rng.standard_normal(DIM // HEADS) / 8).astype(np.float32),
        "q_norm.bias": (rng.standard_normal(DIM // HEADS) / 8).astype(np.float32),
        "k_norm.weight": (1 + rng.standard_normal(DIM // HEADS) / 8).astype(np.float32),
        "k_norm.bias": (rng.standard_normal(DIM // HEADS) / 8).astype(np.float32),
        "proj.weight": (rng.standard_normal((DIM, DIM)) / 8).astype(np.float32),
        "proj.bias": (rng.standard_normal(DIM) / 8).astype(np.float32),
    }
    return x, params


def _compact_parts(x, params, plan):
    """The per-rank half of the block: qkv projection, q/k LayerNorm, compaction (the merged
    q, k, v rows) and the log-mass of the merged keys (oracle math, fp64/fp32)."""
    from oracle import ref
    N = x.shape[0]
    hd = DIM // HEADS
    qkv = (x.astype(np.float64) @ params["qkv.weight"].T.astype(np.float64)
           + params["qkv.bias"] * params["qkv.bias_mask"]).reshape(N, 3, HEADS, hd)
    q = ref.layer_norm(qkv[:, 0], params["q_norm.weight"], params["q_norm.bias"]).reshape(N, DIM).astype(np.float32)
    k = ref.layer_norm(qkv[:, 1], params["k_norm.weight"], params["k_norm.bias"]).reshape(N, DIM).astype(np.float32)
    v = qkv[:, 2].reshape(N, DIM).astype(np.float32)
    args = (plan["keep"], plan["source"], plan["parent"], plan["weights"], plan["normalizer"])
    qc, kc, vc = (ref.compact(t, *args) for t in (q, k, v))
    log_mass = np.log(np.asarray(plan["normalizer"], np.float32)).astype(np.float32)
    return qc, kc, vc, log_mass


def _finish(x_rows, params, plan, qc, kc_all, vc_all, log_mass_all):
    """Attention of this rank's merged queries over all merged keys, projection, restore."""
    from oracle import ref
    hd = DIM // HEADS
    to_bh = lambda t: np.asarray(t, np.float64).reshape(1, -1, HEADS, hd).transpose(0, 2, 1, 3)
    o = ref.mass_bias_attention(to_bh(qc), to_bh(kc_all), to_bh(vc_all), log_mass_all)
    o = o.transpose(0, 2, 1, 3).reshape(-1, DIM)
    y = (o @ params["proj.weight"].T.astype(np.float64) + params["proj.bias"]).astype(np.float32)
    return ref.restore(y, plan["keep"], plan["source"], plan["parent"], plan["weights"], x_rows)


def _single_process(x, params):
    from oracle import pipeline
    layout = pipeline.uniform_layout(FRAMES, TPF, SPECIAL, MERGE, GROUP)
    plan = pipeline.convex_plan(x, layout)
    qc, kc, vc, lm = _compact_parts(x, params, plan)
    return plan, _finish(x.shape[0], params, plan, qc, kc, vc, lm)


def _rank_main(rank: int, world: int, init_file: str, out_dir: str):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        pkg = _pkg()
        from oracle import pipeline
        x, params = _inputs()
        shard = pkg.parallel.frame_shard(FRAMES, TPF, GROUP, world, rank)
        xs = x[shard.token_begin:shard.token_end]
        layout = pipeline.uniform_layout(shard.frames, TPF, SPECIAL, MERGE, GROUP)
        plan = pipeline.convex_plan(xs, layout)
        qc, kc, vc, lm = _compact_parts(xs, params, plan)
        kc_all, vc_all, lm_all = (t.numpy() for t in pkg.parallel.gather_merged(
            [torch.from_numpy(kc), torch.from_numpy(vc), torch.from_numpy(lm)]))
        y = _finish(xs.shape[0], params, plan, qc, kc_all, vc_all, lm_all)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), y=y, keep=plan["keep"] + shard.token_begin,
                 kc_all=kc_all, lm_all=lm_all)
    finally:
        dist.destroy_process_group()


def test_frame_shard_whole_groups():
    pkg = _pkg()
    shards = [pkg.parallel.frame_shard(32, 1029, 4, 4, r) for r in range(4)]
    assert [(s.frame_begin, s.frame_end) for s in shards] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    assert shards[2].token_begin == 16 * 1029 and shards[2].token_end == 24 * 1029
    assert all(s.frames % 4 == 0 for s in shards)
    with pytest.raises(ValueError, match="cannot be split evenly"):
        pkg.parallel.frame_shard(32, 1029, 4, 3, 0)
    with pytest.raises(ValueError, match="multiple of group_frames"):
        pkg.parallel.frame_shard(30, 1029, 4, 2, 0)


def test_sharded_block_equals_single_process(tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, str(tmp_path / "init"), str(tmp_path)), nprocs=world, join=True)
    x, params = _inputs()
    plan, y_full = _single_process(x, params)
    pkg = _pkg()
    for rank in range(world):
        r = np.load(tmp_path / f"rank{rank}.npz")
        shard = pkg.parallel.frame_shard(FRAMES, TPF, GROUP, world, rank)
        # the shard's plan is the restriction of the global plan (supports stay in frame groups)
        lo, hi = np.searchsorted(plan["keep"], [shard.token_begin, shard.token_end])
        np.testing.assert_array_equal(r["keep"], plan["keep"][lo:hi])
        # every rank holds the global merged keys, in the global compact order
        _, kc_g, _, lm_g = _compact_parts(x, params, plan)
        np.testing.assert_allclose(r["kc_all"], kc_g, rtol=0, atol=1e-5)
        np.testing.assert_allclose(r["lm_all"], lm_g, rtol=0, atol=1e-6)
        np.testing.assert_allclose(r["y"], y_full[shard.token_begin:shard.token_end], rtol=0, atol=1e-5)


def _failing_rank_main(rank: int, world: int, init_file: str, out_dir: str) -> None:
    """Rank 1 dies right after joining (no collective in flight); rank 0 then runs the layer's
    all-gather and must get an error back (peer gone, or the short process-group timeout), not
    wait forever."""
    import time
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that exits between steps
    pkg = _pkg()
    t0 = time.monotonic()
    try:
        pkg.parallel.gather_merged([torch.zeros(4, 8), torch.zeros(4)])
        outcome = "completed"
    except Exception as err:  # noqa: BLE001 - any error is the expected outcome
        outcome = f"error {type(err).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as fh:
        fh.write(f"{outcome} {time.monotonic() - t0:.1f}")
    os._exit(0)


def test_dead_rank_ends_the_exchange_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_rank_main, args=(r, 2, str(tmp_path / "init"), str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in procs), "a rank is still waiting"
    assert procs[1].exitcode == 3 and procs[0].exitcode == 0
    outcome = (tmp_path / "rank0.txt").read_text().split()
    assert outcome[0] == "error", outcome
    assert float(outcome[-1]) < 60.0


def _agree_rank_main(rank: int, world: int, init_file: str, out_dir: str) -> None:
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        pkg = _pkg()
        mixed = pkg.parallel.agree_all(rank != 1)  # rank 1's peer-memory setup "failed"
        every = pkg.parallel.agree_all(True)
        with open(os.path.join(out_dir, f"agree{rank}.txt"), "w") as fh:
            fh.write(f"{int(mixed)} {int(every)}")
    finally:
        dist.destroy_process_group()


def test_ranks_agree_on_the_exchange_path(tmp_path):
    """The peer-memory exchange is used only where it was set up on every rank: one rank's
    failure sends all ranks to the NCCL path (no rank left waiting in a different collective)."""
    world = 2
    mp.spawn(_agree_rank_main, args=(world, str(tmp_path / "init"), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        assert (tmp_path / f"agree{rank}.txt").read_text() == "0 1"
