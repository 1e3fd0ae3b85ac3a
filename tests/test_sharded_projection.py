"""Query-sharded top-4 projection (parallel.ShardedProjection): config 5's plan, one million
tokens whose sources take parents anywhere among the merged rows, split by token rows over the
ranks.

  * CPU, two gloo ranks: shard_projection_plan cuts keep / source at the same token bounds,
    every rank's partial numerators (oracle segment sums over its own sources) reach the owners
    through all_to_all_single with the split sizes ShardedProjection uses, and the owners'
    rank-ordered reduction plus the all-gathered restore reproduce the one-process oracle.
  * GPU, one rank: the numerator scatter + rank reduction against the one-GPU compact (same
    sums up to the fp32 order of the keep row) and the oracle; restore bit-identical to the
    one-GPU restore, including the staged hot-row gather.
  * GPU, two NCCL ranks (skipped with fewer GPUs): the sharded compact / restore against the
    one-GPU plan.
"""
from __future__ import annotations

import datetime
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO

N, M, C = 4096, 256, 64


def _pkg():
    import importlib
    import sys
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    return importlib.import_module("4d_ttt_merging_b200")


def _gloo_rank(rank: int, world: int, init_file: str, out_dir: str) -> None:
    import sys
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    import oracle
    from oracle import ref
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        pkg = _pkg()
        keep, src, parent, w = oracle.zipf_plan(5, N, M)
        norm = oracle.normalizer(parent, w, M)
        rng = np.random.default_rng(9)
        x = rng.standard_normal((N, C)).astype(np.float32)
        sh = pkg.parallel.shard_projection_plan(torch.from_numpy(keep), torch.from_numpy(src),
                                                torch.from_numpy(parent), torch.from_numpy(w), N, world, rank)
        x_local = x[sh["t0"]:sh["t1"]]
        pl, wl = sh["parent_local"].numpy(), sh["weights_local"].numpy()
        rows = x_local[sh["source_local"].numpy()]
        numer = np.zeros((M, C), np.float32)
        for c in range(pl.shape[1]):
            numer = (numer + ref._segment_sums(rows, pl[:, c], wl[:, c], M)).astype(np.float32)
        owned = sh["m1"] - sh["m0"]
        recv = torch.empty((world * owned, C), dtype=torch.float32)
        dist.all_to_all_single(recv, torch.from_numpy(numer), output_split_sizes=[owned] * world,
                               input_split_sizes=sh["owned_counts"])
        acc = x_local[sh["keep_local"].numpy()].astype(np.float32)
        for r in range(world):  # rank order
            acc = (acc + recv[r * owned:(r + 1) * owned].numpy()).astype(np.float32)
        out = (acc / norm[sh["m0"]:sh["m1"], None]).astype(np.float32)
        # restore: all-gather the owned rows in rank order, then the rank's own tokens
        full = pkg.parallel.gather_merged([torch.from_numpy(out)])[0].numpy()
        tokens = np.zeros((sh["t1"] - sh["t0"], C), np.float32)
        tokens[sh["keep_local"].numpy()] = full[sh["m0"]:sh["m1"]]
        acc = np.zeros((len(pl), C), np.float32)
        for c in range(pl.shape[1]):
            acc = (acc + (wl[:, c, None] * full[pl[:, c]]).astype(np.float32)).astype(np.float32)
        tokens[sh["source_local"].numpy()] = acc
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), compact=out, restore=tokens, t0=sh["t0"], m0=sh["m0"],
                 counts=np.array(sh["owned_counts"]))
    finally:
        dist.destroy_process_group()


def test_sharded_projection_logic_gloo(tmp_path, oracle):
    world = 2
    mp.spawn(_gloo_rank, args=(world, str(tmp_path / "init"), str(tmp_path)), nprocs=world, join=True)
    keep, src, parent, w = oracle.zipf_plan(5, N, M)
    norm = oracle.normalizer(parent, w, M)
    x = np.random.default_rng(9).standard_normal((N, C)).astype(np.float32)
    ref_compact = oracle.compact(x, keep, src, parent, w, norm)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    assert [int(p["t0"]) for p in parts] == [0, N // 2]
    assert parts[0]["counts"].tolist() == [M // 2, M // 2]
    got = np.concatenate([p["compact"] for p in parts])
    # same sums, grouped per rank: fp32 reassociation only
    np.testing.assert_allclose(got, ref_compact, rtol=1e-5, atol=1e-5)
    ref_restore = oracle.restore(got, keep, src, parent, w, N)
    np.testing.assert_array_equal(np.concatenate([p["restore"] for p in parts]), ref_restore)


def test_shard_bounds_ragged():
    """Bounds on a plan whose keep tokens are not evenly spread: every token, merged row and
    source lands on exactly one rank, and ranks own unequal merged-row counts."""
    pkg = _pkg()
    n = 1000
    keep = torch.tensor([0, 3, 4, 5, 600, 601, 999])
    mask = torch.ones(n, dtype=torch.bool)
    mask[keep] = False
    src = torch.nonzero(mask).flatten()
    parent = torch.randint(0, keep.numel(), (src.numel(), 4))
    w = torch.full((src.numel(), 4), 0.25)
    shards = [pkg.parallel.shard_projection_plan(keep, src, parent, w, n, 3, r) for r in range(3)]
    assert [s["owned_counts"] for s in shards] == [[4, 2, 1]] * 3
    assert torch.equal(torch.cat([s["keep_local"] + s["t0"] for s in shards]), keep)
    assert torch.equal(torch.cat([s["source_local"] + s["t0"] for s in shards]), src)
    assert torch.equal(torch.cat([s["parent_local"] for s in shards]), parent)
    assert shards[-1]["t1"] == n


def _device_plan(pkg, dev, n, m, seed):
    """A config-5-shaped plan on the device: m evenly spaced keep tokens, four distinct parents
    per source (a random permutation window), Dirichlet(1,1,1,1) weights."""
    g = torch.Generator(device=dev).manual_seed(seed)
    keep = torch.arange(m, device=dev) * (n // m)
    mask = torch.ones(n, dtype=torch.bool, device=dev)
    mask[keep] = False
    src = torch.nonzero(mask).flatten()
    S = src.numel()
    base = torch.randint(0, m, (S, 1), device=dev, generator=g)
    step = torch.randint(1, m // 4, (S, 1), device=dev, generator=g)
    parent = (base + step * torch.arange(4, device=dev)[None]) % m
    e = -torch.rand(S, 4, device=dev, generator=g).clamp_min(1e-12).log()
    w = (e / e.sum(1, keepdim=True)).float()
    norm = pkg.deterministic_weighted_normalizer(parent[None], w[None], m)
    plan = pkg.WeightedBilinearTokenPlan(
        keep=keep[None], source_original=src[None], source_parent_compact=parent[None], source_pool_weights=w[None],
        source_restore_weights=w[None], original_tokens=n, normalizer=norm, key_log_mass=norm[..., 0].log())
    return keep, src, parent, w, norm[0, :, 0], plan


@pytest.mark.gpu
@pytest.mark.parametrize("n,m,c", [(N, M, C), (1 << 18, 1 << 14, 256)])
def test_one_rank_matches_single_gpu(pkg, oracle, cuda_device, n, m, c):
    dev = cuda_device
    keep, src, parent, w, norm, plan = _device_plan(pkg, dev, n, m, 3)
    proj = pkg.parallel.ShardedProjection(keep, src, parent, w, norm, n)
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn(n, c, device=dev, generator=g).to(torch.bfloat16)
    got = proj.compact(x)
    ref = plan.compact(x[None])[0]
    err = (got.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert err <= 8e-3, err
    if n == N:
        o = oracle.compact(x.float().cpu().numpy(), keep.cpu().numpy(), src.cpu().numpy(), parent.cpu().numpy(),
                           w.cpu().numpy(), norm.cpu().numpy(), dtype="bf16")
        assert np.abs(got.float().cpu().numpy() - o).max() <= 2 ** -7 * np.abs(o).max()
    y = torch.randn(m, c, device=dev, generator=g).to(torch.bfloat16)
    assert torch.equal(proj.restore(y), plan.restore(y[None])[0])
    assert pkg.device_error_flags() == 0


def _nccl_rank(rank: int, world: int, init_file: str, out_dir: str) -> None:
    import sys
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    pkg = _pkg()
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        n, m, c = 1 << 18, 1 << 14, 256
        keep, src, parent, w, norm, plan = _device_plan(pkg, dev, n, m, 3)
        g = torch.Generator(device=dev).manual_seed(4)
        x = torch.randn(n, c, device=dev, generator=g).to(torch.bfloat16)
        y = torch.randn(m, c, device=dev, generator=g).to(torch.bfloat16)
        proj = pkg.parallel.ShardedProjection(keep, src, parent, w, norm, n)
        got = proj.compact(x[proj.t0:proj.t1].contiguous())
        ref = plan.compact(x[None])[0][proj.m0:proj.m1]
        restored = proj.restore(y[proj.m0:proj.m1].contiguous())
        ref_r = plan.restore(y[None])[0][proj.t0:proj.t1]
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
        ok = err <= 8e-3 and torch.equal(restored, ref_r) and pkg.device_error_flags() == 0
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write(f"{int(ok)} {err}\n")
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_ranks_match_single_gpu(tmp_path, cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.spawn(_nccl_rank, args=(world, str(tmp_path / "init"), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        ok, err = (tmp_path / f"rank{r}").read_text().split()
        assert ok == "1", (r, err)
