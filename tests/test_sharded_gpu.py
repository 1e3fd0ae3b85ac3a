"""The query-sharded layer on two GPUs (skipped with fewer): two NCCL ranks, each running
ShardedGlobalBlock on its 4 frames, against one GPU running the whole 8-frame block.  The
merged K|V all-gather is fused into the compaction (one posted store per rank, or, opted in,
one multicast store per row where the symmetric-memory allocation has a multicast object); both
forms are checked,
and a recorded step graph must replay the eager sharded step bit for bit."""
from __future__ import annotations

import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

FRAMES, TPF, DIM, HEADS = 8, 1029, 1024, 16


def _weights(pkg, dev):
    torch.manual_seed(0)
    attn = pkg.GlobalAttention(DIM, HEADS, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in attn.parameters():
            p.normal_(0.0, 0.02)
        attn.q_norm.weight.fill_(1.0)
        attn.k_norm.weight.fill_(1.0)
    return attn


def _rank(rank: int, world: int, init_file: str, result_file: str) -> None:
    import importlib
    import sys
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    pkg = importlib.import_module("4d_ttt_merging_b200")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        attn = _weights(pkg, dev)
        gen = torch.Generator(device="cpu").manual_seed(1)
        tokens = torch.randn(1, FRAMES * TPF, DIM, generator=gen).to(dev, torch.bfloat16)
        kw = dict(frames=FRAMES, tokens_per_frame=TPF, patch_token_start=5, merge_factor=4, group_frames=4)
        full = pkg.parallel.ShardedGlobalBlock(attn, **kw).step(tokens)
        res = {}
        for mode in ("multicast", "per_rank"):
            os.environ["VB200_PEER_MULTICAST"] = "1" if mode == "multicast" else "0"
            block = pkg.parallel.ShardedGlobalBlock(attn, world=world, rank=rank, **kw)
            sh = block.shard
            x = tokens[:, sh.token_begin:sh.token_end].contiguous()
            out = block.step(x).clone()
            ref = full[:, sh.token_begin:sh.token_end].float()
            err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
            cos = torch.nn.functional.cosine_similarity(out.float().flatten(), ref.flatten(), dim=0).item()
            g = pkg.parallel.StepGraph(block, x)
            rep = g.replay().clone()
            torch.cuda.synchronize()
            same = bool(torch.equal(rep, out))
            g.release()
            res[mode] = (err, cos, same, block._xchg is not None,
                         bool(block._xchg is not None and block._xchg.multicast))
        os.environ.pop("VB200_PEER_MULTICAST", None)
        res["flags"] = pkg.device_error_flags()
        if rank == 0:
            torch.save(res, result_file)
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_block_two_ranks():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        init_file, result_file = os.path.join(d, "init"), os.path.join(d, "res.pt")
        mp.spawn(_rank, args=(2, init_file, result_file), nprocs=2, join=True)
        res = torch.load(result_file)
    assert res["flags"] == 0
    for mode in ("multicast", "per_rank"):
        err, cos, same, peer, _ = res[mode]
        assert peer, "the peer-memory exchange was not used"
        assert err <= 2e-2 and cos > 0.999, (mode, err, cos)
        assert same, mode
    assert not res["per_rank"][4]
    print("multicast object available:", res["multicast"][4])
