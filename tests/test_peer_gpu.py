"""The rank-ordered exchange kernels of the sharded block (vb200_peer_gather / vb200_peer_push)
on one GPU: several local buffers stand in for the ranks' peer-mapped blocks, so the copies,
row offsets, strides and both vector paths are checked against torch.cat."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _u64(ptrs):
    return (ctypes.c_uint64 * len(ptrs))(*ptrs)


@pytest.mark.parametrize("cols,pad,dtype", [(96, 8, torch.bfloat16), (7, 5, torch.float32)])  # 16- / 4-byte paths
def test_peer_gather_rank_order(pkg, cuda_device, cols, pad, dtype):
    lib, C = pkg.load_library(), pkg._clib
    world, rows = 3, 37
    g = torch.Generator(device="cpu").manual_seed(0)
    # each "rank" holds a [rows, pad + cols] block; the exchanged part is its last `cols` columns
    blocks = [torch.randn(rows, pad + cols, generator=g).to(cuda_device, dtype) for _ in range(world)]
    es = blocks[0].element_size()
    src = _u64([b.data_ptr() + pad * es for b in blocks])
    out = torch.empty(world * rows, cols, device=cuda_device, dtype=dtype)
    rc = lib.vb200_peer_gather(src, world, rows, (pad + cols) * es, cols * es, out.data_ptr(), cols * es,
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.vb200_last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, torch.cat([b[:, pad:] for b in blocks]))


def test_peer_push_to_every_rank(pkg, cuda_device):
    lib = pkg.load_library()
    world, rows, cols = 4, 29, 64
    g = torch.Generator(device="cpu").manual_seed(1)
    full = [torch.zeros(world * rows, cols, device=cuda_device, dtype=torch.bfloat16) for _ in range(world)]
    mine = [torch.randn(rows, 3 * cols, generator=g).to(cuda_device, torch.bfloat16) for _ in range(world)]
    dst = _u64([f.data_ptr() for f in full])
    for r in range(world):  # rank r pushes columns [cols, 2 cols) of its rows into every buffer
        rc = lib.vb200_peer_push(mine[r].data_ptr() + cols * 2, rows, 3 * cols * 2, cols * 2, dst, world, r * rows,
                                 cols * 2, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.vb200_last_error()
    torch.cuda.synchronize()
    expect = torch.cat([m[:, cols:2 * cols] for m in mine])
    for f in full:
        assert torch.equal(f, expect)


@pytest.mark.parametrize("dim", [256, 1024])  # 8- and 16-channel consumer threads
def test_compact_qkv_peer_writes_every_rank(pkg, cuda_device, dim):
    """The compaction with the fused k|v all-gather: `out` equals the plain compaction bit for
    bit, and every destination buffer (three local buffers standing in for the ranks) holds the
    merged k|v rows at the given row offset, other rows untouched."""
    dev = cuda_device
    g = torch.Generator(device="cpu").manual_seed(3)
    frames, tpf = 4, 100
    tok = torch.randn(1, frames * tpf, dim, generator=g).to(dev, torch.bfloat16)
    plan = pkg.build_uniform_convex_plan(tok, frames=frames, tokens_per_frame=tpf, patch_token_start=5,
                                         merge_factor=4, group_frames=4)
    qkv = torch.randn(frames * tpf, 3 * dim, generator=g).to(dev, torch.bfloat16)
    lw = (1 + 0.1 * torch.randn(2, 64, generator=g)).to(dev)
    lb = (0.1 * torch.randn(2, 64, generator=g)).to(dev)
    ref = plan.compact_qkv(qkv, lw, lb, 1e-6)
    M = plan.kept_tokens
    world, row0, stride = 3, 7, 2 * dim + 64
    sentinel = 12345.0
    bufs = [torch.full((row0 + M + 5, stride), sentinel, device=dev, dtype=torch.bfloat16) for _ in range(world)]
    ptrs = _u64([b.data_ptr() for b in bufs])
    out = torch.empty_like(ref)
    got = plan.compact_qkv(qkv, lw, lb, 1e-6, out=out, kv_peers=(ptrs, world, row0, stride))
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    # the statistics computed ahead on another stream (vb200_qkv_head_stats) give the same rows
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        stats = pkg.ops.qkv_head_stats(qkv, 1e-6)
    torch.cuda.current_stream(dev).wait_stream(side)
    assert torch.equal(plan.compact_qkv(qkv, lw, lb, 1e-6, stats=stats), ref)
    for b in bufs:
        assert torch.equal(b[row0:row0 + M, :2 * dim], ref[:, dim:])
        assert torch.all(b[:row0] == sentinel) and torch.all(b[row0 + M:] == sentinel)
        assert torch.all(b[:, 2 * dim:] == sentinel)
    assert pkg.device_error_flags() == 0


def _barrier(lib, pads, world, rank, epoch, timeout_ns):
    ptrs = _u64([p.data_ptr() for p in pads])
    rc = lib.vb200_peer_barrier(ptrs, world, rank, epoch.data_ptr(), timeout_ns,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.vb200_last_error()


def test_peer_barrier_single_rank_and_graph_replay(pkg, cuda_device):
    """One rank: every barrier passes at once and advances the device-side epoch, also when
    replayed from a recorded CUDA graph (the epoch is not baked into the launch)."""
    lib = pkg.load_library()
    pad = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for _ in range(3):
        _barrier(lib, [pad], 1, 0, epoch, 1_000_000_000)
    torch.cuda.synchronize()
    assert int(epoch) == 3 and int(pad) == 3
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            _barrier(lib, [pad], 1, 0, epoch, 1_000_000_000)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    assert int(epoch) == 7 and int(pad) == 7
    assert pkg.device_error_flags() == 0


def test_peer_barrier_gives_up_with_an_error(pkg, cuda_device):
    """Rank 0 of two, on one GPU: a local buffer stands in for rank 1's pad.  The barrier signals
    'rank 1' and waits for a signal that nothing sends; after its 50 ms limit it sets error
    bit 0 and returns.  The context stays usable: with the peer's signal already in place the
    next barrier passes."""
    lib = pkg.load_library()
    pads = [torch.zeros(2, dtype=torch.int32, device=cuda_device) for _ in range(2)]  # rank 0's, rank 1's
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _barrier(lib, pads, 2, 0, epoch, 50_000_000)
    assert pkg.device_error_flags() & 1
    assert int(pads[1][0]) == 1 and int(epoch) == 1  # the signal to rank 1 was sent
    pads[0][1] = 2  # rank 1's next signal has arrived
    _barrier(lib, pads, 2, 0, epoch, 50_000_000)
    assert pkg.device_error_flags() == 0
    assert int(pads[1][0]) == 2 and int(epoch) == 2
    x = torch.arange(10, device=cuda_device)
    assert int(x.sum()) == 45
