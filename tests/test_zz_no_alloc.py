"""The no-allocation attention entry point (vb200_mass_bias_attention_noalloc), through the C
ABI.  It serves callers that cannot allocate device memory (raw pointers from another
runtime, or loops that must not call cudaMalloc / cudaFree because those synchronise the
device); its scratch is a fixed array inside the library.  The test compares it with the
workspace entry point on calls in a row — the second with fewer keys, so any scratch left
over from the first call would show, and a last one with 131,072 keys, the most the fixed
array holds — and checks the size limit.

The fixed array only ever holds the bias operand, so the no-allocation call always takes the
unsplit launch.  The first shape is one the split planner would split on a B200, so the
comparison with the minimal-workspace call (which cannot split either) shows that form: the
two outputs are bit-identical.

Collected last (file name) so a run that stops at the first failure has run everything else."""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

MAX_KEYS = 131072


def _strides(t):
    return (ctypes.c_int64 * 3)(*t.stride()[:3])


def _inputs(seed, H, Nq, Nk, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(1, H, Nq, 64, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(1, H, Nk, 64, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(1, H, Nk, 64, generator=g).to(dev, torch.bfloat16)
    lm = torch.log(torch.randint(1, 20, (Nk,), generator=g).float()).to(dev)
    return q, k, v, lm


def _with_workspace(lib, q, k, v, lm):
    """The workspace entry point with the minimal workspace (bias operand only)."""
    out = torch.empty_like(q)
    H, Nk = q.shape[1], k.shape[2]
    ws_bytes = lib.vb200_mass_bias_attention_workspace_size(Nk)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    rc = lib.vb200_mass_bias_attention(1, q.data_ptr(), k.data_ptr(), v.data_ptr(), lm.data_ptr(), 0,
                                       out.data_ptr(), 1, H, q.shape[2], Nk, 64, _strides(q), _strides(k),
                                       _strides(v), _strides(out), ws.data_ptr(), ws_bytes,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.vb200_last_error()
    return out


def _no_alloc(lib, q, k, v, lm):
    out = torch.empty_like(q)
    rc = lib.vb200_mass_bias_attention_noalloc(1, q.data_ptr(), k.data_ptr(), v.data_ptr(), lm.data_ptr(), 0,
                                               out.data_ptr(), 1, q.shape[1], q.shape[2], k.shape[2], 64,
                                               _strides(q), _strides(k), _strides(v), _strides(out),
                                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.vb200_last_error()
    return out


def test_no_alloc_matches_workspace_entry_point(pkg, cuda_device):
    lib = pkg.load_library()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    plan = (ctypes.c_int64 * 5)()
    assert lib.vb200_mass_bias_attention_plan(1, 4, 300, 2000, sms, plan) == 0
    assert plan[3] > 1  # a caller workspace with room for partials would split this shape
    # second call uses fewer keys; the last fills the fixed array exactly
    for seed, (H, Nq, Nk) in enumerate([(4, 300, 2000), (4, 257, 333), (1, 130, MAX_KEYS)]):
        q, k, v, lm = _inputs(seed, H, Nq, Nk, cuda_device)
        ref = _with_workspace(lib, q, k, v, lm)
        got = _no_alloc(lib, q, k, v, lm)
        torch.cuda.synchronize()
        assert_close(to_np(got), to_np(ref), "bf16")
        assert torch.equal(got, ref)  # same (unsplit) launch, same bits
    assert pkg.device_error_flags() == 0


def test_no_alloc_rejects_oversized_key_count(pkg, cuda_device):
    lib = pkg.load_library()
    s = (ctypes.c_int64 * 3)(0, 0, 64)
    rc = lib.vb200_mass_bias_attention_noalloc(1, 16, 16, 16, None, 0, 16, 1, 1, 1, MAX_KEYS + 1, 64, s, s, s, s,
                                               None)
    assert rc == pkg._clib.EINVAL
    assert b"exceed the fixed scratch" in lib.vb200_last_error()
