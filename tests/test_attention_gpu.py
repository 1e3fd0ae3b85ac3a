"""Mass-bias attention on the GPU (tcgen05 path for bf16 / fp16, FMA path for fp32) against
the oracle restatement of vggt_omega/models/mass_bias_attention.py:85-129, through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import TORCH_DTYPE, assert_close, to_np

pytestmark = pytest.mark.gpu


def _inputs(seed, B, H, Nq, Nk, dtype, oracle, mass_max=50):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, Nq, 64)).astype(np.float32)
    k = rng.standard_normal((B, H, Nk, 64)).astype(np.float32)
    v = rng.standard_normal((B, H, Nk, 64)).astype(np.float32)
    mass = rng.integers(1, mass_max, size=Nk).astype(np.float32)
    log_mass = np.log(mass).astype(np.float32)
    q, k, v = (oracle.round_to(t, dtype) for t in (q, k, v))
    return q, k, v, log_mass


def _run(pkg, q, k, v, log_mass, dtype, device, bias_dtype=torch.float32):
    td = TORCH_DTYPE[dtype]
    qt, kt, vt = (torch.from_numpy(t).to(device=device, dtype=td) for t in (q, k, v))
    lm = None if log_mass is None else torch.from_numpy(log_mass).to(device=device, dtype=bias_dtype)
    out = pkg.mass_bias_attention(qt, kt, vt, lm)
    torch.cuda.synchronize()
    assert out.dtype == td
    return to_np(out)


SHAPES = [
    (1, 1, 1, 1),      # single query, single key
    (1, 2, 5, 7),      # everything inside one partial tile
    (1, 3, 130, 129),  # ragged query and key tails
    (2, 2, 257, 300),  # batch > 1, three query tiles, three key tiles
    (1, 4, 1029, 1029),
    (1, 2, 640, 2176),  # many key tiles (pipeline phases wrap several times)
]


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_against_oracle(pkg, oracle, cuda_device, dtype, shape):
    B, H, Nq, Nk = shape
    q, k, v, lm = _inputs(sum(shape), B, H, Nq, Nk, dtype, oracle)
    out = _run(pkg, q, k, v, lm, dtype, cuda_device)
    ref = oracle.mass_bias_attention(q, k, v, lm, dtype=dtype, round_p=dtype != "f32")
    assert_close(out, ref, dtype)
    assert pkg.device_error_flags() == 0


@pytest.mark.parametrize("bias_dtype", [torch.float32, torch.bfloat16])
def test_bias_rounding_and_no_bias(pkg, oracle, cuda_device, bias_dtype):
    q, k, v, lm = _inputs(7, 1, 2, 300, 333, "bf16", oracle, mass_max=5000)
    out = _run(pkg, q, k, v, lm, "bf16", cuda_device, bias_dtype=bias_dtype)
    ref = oracle.mass_bias_attention(q, k, v, lm, dtype="bf16", round_p=True)
    assert_close(out, ref, "bf16")
    # None bias = plain softmax attention (the dense special-query call)
    out0 = _run(pkg, q, k, v, None, "bf16", cuda_device)
    assert_close(out0, oracle.mass_bias_attention(q, k, v, None, dtype="bf16", round_p=True), "bf16")


def test_config1_shape_fp32(pkg, oracle, golden, cuda_device):
    """Config 1 (fp32): N=4116 queries over M=1029 merged keys with integer masses, all 16
    heads in one launch: the reference-generated golden head (its SDPA-with-mask call) and
    three more heads against the oracle, to the fp32 bar."""
    c1 = oracle.c1_inputs(seed=0)
    out = _run(pkg, c1["q"], c1["k"], c1["v"], c1["log_mass"], "f32", cuda_device)
    h = int(golden["c1_heads"][0])
    assert_close(out[0, h], golden["c1_attention"][0], "f32")
    for hh in (0, 9, 15):
        sl = slice(hh, hh + 1)
        ref = oracle.mass_bias_attention(c1["q"][:, sl], c1["k"][:, sl], c1["v"][:, sl], c1["log_mass"])
        assert_close(out[:, sl], ref, "f32")


def test_strided_views_and_autocast(pkg, oracle, cuda_device):
    """q/k/v as views of an interleaved [B, N, 3, H, 64] qkv buffer (the layout of the
    attention layer), fp32 under bf16 autocast -> bf16 output, as the reference wrapper."""
    rng = np.random.default_rng(3)
    B, N, H = 1, 333, 4
    qkv = torch.from_numpy(rng.standard_normal((B, N, 3, H, 64)).astype(np.float32)).to(cuda_device)
    q, k, v = (t.transpose(1, 2) for t in qkv.unbind(2))
    lm = torch.from_numpy(np.log(rng.integers(1, 9, N)).astype(np.float32)).to(cuda_device)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = pkg.mass_bias_attention(q, k, v, lm)
    assert out.dtype == torch.bfloat16
    qb, kb, vb = (oracle.round_bf16(to_np(t)) for t in (q, k, v))
    ref = oracle.mass_bias_attention(qb, kb, vb, to_np(lm), dtype="bf16", round_p=True)
    assert_close(to_np(out), ref, "bf16")
    # the returned [B,H,N,64] tensor is a view of a token-major buffer
    assert out.transpose(1, 2).is_contiguous()


def test_output_into_strided_buffer(pkg, oracle, cuda_device):
    q, k, v, lm = _inputs(11, 1, 2, 200, 150, "bf16", oracle)
    dev = cuda_device
    qt, kt, vt = (torch.from_numpy(t).to(dev, torch.bfloat16) for t in (q, k, v))
    big = torch.zeros(1, 200, 4, 64, device=dev, dtype=torch.bfloat16)
    out = big[:, :, 1:3].transpose(1, 2)  # heads interleaved with untouched columns
    pkg.mass_bias_attention_into(qt, kt, vt, torch.from_numpy(lm).to(dev), out)
    torch.cuda.synchronize()
    ref = oracle.mass_bias_attention(q, k, v, lm, dtype="bf16", round_p=True)
    assert_close(to_np(out), ref, "bf16")
    assert torch.count_nonzero(big[:, :, 0]) == 0 and torch.count_nonzero(big[:, :, 3]) == 0


def test_errors(pkg, cuda_device):
    q = torch.zeros(1, 2, 8, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="log_key_mass length"):
        pkg.mass_bias_attention(q, q, q, torch.zeros(7, device=cuda_device))
    with pytest.raises(ValueError, match="head_dim"):
        pkg.mass_bias_attention(q[..., :32], q[..., :32], q[..., :32], torch.zeros(8, device=cuda_device))


def test_exp2_polynomial_against_exact(pkg, cuda_device):
    """The softmax's FMA-pipe exponential: relative error <= 1e-4 against exact 2^x over the
    range the kernel feeds it (x - running max <= 8), tiny positive values below -125."""
    import ctypes  # noqa: F401
    x = torch.cat([torch.linspace(-125, 8, 2_000_001), torch.tensor([-1000.0, -126.0, 0.0, 0.5, -0.5])])
    xd = x.to(cuda_device)
    y = torch.empty_like(xd)
    rc = pkg.load_library().vb200_exp2_poly(xd.data_ptr(), y.data_ptr(), xd.numel(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    got = y.cpu().double()
    exact = torch.exp2(x.double())
    main = x >= -125
    rel = ((got[main] - exact[main]).abs() / exact[main]).max().item()
    assert rel <= 1e-4, rel
    assert torch.all(got[~main] >= 0) and torch.all(got[~main] < 1e-37)


def _abi_call(pkg, qt, kt, vt, lm, out, ws_bytes):
    """One launch through the C ABI with a workspace of ws_bytes."""
    import ctypes
    lib = pkg.load_library()
    i64x3 = ctypes.c_int64 * 3
    st = lambda t: i64x3(*t.stride()[:3])  # noqa: E731
    B, H, Nq, _ = qt.shape
    Nk = kt.shape[2]
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=qt.device)
    rc = lib.vb200_mass_bias_attention(1, qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), lm.data_ptr(), 0,
                                       out.data_ptr(), B, H, Nq, Nk, 64, st(qt), st(kt), st(vt), st(out),
                                       ws.data_ptr(), ws_bytes, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.vb200_last_error()
    torch.cuda.synchronize()
    return out.clone()


def test_split_last_wave(pkg, oracle, cuda_device):
    """More (query block, head) items than one wave of SMs, with a partial last wave: that
    wave's items run as key-range pieces merged by the last piece to finish.  The result
    matches the oracle, is bit-identical from run to run (fixed merge order), and agrees with
    the unsplit launch (workspace without room for the pieces) to within bf16 rounding."""
    B, H, Nq, Nk = 1, 16, 2600, 1100  # 11 query blocks x 16 heads = 176 items, 9 key tiles
    q, k, v, lm = _inputs(23, B, H, Nq, Nk, "bf16", oracle)
    qt, kt, vt = (torch.from_numpy(t).to(cuda_device, torch.bfloat16) for t in (q, k, v))
    lmt = torch.from_numpy(lm).to(cuda_device)
    lib = pkg.load_library()
    base = lib.vb200_mass_bias_attention_workspace_size(Nk)
    full = lib.vb200_mass_bias_attention_split_workspace_size(B, H, Nq, Nk)
    assert full > base  # 176 items leave a partial wave on a 148-SM B200
    out = torch.empty(B, Nq, H, 64, device=cuda_device, dtype=torch.bfloat16).transpose(1, 2)
    split1 = _abi_call(pkg, qt, kt, vt, lmt, out, full)
    split2 = _abi_call(pkg, qt, kt, vt, lmt, out, full)
    plain = _abi_call(pkg, qt, kt, vt, lmt, out, base)
    assert torch.equal(split1, split2)
    ref = oracle.mass_bias_attention(q, k, v, lm, dtype="bf16", round_p=True)
    assert_close(to_np(split1), ref, "bf16")
    assert_close(to_np(plain), ref, "bf16")
    diff = (split1.float() - plain.float()).abs().max().item()
    assert diff <= 2.0 ** -6 * plain.float().abs().max().item(), diff
    assert pkg.device_error_flags() == 0
