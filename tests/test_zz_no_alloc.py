"""sb_qgemm_static: the tensor-core dense GEMM with file-scope device scratch (no allocation, no
workspace) against sb_qgemm with a caller workspace, through the C ABI.

Both entry points run the same panel and tcgen05 kernels on the same inputs; sb_qgemm may also
split K across CTAs for narrow batches (fp32 partials in its workspace), which the static entry
point never does, so the two can differ in fp32 summation order, and the test allows the parity
tolerance of the GEMM tests (max relative error 1e-2). Two calls in a row check that the static
scratch is reused cleanly.
"""
import ctypes

import pytest
import torch

from shard_b200 import _lib
from shard_b200 import formats as F

TOL = 1e-2


def _weights(fmt, n, k, seed):
    from shard_b200 import moe
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    ts = None
    if fmt == F.FMT_NVFP4:
        p, s, t = F.quant_nvfp4(w)
        ts = torch.tensor([float(t)], dtype=torch.float32, device="cuda")
        s = s.view(torch.uint8)
    elif fmt == F.FMT_MXFP4:
        p, s = F.quant_mxfp4(w)
        s = s.view(torch.uint8)
    else:
        p, s = F.quant_fp8_block(w)
        s = s.float()
    wt, st = moe.tile(fmt, _lib.MAT_PLAIN, p.view(torch.uint8).cuda(), s.cuda(), 1, n, k, _lib.LAYOUT_TC)
    return wt, st, ts


def _acts(m, k, seed):
    from shard_b200 import ops
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g, dtype=torch.float32).to(torch.bfloat16).cuda()
    q, s = ops.act_quant(x, 128, "ue8m0")
    return q, s.float().contiguous()


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [F.FMT_NVFP4, F.FMT_MXFP4, F.FMT_FP8])
@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (13, 512, 2048), (40, 384, 4096)])
def test_static_scratch_matches_workspace_entry(fmt, m, n, k):
    L = _lib.lib()
    st = _lib.stream_ptr()
    wt, ws_, ts = _weights(fmt, n, k, seed=n + k + fmt)
    q, s = _acts(m, k, seed=m + k)
    wsb = L.sb_qgemm_workspace_bytes(fmt, _lib.LAYOUT_TC, n, k, m)
    work = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib.check(L.sb_qgemm(fmt, _lib.LAYOUT_TC, wt.data_ptr(), ws_.data_ptr(), _lib.ptr(ts), n, k,
                          q.data_ptr(), s.data_ptr(), m, ref.data_ptr(), work.data_ptr(), wsb, st), "sb_qgemm")
    outs = []
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.check(L.sb_qgemm_static(fmt, wt.data_ptr(), ws_.data_ptr(), _lib.ptr(ts), n, k, q.data_ptr(),
                                     s.data_ptr(), m, y.data_ptr(), st), "sb_qgemm_static")
        assert _static_error() == 0, "a kernel of sb_qgemm_static gave up a bounded wait"
        outs.append(y)
    torch.cuda.synchronize()
    for y in outs:
        assert torch.isfinite(y.float()).all()
        assert _rel(y, ref) < TOL
    assert torch.equal(outs[0], outs[1])


def _static_error():
    flag = ctypes.c_int(-1)
    _lib.check(_lib.lib().sb_qgemm_static_error(ctypes.byref(flag), _lib.stream_ptr()), "sb_qgemm_static_error")
    return flag.value


def _run_both(fmt, m, n, k):
    """(static result, workspace result) for one shape."""
    L = _lib.lib()
    st = _lib.stream_ptr()
    wt, ws_, ts = _weights(fmt, n, k, seed=3 * n + k + fmt)
    q, s = _acts(m, k, seed=7 * m + k)
    wsb = L.sb_qgemm_workspace_bytes(fmt, _lib.LAYOUT_TC, n, k, m)
    work = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _lib.check(L.sb_qgemm(fmt, _lib.LAYOUT_TC, wt.data_ptr(), ws_.data_ptr(), _lib.ptr(ts), n, k,
                          q.data_ptr(), s.data_ptr(), m, ref.data_ptr(), work.data_ptr(), wsb, st), "sb_qgemm")
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    _lib.check(L.sb_qgemm_static(fmt, wt.data_ptr(), ws_.data_ptr(), _lib.ptr(ts), n, k, q.data_ptr(),
                                 s.data_ptr(), m, y.data_ptr(), st), "sb_qgemm_static")
    assert _static_error() == 0
    return y, ref


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [F.FMT_NVFP4, F.FMT_FP8])
def test_static_scratch_smaller_call_after_larger(fmt):
    """A call with fewer passes and a shorter K right after a larger one: the region still holds the
    larger call's panel, and the smaller call must read only what it wrote."""
    for m, n, k in [(40, 384, 4096), (13, 512, 2048), (1, 256, 512)]:
        y, ref = _run_both(fmt, m, n, k)
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
        assert _rel(y, ref) < TOL


def test_static_scratch_rejects_oversize():
    """Host-side check, no device work: a shape whose panel exceeds the static region is refused."""
    L = _lib.lib()
    m, n, k = 4096, 256, 7168
    need = _static_need(F.FMT_FP8, k, m)
    assert need > 2 << 20
    rc = L.sb_qgemm_static(F.FMT_FP8, ctypes.c_void_p(256), ctypes.c_void_p(256), None, n, k,
                           ctypes.c_void_p(256), ctypes.c_void_p(256), m, ctypes.c_void_p(256), None)
    assert rc == -2
    msg = L.sb_last_error()
    msg = msg.decode() if isinstance(msg, bytes) else msg
    assert "static region" in msg and str(need) in msg


def _static_need(fmt, k, m):
    """The static region's use as the header states it: a 256-byte flag block, then ceil(m / p)
    passes x k/128 stages of 2048 panel bytes and 64 scale bytes (p = 8 for NVFP4, 16 otherwise),
    each part rounded up to 256 bytes."""
    p = 8 if fmt == F.FMT_NVFP4 else 16
    tiles = -(-m // p) * (k // 128)
    up = lambda b: -(-b // 256) * 256
    return 256 + up(tiles * 2048) + up(tiles * 64)


@pytest.mark.parametrize("fmt,m_max", [(F.FMT_FP8, 272), (F.FMT_MXFP4, 272), (F.FMT_NVFP4, 136)])
def test_static_scratch_limits_at_k7168(fmt, m_max):
    """The stated limits at k = 7168 (m <= 272, NVFP4 m <= 136), pinned from both sides on the host:
    the largest allowed m fits the region, the next pass (one more pass of 16 or 8 tokens) is refused."""
    L = _lib.lib()
    n, k = 256, 7168
    step = 8 if fmt == F.FMT_NVFP4 else 16
    assert _static_need(fmt, k, m_max) <= 2 << 20
    assert _static_need(fmt, k, m_max + step) > 2 << 20
    p = ctypes.c_void_p(256)
    ts = p if fmt == F.FMT_NVFP4 else None
    rc = L.sb_qgemm_static(fmt, p, p, ts, n, k, p, p, m_max + step, p, None)
    assert rc == -2, "one pass beyond the limit must be refused"
    rc = L.sb_qgemm_static(fmt, p, p, ts, n, k, p, p, m_max + 1, p, None)
    assert rc == -2
