"""The FP8 activation wire (stage-boundary codec, engines/deepseek_v4/v4_pipe.py:335-384): the CPU oracle
against the reference's own outputs (CPU), and the CUDA codec and the combine kernel with the pack
fused in against both (GPU, through the C ABI). Everything is bit-exact: the codec is integer and
rounding work with one defined result."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle import wire_oracle as W

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "wire_*.npz")))


def _load(path):
    g = np.load(path)
    shape = tuple(int(v) for v in g["shape"])
    x = O.bf16_from_bits(g["x"].view(np.uint16)).reshape(shape)
    s = O.bf16_from_bits(g["scale"].view(np.uint16)).reshape(shape[:-1])
    y = O.bf16_from_bits(g["y"].view(np.uint16)).reshape(shape)
    return x, g["q"].reshape(shape), s, y


def _same(a, b):
    """Bit equality of fp32 arrays holding bf16 values (NaN == NaN, -0 != +0)."""
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_goldens_present():
    assert len(GOLDEN) >= 5


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[5:-4] for p in GOLDEN])
def test_oracle_matches_the_reference_codec(path):
    x, q, s, y = _load(path)
    oq, os_ = W.pack(x)
    assert np.array_equal(oq, q)
    assert _same(os_, s)
    assert _same(W.unpack(q, s), y)


def test_zero_row_and_inf_are_contained():
    x, q, s, y = _load(os.path.join(HERE, "golden", "wire_edges.npz"))
    assert s[0] > 0 and not q[0].any()           # zero row: clamped scale, all-zero codes
    assert q[1, 17] == 0x7E                      # +inf saturates to 448
    assert np.isfinite(y[1, :17]).all() and np.isfinite(y[1, 18:]).all()


def _cuda():
    from shard_b200 import wire
    return wire


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[5:-4] for p in GOLDEN])
def test_cuda_codec_matches_the_reference(path):
    wire = _cuda()
    x, q, s, y = _load(path)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    gq, gs = wire.pack(xt)
    assert tuple(gq.shape) == x.shape and tuple(gs.shape) == x.shape[:-1]
    assert np.array_equal(gq.view(torch.uint8).cpu().numpy(), q)
    assert _same(gs.float().cpu().numpy(), s)
    gy = wire.unpack(torch.from_numpy(q).cuda().view(torch.float8_e4m3fn),
                     torch.from_numpy(s).to(torch.bfloat16).cuda())
    assert _same(gy.float().cpu().numpy(), y)


@pytest.mark.gpu
@pytest.mark.parametrize("name,m", [("c0", 8), ("c1", 16), ("c1", 5)])
def test_forward_with_fused_pack_equals_forward_then_pack(name, m):
    from shard_b200 import synth as S
    wire = _cuda()
    cfg = S.CONFIGS[name]
    lay = S.device_layer(cfg, 0, "cuda", seeded=[] if cfg.n_experts > 32 else None)
    x, _ = S.make_inputs(cfg, m)
    x = x.cuda()
    y = lay.forward(x)
    q, s = lay.forward_wire(x)
    rq, rs = wire.pack(y)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s, rs)
    oq, os_ = W.pack(y.float().cpu().numpy())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), oq)
    assert lay.device_error() == 0
