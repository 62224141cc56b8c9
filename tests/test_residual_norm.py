"""sb_residual_rmsnorm: the block around the MoE operator (Block.forward's ffn half, model.py:701-706;
RMSNorm.forward, model.py:197-202) against a torch fp32 restatement, and the residual stack it
serves (StageStack(residual=True))."""
import pytest
import torch

from shard_b200 import wire

TOL = 1e-2


def _ref(x, y, w, eps):
    xs = x if y is None else (x.float() + y.float()).to(torch.bfloat16)
    xf = xs.float()
    n = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return xs, (n if w is None else w.float() * n).to(torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,dim", [(1, 512), (16, 4096), (37, 7168)])
@pytest.mark.parametrize("with_y,with_w", [(True, False), (False, True), (True, True)])
def test_residual_rmsnorm_matches_torch(rows, dim, with_y, with_w):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = torch.Generator().manual_seed(rows + dim)
    x = (torch.randn(rows, dim, generator=g) * 3).to(torch.bfloat16).cuda()
    y = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda() if with_y else None
    w = (1 + 0.1 * torch.randn(dim, generator=g)).cuda() if with_w else None
    xs, ref = _ref(x.clone(), y, w, 1e-6)
    xio = x.clone()
    out = wire.residual_rmsnorm(xio, y, weight=w, eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(xio, xs), "the residual add is one bf16 rounding of the fp32 sum"
    # the norm's mean is summed in another order than torch's: at most one bf16 ulp apart
    err = ((out.float() - ref.float()).abs() / ref.float().abs().clamp_min(1e-3)).max().item()
    assert err <= 2 ** -7
    # add alone
    x2 = x.clone()
    assert wire.residual_rmsnorm(x2, y, norm=False) is None
    torch.cuda.synchronize()
    assert torch.equal(x2, xs)


@pytest.mark.gpu
def test_residual_stack_matches_its_definition():
    """StageStack(residual=True): x <- x + layer(RMSNorm(x)) per layer, the chunk left unchanged."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from shard_b200.pipeline import StageStack

    class Scale:
        def __init__(self, a):
            self.a = a

        def forward(self, x):
            return (x.float() * self.a).to(torch.bfloat16)

    layers = [Scale(0.5), Scale(-0.25), Scale(2.0)]
    x = torch.randn(8, 1024, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    x0 = x.clone()
    got = StageStack(layers, residual=True).forward(x)
    torch.cuda.synchronize()
    assert torch.equal(x, x0)
    ref = x0.clone()
    for l in layers:
        _, n = _ref(ref, None, None, 1e-6)
        ref = (ref.float() + l.forward(n).float()).to(torch.bfloat16)
    err = ((got.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err < TOL
