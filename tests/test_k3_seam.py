"""Kimi-K3's routed experts: KimiSparseMoeBlock.moe_infer (vendor/kimi_k3_ref/modeling_kimi_linear.py:
850-876), the method the reference's K3 engine replaces (engines/kimi_k3/k3_moe_mxfp4.py:405-412).

The golden vectors are the reference block's own outputs (tests/golden/make_golden.py, K3_CASES):
its KimiMoEGate's routing and its moe_infer on MXFP4 experts held as their exact bf16 values. The
CPU tests pin the oracle to them and rebuild the block's layout from the recorded seam fixture; the
GPU tests run the K3-mode forward (sb_moe_forward_routed) and the installed seam against them."""
import json
import os
import types

import numpy as np
import pytest
import torch
from torch import nn

from make_golden import K3_CASES, k3_config
from oracle import moe_oracle as O
from shard_b200 import formats as F
from shard_b200 import k3 as K3
from shard_b200 import synth as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-2
CASES = list(K3_CASES)


def _golden(name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: g[k] for k in g.files}


def _inputs(name):
    cfg, m, beta, lb = k3_config(name)
    x, _ = S.make_inputs(cfg, m)
    return cfg, m, beta, lb, x


def _oracle_expert(cfg):
    i = cfg.inter

    def expert(e):
        ew = S.make_expert(cfg, 0, e)
        return ew.w13.numpy(), ew.w13_s.numpy(), ew.w2.numpy(), ew.w2_s.numpy()
    return expert


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_moe_infer(name):
    g = _golden(name)
    cfg, m, beta, lb, x = _inputs(name)
    assert S.tensor_sha(x) == str(g["x_sha"]), "the seeded inputs drifted from the golden's"
    shas = json.loads(str(g["expert_sha"]))
    ew = S.make_expert(cfg, 0, 3)
    assert S.tensor_sha(ew.w13, ew.w13_s, ew.w2, ew.w2_s) == shas["3"]
    y = O.k3_moe_infer(x.float().numpy(), g["topk_idx"], g["topk_weight"], _oracle_expert(cfg), beta, lb)
    yref = O.bf16_from_bits(g["y_bits"])
    assert O.max_rel_err(y, yref) < TOL
    assert (y != yref).mean() < 0.02


# ── a stand-in for the reference module, rebuilt from the recorded seam fixture ───────────────────

class _Situ:
    def __init__(self, beta, linear_beta):
        self.beta, self.linear_beta = beta, linear_beta


class _Expert(nn.Module):
    """KimiBlockSparseMLP (modeling_kimi_linear.py:242-270): w1 (gate), w2 (down), w3 (up), act_fn."""

    def __init__(self, h, i, act):
        super().__init__()
        self.w1 = nn.Linear(h, i, bias=False, dtype=torch.bfloat16)
        self.w2 = nn.Linear(i, h, bias=False, dtype=torch.bfloat16)
        self.w3 = nn.Linear(h, i, bias=False, dtype=torch.bfloat16)
        self.act_fn = act


class KimiSparseMoeBlock(nn.Module):
    """The attributes moe_infer's replacement reads (modeling_kimi_linear.py:782-807); the method
    itself stands in for the reference's and counts its calls (a declined call lands here)."""

    calls = 0

    def __init__(self, rec, experts):
        super().__init__()
        self.top_k, self.num_experts = rec["top_k"], rec["num_experts"]
        self.ep_size, self.ep_rank, self.experts_per_rank = rec["ep_size"], rec["ep_rank"], rec["experts_per_rank"]
        self.moe_hidden_size = rec["moe_hidden_size"]
        self.experts = nn.ModuleList(experts)

    def moe_infer(self, x, topk_ids, topk_weight):
        type(self).calls += 1
        return torch.zeros_like(x)


def _mirror(name):
    with open(os.path.join(GOLDEN, f"seam_{name}.json")) as f:
        rec = json.load(f)
    cfg, m, beta, lb = k3_config(name)
    h, i = cfg.hidden, cfg.inter
    act = _Situ(rec["act"]["beta"], rec["act"]["linear_beta"])
    experts = []
    for e in range(rec["num_experts"]):
        ex = _Expert(h, i, act)
        ew = S.make_expert(cfg, 0, e)
        with torch.no_grad():
            ex.w1.weight.copy_(F.dequant_weight(F.FMT_MXFP4, ew.w13[:i], ew.w13_s[:i]).to(torch.bfloat16))
            ex.w3.weight.copy_(F.dequant_weight(F.FMT_MXFP4, ew.w13[i:], ew.w13_s[i:]).to(torch.bfloat16))
            ex.w2.weight.copy_(F.dequant_weight(F.FMT_MXFP4, ew.w2, ew.w2_s).to(torch.bfloat16))
        experts.append(ex)
    block = KimiSparseMoeBlock(rec, experts)
    import hashlib
    for pname, d in rec["params"].items():
        t = block.get_parameter(pname)
        assert str(t.dtype) == d["dtype"] and list(t.shape) == d["shape"], pname
        assert hashlib.sha256(t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest() == d["sha"], pname
    mod = types.ModuleType("modeling_kimi_linear")
    mod.KimiSparseMoeBlock = KimiSparseMoeBlock
    return mod, block


@pytest.mark.parametrize("name", CASES)
def test_fixture_rebuilds_the_reference_block_and_declines_on_cpu(name):
    g = _golden(name)
    mod, block = _mirror(name)
    _, m, _, _, x = _inputs(name)
    assert K3.install(mod)
    try:
        assert not K3.install(mod)
        before = KimiSparseMoeBlock.calls
        block.moe_infer(x, torch.from_numpy(g["topk_idx"]), torch.from_numpy(g["topk_weight"]))
        assert KimiSparseMoeBlock.calls == before + 1
        assert K3.coverage(block) == {0: (0, {"not-on-cuda": 1})}
    finally:
        assert K3.uninstall(mod)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_k3_forward_matches_reference_moe_infer(name):
    """sb_moe_forward_routed in K3 mode: bf16 activations into MXFP4 experts, situ, the routing
    weights applied to the expert outputs, slot-order sum, against the reference block's output."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = _golden(name)
    mod, block = _mirror(name)
    layer = K3.layer_from_block(block, torch.device("cuda"))
    _, m, _, _, x = _inputs(name)
    ids = torch.from_numpy(g["topk_idx"]).cuda()
    w = torch.from_numpy(g["topk_weight"]).cuda()
    y = layer.forward_routed(x.cuda(), ids, w)
    y2 = layer.forward_routed(x.cuda(), ids, w)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    assert layer.device_error() == 0
    err = O.max_rel_err(y.float().cpu().numpy(), O.bf16_from_bits(g["y_bits"]))
    assert err < TOL, f"{name}: max rel err {err:.3e}"
    # each token alone gives its row of the batch (row invariance)
    for t in (0, m - 1):
        yt = layer.forward_routed(x[t:t + 1].cuda(), ids[t:t + 1], w[t:t + 1])
        assert torch.equal(yt, y[t:t + 1])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_installed_moe_infer_on_the_reference_block(name):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = _golden(name)
    mod, block = _mirror(name)
    block.cuda()
    _, m, _, _, x = _inputs(name)
    assert K3.install(mod)
    try:
        before = KimiSparseMoeBlock.calls
        y = block.moe_infer(x.cuda(), torch.from_numpy(g["topk_idx"]).cuda(), torch.from_numpy(g["topk_weight"]).cuda())
        torch.cuda.synchronize()
        assert KimiSparseMoeBlock.calls == before, "the reference method must not run"
        assert K3.coverage(block) == {0: (1, {})}
        err = O.max_rel_err(y.float().cpu().numpy(), O.bf16_from_bits(g["y_bits"]))
        assert err < TOL, f"{name}: max rel err {err:.3e}"
    finally:
        assert K3.uninstall(mod)
