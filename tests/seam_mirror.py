"""A stand-in for the reference's model module, rebuilt from a recorded seam fixture, for the
operator-seam tests.

The reference's MoE module (vendor/deepseek_v4_ref/inference/model.py) cannot be imported where the
GPU tests run, so tests/golden/make_golden.py records, next to each golden case, everything
`shard_b200.moe.install` / `layer_from_module` / `b200_moe_forward` read from the reference module
it built: the module-level globals, the MoE / Gate / Expert / Linear attributes, every parameter's
name, dtype and shape, the `weight.scale is scale` link and the NVFP4 `weight.tensor_scale`
attribute, and the SHA-256 of every parameter's bytes (tests/golden/seam_<case>.json).

`build(case)` rebuilds that module tree with the same class layout as model.py (Linear :129-158,
Gate :569-589, Expert :592-611, MoE :614-632), fills it with the seeded bytes of shard_b200.synth,
and checks every parameter against the recorded dtype, shape and hash, so the tree the seam is
installed on holds exactly what the reference module held. Its MoE.forward (the forward `install`
captures as the fallback) is a stand-in that counts its calls.
"""
from __future__ import annotations

import hashlib
import json
import os
import types

import torch
from torch import nn

from make_golden import case_config
from shard_b200 import formats as F
from shard_b200 import synth as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

_DTYPES = {str(d): d for d in (torch.bfloat16, torch.float32, torch.int32, torch.float4_e2m1fn_x2,
                               torch.float8_e4m3fn, torch.float8_e8m0fnu)}


def load_record(case):
    with open(os.path.join(GOLDEN, f"seam_{case}.json")) as f:
        return json.load(f)


class Linear(nn.Module):
    """model.py:129-158: weight [out, in] (fp4 packed [out, in/2]), `weight.scale is self.scale`."""

    def __init__(self, in_features, out_features, wdtype, wshape, sdtype, sshape):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(*wshape, dtype=wdtype), requires_grad=False)
        self.weight.scale = self.scale = nn.Parameter(torch.empty(*sshape, dtype=sdtype), requires_grad=False)


class Expert(nn.Module):
    """model.py:592-611 (w1, w2, w3 and swiglu_limit)."""

    def __init__(self, lins, swiglu_limit):
        super().__init__()
        self.w1, self.w2, self.w3 = lins
        self.swiglu_limit = swiglu_limit


class Gate(nn.Module):
    """model.py:569-589 (score routing: weight and bias; no tid2eid)."""

    def __init__(self, g, wshape, bshape):
        super().__init__()
        self.dim, self.topk, self.score_func = g["dim"], g["topk"], g["score_func"]
        self.route_scale, self.hash = g["route_scale"], g["hash"]
        self.weight = nn.Parameter(torch.empty(*wshape, dtype=torch.bfloat16), requires_grad=False)
        self.bias = nn.Parameter(torch.empty(*bshape, dtype=torch.float32), requires_grad=False)


class MoE(nn.Module):
    """model.py:614-632. forward is the reference forward `install` captures; here it only counts
    its calls (a declined call lands here)."""

    fallback_calls = 0

    def __init__(self, rec, gate, experts, shared):
        super().__init__()
        m = rec["moe"]
        self.layer_id, self.dim = m["layer_id"], m["dim"]
        self.n_routed_experts, self.n_activated_experts = m["n_routed_experts"], m["n_activated_experts"]
        self.experts_start_idx, self.experts_end_idx = m["experts_start_idx"], m["experts_end_idx"]
        self.gate = gate
        self.experts = nn.ModuleList(experts)
        self.shared_experts = shared

    def forward(self, x, input_ids):
        type(self).fallback_calls += 1
        return torch.zeros_like(x)


def _sha(t):
    return hashlib.sha256(t.detach().contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def _linear(rec, name, packed, scale, fmt, ts):
    """A Linear holding the canonical bytes `packed` / `scale` in the reference's dtypes."""
    p = rec["params"]
    wd, sd = p[f"{name}.weight"], p[f"{name}.scale"]
    li = rec["linears"][name]
    lin = Linear(li["in_features"], li["out_features"], _DTYPES[wd["dtype"]], wd["shape"], _DTYPES[sd["dtype"]],
                 sd["shape"])
    with torch.no_grad():
        lin.weight.view(torch.uint8).copy_(packed.view(torch.uint8))
        if fmt == F.FMT_FP8:
            lin.scale.view(torch.uint8).copy_(F.e8m0_encode(scale))
        else:
            lin.scale.view(torch.uint8).copy_(scale.view(torch.uint8))
    if li["tensor_scale"] is not None:
        lin.weight.tensor_scale = float(ts)
    return lin


def _expert(rec, prefix, fmt, ew, inter):
    if fmt == F.FMT_FP8:
        bi = inter // 128
        w1 = _linear(rec, f"{prefix}.w1", ew.w13[:inter], ew.w13_s[:bi], fmt, 1.0)
        w3 = _linear(rec, f"{prefix}.w3", ew.w13[inter:], ew.w13_s[bi:], fmt, 1.0)
    else:
        w1 = _linear(rec, f"{prefix}.w1", ew.w13[:inter], ew.w13_s[:inter], fmt, ew.w13_ts[0])
        w3 = _linear(rec, f"{prefix}.w3", ew.w13[inter:], ew.w13_s[inter:], fmt, ew.w13_ts[1])
    w2 = _linear(rec, f"{prefix}.w2", ew.w2, ew.w2_s, fmt, ew.w2_ts[0])
    return Expert((w1, w2, w3), rec["swiglu_limit"])


def _zero_shared(rec, inter, hidden):
    """The "no shared expert" stand-in of the golden generator: zero FP8 weights, unit scales."""
    lins = []
    for name, (n, k) in (("w1", (inter, hidden)), ("w2", (hidden, inter)), ("w3", (inter, hidden))):
        lins.append(_linear(rec, f"shared_experts.{name}", torch.zeros(n, k, dtype=torch.uint8),
                            torch.ones(n // 128, k // 128), F.FMT_FP8, 1.0))
    w1, w2, w3 = lins
    return Expert((w1, w2, w3), rec["swiglu_limit"])


def build(case):
    """(stand-in model module, its MoE instance on the CPU) for a recorded seam case. Raises
    AssertionError if any parameter differs from the reference module's recorded dtype, shape or bytes."""
    rec = load_record(case)
    cfg, m, xs, sfmt = case_config(case)
    h, i = cfg.hidden, cfg.inter
    gw, gb = S.make_gate(cfg)
    p = rec["params"]
    gate = Gate(rec["gate"], p["gate.weight"]["shape"], p["gate.bias"]["shape"])
    with torch.no_grad():
        gate.weight.copy_(gw)
        gate.bias.copy_(gb)
    experts = [_expert(rec, f"experts.{e}", cfg.expert_fmt, S.make_expert(cfg, 0, e), i)
               for e in range(cfg.n_experts)]
    if cfg.n_shared:
        shared = _expert(rec, "shared_experts", F.FMT_FP8, S.make_expert(cfg, 0, -1, F.FMT_FP8), i)
    else:
        shared = _zero_shared(rec, i, h)
    moe = MoE(rec, gate, experts, shared)
    got = {n: (str(t.dtype), list(t.shape), _sha(t)) for n, t in moe.named_parameters()}
    want = {n: (d["dtype"], d["shape"], d["sha"]) for n, d in p.items()}
    assert set(got) == set(want), f"parameter names differ: {sorted(set(got) ^ set(want))[:6]}"
    bad = [n for n in want if got[n] != want[n]]
    assert not bad, f"parameters differ from the reference module's: {bad[:6]}"
    for name, li in rec["linears"].items():
        sub = moe.get_submodule(name)
        assert (sub.weight.scale is sub.scale) == li["weight_scale_is_scale"]
        assert getattr(sub.weight, "tensor_scale", None) == li["tensor_scale"]
    mod = types.ModuleType("model")
    mod.MoE, mod.Gate, mod.Expert, mod.Linear = MoE, Gate, Expert, Linear
    g = rec["module"]
    mod.world_size, mod.rank, mod.scale_fmt = g["world_size"], g["rank"], g["scale_fmt"]
    mod.block_size, mod.fp4_block_size = g["block_size"], g["fp4_block_size"]
    mod.scale_dtype = torch.float8_e8m0fnu if g["scale_dtype"] == str(torch.float8_e8m0fnu) else torch.float32
    return mod, moe
