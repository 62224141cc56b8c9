"""Seeded synthetic MoE layers and inputs for the benchmark configurations c0-c4.

No checkpoint and no dataset is involved: every weight is drawn from a seeded generator and
quantised with `shard_b200.formats`, every activation is bf16 N(0, 1). Each weight matrix has its own
generator, seeded from (config seed, layer, expert, matrix), so an expert can be generated alone
(the parity tests only materialise the experts a batch routes to) and comes out the same bytes
whichever order experts are generated in.

Configurations (the reference's MoE shapes; V4-Flash is H=4096, I=2048, 256 experts):
  c0  H=512  E=16  k=4 I=256  shared, sigmoid, NVFP4 experts (MXFP4 twin), M=8, seed 0
  c1  H=4096 E=256 k=8 I=2048 shared, sigmoid, NVFP4 experts, M in {1,8,32,64}, seed 1
  c2  48 layers of c1, pipeline-partitioned, M=16 chunks, seed 1
  c3  H=3072 E=256 k=8 I=1536 no shared, FP8 experts, Zipf(1.1) selection bias, M in {1,16,64}, seed 2
  c4  H=7168 E=384 k=8 I=2048 shared, NVFP4 experts, Zipf(1.1), M in {256,1024}, seed 3
"""
from __future__ import annotations

import dataclasses
import hashlib
import math
from typing import Optional, Sequence

import torch

from . import formats as F


@dataclasses.dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    n_experts: int
    topk: int
    inter: int
    n_shared: int = 1
    expert_fmt: int = F.FMT_NVFP4
    shared_fmt: int = F.FMT_FP8
    score_func: str = "sigmoid"        # "softmax" | "sigmoid" | "sqrtsoftplus"
    route_scale: float = 1.0
    swiglu_limit: float = 0.0
    zipf_s: Optional[float] = None     # selection skew through the gate bias
    gate_init: str = "uniform"         # "uniform" | "normal"
    seed: int = 0
    ms: Sequence[int] = (8,)

    def replace(self, **kw) -> "MoEConfig":
        return dataclasses.replace(self, **kw)


CONFIGS = {
    "c0": MoEConfig("c0", 512, 16, 4, 256, seed=0, ms=(8,)),
    "c1": MoEConfig("c1", 4096, 256, 8, 2048, seed=1, ms=(1, 8, 32, 64)),
    "c3": MoEConfig("c3", 3072, 256, 8, 1536, n_shared=0, expert_fmt=F.FMT_FP8, zipf_s=1.1,
                    gate_init="normal", seed=2, ms=(1, 16, 64)),
    "c4": MoEConfig("c4", 7168, 384, 8, 2048, zipf_s=1.1, gate_init="normal", seed=3, ms=(256, 1024)),
}

# Selection bias strength for the Zipf configs: bias_e = ZIPF_BETA * log(p_e). The sigmoid scores
# of these gates spread over roughly +-0.25, so this makes the selection frequency fall off with
# popularity rank the way a Zipf(1.1) law does over the top few dozen experts.
ZIPF_BETA = 0.06


def _seed(*tags) -> int:
    h = hashlib.sha256(repr(tags).encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def _gen(device, *tags) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(_seed(*tags))
    return g


def _randn_bf16(shape, std, device, *tags):
    g = _gen(device, *tags)
    return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


@dataclasses.dataclass
class ExpertWeights:
    """One expert's three matrices in the canonical (reference) layout, quantised."""
    w13: torch.Tensor          # fp4: uint8 [2I, H/2] (w1 rows then w3 rows); fp8: uint8 [2I, H]
    w13_s: torch.Tensor        # nvfp4: uint8 e4m3 [2I, H/16]; mxfp4: uint8 e8m0 [2I, H/32]; fp8: f32 [2I/128, H/128]
    w13_ts: torch.Tensor       # f32 [2] tensor scales of w1, w3 (1.0 unless NVFP4)
    w2: torch.Tensor
    w2_s: torch.Tensor
    w2_ts: torch.Tensor        # f32 [1]


def _quant(fmt, w):
    if fmt == F.FMT_NVFP4:
        p, s, ts = F.quant_nvfp4(w)
        return p, s, ts
    if fmt == F.FMT_MXFP4:
        p, s = F.quant_mxfp4(w)
        return p, s, 1.0
    if fmt == F.FMT_FP8:
        p, s = F.quant_fp8_block(w)
        return p, s, 1.0
    raise ValueError(fmt)


def expert_bf16(cfg: MoEConfig, layer: int, expert: int, device="cpu"):
    """The unquantised bf16 draws (w1 [I,H], w3 [I,H], w2 [H,I]) of one expert; expert -1 = shared."""
    h, i = cfg.hidden, cfg.inter
    w1 = _randn_bf16((i, h), 0.02, device, cfg.seed, layer, expert, "w1")
    w3 = _randn_bf16((i, h), 0.02, device, cfg.seed, layer, expert, "w3")
    w2 = _randn_bf16((h, i), 0.02, device, cfg.seed, layer, expert, "w2")
    return w1, w3, w2


def make_expert(cfg: MoEConfig, layer: int, expert: int, fmt: Optional[int] = None, device="cpu") -> ExpertWeights:
    fmt = cfg.expert_fmt if fmt is None else fmt
    w1, w3, w2 = expert_bf16(cfg, layer, expert, device)
    p1, s1, t1 = _quant(fmt, w1)
    p3, s3, t3 = _quant(fmt, w3)
    p2, s2, t2 = _quant(fmt, w2)
    return ExpertWeights(
        w13=torch.cat([p1, p3]).contiguous(), w13_s=torch.cat([s1, s3]).contiguous(),
        w13_ts=torch.tensor([t1, t3], dtype=torch.float32, device=device),
        w2=p2, w2_s=s2, w2_ts=torch.tensor([t2], dtype=torch.float32, device=device))


def zipf_popularity(cfg: MoEConfig) -> torch.Tensor:
    """Zipf(s) popularity over experts, ranks assigned by a seeded permutation."""
    e = cfg.n_experts
    rank = torch.randperm(e, generator=_gen("cpu", cfg.seed, "zipf-rank"))
    p = 1.0 / (rank.double() + 1.0) ** cfg.zipf_s
    return (p / p.sum()).float()


def make_gate(cfg: MoEConfig, layer: int = 0, device="cpu"):
    """(gate weight bf16 [E, H], selection bias fp32 [E])."""
    e, h = cfg.n_experts, cfg.hidden
    g = _gen(device, cfg.seed, layer, "gate")
    if cfg.gate_init == "uniform":
        a = 0.02 * math.sqrt(3.0)
        w = ((torch.rand(e, h, generator=g, device=device, dtype=torch.float32) * 2 - 1) * a).to(torch.bfloat16)
    else:
        w = (torch.randn(e, h, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    if cfg.zipf_s is not None:
        bias = (ZIPF_BETA * torch.log(zipf_popularity(cfg))).to(device)
    else:
        bias = torch.zeros(e, dtype=torch.float32, device=device)
    return w, bias.float()


def make_inputs(cfg: MoEConfig, m: int, step: int = 0, device="cpu"):
    """x bf16 [M, H] ~ N(0,1) and input_ids int64 [M] for one forward."""
    g = _gen("cpu", cfg.seed, "x", m, step)
    x = torch.randn(m, cfg.hidden, generator=g, dtype=torch.float32).to(torch.bfloat16)
    ids = torch.randint(0, 129280, (m,), generator=g)
    return x.to(device), ids.to(device)


def tensor_sha(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        t = t.detach().contiguous().cpu()
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.float32
                 else t.numpy().tobytes())
    return h.hexdigest()


# ── device layers ─────────────────────────────────────────────────────────────────────────────

def _random_canonical(fmt, n_mat, n, k, device, gen):
    """Valid random canonical bytes (values and scales) for experts whose values no test reads."""
    if fmt == F.FMT_FP8:
        w = torch.randint(0, 255, (n_mat, n, k), dtype=torch.uint8, device=device, generator=gen)
        w = torch.where((w & 0x7F) == 0x7F, w ^ 1, w)
        s = torch.ldexp(torch.ones(n_mat, n // 128, k // 128, device=device),
                        torch.randint(-8, -4, (n_mat, n // 128, k // 128), device=device, generator=gen))
        return w, s
    w = torch.randint(0, 256, (n_mat, n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    if fmt == F.FMT_NVFP4:
        s = torch.randint(0x20, 0x38, (n_mat, n, k // 16), dtype=torch.uint8, device=device, generator=gen)
    else:
        s = torch.randint(118, 124, (n_mat, n, k // 32), dtype=torch.uint8, device=device, generator=gen)
    return w, s


def normal_expert(cfg: MoEConfig, layer: int, expert: int, device="cuda") -> ExpertWeights:
    """The canonical bytes of one expert of a fill="normal" device layer (regenerated: the same
    generator seeds give the same draws and the same quantisation)."""
    return _normal_expert_on_device(cfg, layer, expert, cfg.expert_fmt, device)


def _normal_expert_on_device(cfg, layer, expert, fmt, device):
    """N(0, 0.02) draws quantised on the device (fast path for benchmark layers)."""
    h, i = cfg.hidden, cfg.inter
    g = _gen(device, cfg.seed, layer, expert, "dev")
    w1 = (torch.randn(i, h, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn(i, h, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(h, i, generator=g, device=device) * 0.02).to(torch.bfloat16)
    p1, s1, t1 = _quant(fmt, w1)
    p3, s3, t3 = _quant(fmt, w3)
    p2, s2, t2 = _quant(fmt, w2)
    return ExpertWeights(torch.cat([p1, p3]), torch.cat([s1, s3]),
                         torch.tensor([t1, t3], dtype=torch.float32, device=device),
                         p2, s2, torch.tensor([t2], dtype=torch.float32, device=device))


def device_layer(cfg: MoEConfig, layer: int = 0, device="cuda", seeded=None, fill="random", act_pow2=True,
                 layout=None, prefill=0):
    """A MoELayer on `device` for config `cfg`.

    seeded: expert ids generated from their CPU-seeded draws (the bytes the oracle and the golden
            vectors use); None means all of them.
    fill:   how the other experts are made: "random" (valid random bytes, for experts no check
            reads) or "normal" (N(0, 0.02) drawn and quantised on the device, for benchmarks).
    prefill: expert-kernel choice on the tensor-core layout (0 by batch size, 1 verify, 2 prefill).
    The shared expert and the gate are always the seeded ones."""
    from .moe import MoELayer
    e, h, i, fmt = cfg.n_experts, cfg.hidden, cfg.inter, cfg.expert_fmt
    seeded = set(range(e)) if seeded is None else set(int(v) for v in seeded)
    gw, gb = make_gate(cfg, layer)
    if fmt == F.FMT_FP8:
        w13 = torch.empty(e, 2 * i, h, dtype=torch.uint8, device=device)
        w13_s = torch.empty(e, 2 * i // 128, h // 128, dtype=torch.float32, device=device)
        w2 = torch.empty(e, h, i, dtype=torch.uint8, device=device)
        w2_s = torch.empty(e, h // 128, i // 128, dtype=torch.float32, device=device)
    else:
        g = 16 if fmt == F.FMT_NVFP4 else 32
        w13 = torch.empty(e, 2 * i, h // 2, dtype=torch.uint8, device=device)
        w13_s = torch.empty(e, 2 * i, h // g, dtype=torch.uint8, device=device)
        w2 = torch.empty(e, h, i // 2, dtype=torch.uint8, device=device)
        w2_s = torch.empty(e, h, i // g, dtype=torch.uint8, device=device)
    w13_ts = torch.ones(e, 2, dtype=torch.float32, device=device)
    w2_ts = torch.ones(e, dtype=torch.float32, device=device)
    rest = [x for x in range(e) if x not in seeded]
    if rest and fill == "random":
        gen = _gen(device, cfg.seed, layer, "filler")
        a, b = _random_canonical(fmt, len(rest), 2 * i, h, device, gen)
        c, d = _random_canonical(fmt, len(rest), h, i, device, gen)
        idx = torch.tensor(rest, device=device)
        w13[idx], w13_s[idx], w2[idx], w2_s[idx] = a, b, c, d
        if fmt == F.FMT_NVFP4:
            w13_ts[idx] = 1e-3
            w2_ts[idx] = 1e-3
        del a, b, c, d
    for x in range(e):
        if x in seeded:
            ew = make_expert(cfg, layer, x)
        elif fill == "normal":
            ew = _normal_expert_on_device(cfg, layer, x, fmt, device)
        else:
            continue
        w13[x].copy_(ew.w13)
        w13_s[x].copy_(ew.w13_s)
        w2[x].copy_(ew.w2)
        w2_s[x].copy_(ew.w2_s)
        w13_ts[x].copy_(ew.w13_ts)
        w2_ts[x].copy_(ew.w2_ts.reshape(()))
    shared = None
    if cfg.n_shared:
        sh = make_expert(cfg, layer, -1, F.FMT_FP8)
        shared = tuple(t.to(device) for t in (sh.w13, sh.w13_s, sh.w2, sh.w2_s))
    lay = MoELayer(hidden=h, inter=i, n_experts=e, topk=cfg.topk, expert_fmt=fmt, gate_w=gw.to(device),
                   gate_bias=gb.to(device), score_func=cfg.score_func, route_scale=cfg.route_scale,
                   swiglu_limit=cfg.swiglu_limit, act_pow2=act_pow2, w13=w13, w13_s=w13_s,
                   w13_ts=w13_ts if fmt == F.FMT_NVFP4 else None, w2=w2, w2_s=w2_s,
                   w2_ts=w2_ts if fmt == F.FMT_NVFP4 else None, shared=shared, layout=layout,
                   prefill=prefill)
    del w13, w13_s, w2, w2_s
    return lay
