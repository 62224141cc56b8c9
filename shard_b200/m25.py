"""The MiniMax-M2.5 engine's MoE on the B200: a drop-in for `Layer.mlp` / `Layer.mlp_b` of
engines/minimax_m25/m25_stage.py (paths relative to the leyten/shard tree).

There, a layer's MoE is vLLM's NVFP4 `FusedMoE` (m25_stage.py:288-311), fed bf16 router logits
`F.linear(h, self.gate)` (:412-416, :547-553), scoring "sigmoid", `e_score_correction_bias` for
selection only, `renormalize=norm_topk_prob`, `routed_scaling_factor`, no shared expert. This module
builds the same layer as a `shard_b200.moe.MoELayer` straight from the checkpoint tensors
`_build_moe` reads (`model.layers.{li}.block_sparse_moe.gate.weight`, `.e_score_correction_bias`,
`.experts.{e}.{w1,w3,w2}.{weight, weight_scale, weight_scale_2}`: ModelOpt NVFP4, e2m1 packed low
nibble first, e4m3 scale per 16, fp32 global scale) and runs it through the C ABI.

Routing is restated from those call sites: logits rounded to bf16, sigmoid in fp32, selection by
score + bias (ties to the lower id), weights from the unbiased scores, renormalised when the
config says so, times routed_scaling_factor. The experts compute like the V4 path (e4m3
activations with one power-of-two scale per 128 K); vLLM's NVFP4 FusedMoE quantises activations its
own way (not vendored, so not pinned here).

    import shard_b200.m25 as m25
    m25.install(m25_stage)      # after the stage module is imported; Layer.mlp -> the B200 MoE
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import formats as F
from .moe import MoELayer

_REF = {}


def _u8(t):
    return t.contiguous().view(torch.uint8)


def layer_from_checkpoint(raw: Callable[[str], torch.Tensor], li: int, n_experts: int, topk: int, hidden: int,
                          inter: int, norm_topk: bool = True, routed_scale: float = 1.0, device=None,
                          act_pow2: bool = True, layout=None) -> MoELayer:
    """The MoE of layer `li` from checkpoint tensors (`raw(name)`, as m25_stage.raw)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    pm = f"model.layers.{li}.block_sparse_moe."
    pe = pm + "experts."
    gate = raw(pm + "gate.weight").to(torch.bfloat16).to(dev).contiguous()
    bias = raw(pm + "e_score_correction_bias").float().to(dev).contiguous()

    def proj(e, name):
        p = f"{pe}{e}.{name}."
        w = _u8(raw(p + "weight")).to(dev)
        s = _u8(raw(p + "weight_scale")).to(dev)
        g = float(raw(p + "weight_scale_2").float().reshape(-1)[0])
        return w, s, g

    w13, w13_s, w13_ts, w2, w2_s, w2_ts = [], [], [], [], [], []
    for e in range(n_experts):
        a, sa, ga = proj(e, "w1")
        b, sb, gb = proj(e, "w3")
        c, sc, gc = proj(e, "w2")
        assert a.shape == (inter, hidden // 2) and sa.shape == (inter, hidden // 16), "w1: ModelOpt NVFP4 shapes"
        assert c.shape == (hidden, inter // 2) and sc.shape == (hidden, inter // 16), "w2: ModelOpt NVFP4 shapes"
        w13.append(torch.cat([a, b]))
        w13_s.append(torch.cat([sa, sb]))
        w13_ts.append(torch.tensor([ga, gb], dtype=torch.float32))
        w2.append(c)
        w2_s.append(sc)
        w2_ts.append(torch.tensor([gc], dtype=torch.float32))
    return MoELayer(hidden=hidden, inter=inter, n_experts=n_experts, topk=topk, expert_fmt=F.FMT_NVFP4,
                    gate_w=gate, gate_bias=bias, score_func="sigmoid", route_scale=routed_scale,
                    act_pow2=act_pow2, w13=torch.stack(w13), w13_s=torch.stack(w13_s),
                    w13_ts=torch.stack(w13_ts).to(dev), w2=torch.stack(w2), w2_s=torch.stack(w2_s),
                    w2_ts=torch.stack(w2_ts).to(dev), layout=layout, logits_bf16=True, renormalize=norm_topk)


def _layer_of(mod, layer):
    lay = getattr(layer, "_b200_moe", None)
    if lay is None:
        lay = layer._b200_moe = layer_from_checkpoint(
            mod.raw, layer.li, mod.E, mod.K, mod.H, mod.I, norm_topk=bool(getattr(mod, "NORM_TOPK", True)),
            routed_scale=float(getattr(mod, "ROUTED_SCALE", 1.0)), device=layer.gate.device)
    return lay


def _decline(layer, why):
    tally = getattr(layer, "_b200_declined", None)
    if tally is None:
        tally = layer._b200_declined = {}
    tally[why] = tally.get(why, 0) + 1


def install(mod) -> bool:
    """Rebind mod.Layer.mlp and mod.Layer.mlp_b (m25_stage.py:412-416, :547-553) to the B200 MoE;
    the previous methods stay the fallback (CPU tensors). Idempotent."""
    L = mod.Layer
    if getattr(L.mlp, "_b200", False):
        return False
    ref_mlp = L.mlp
    ref_mlp_b = getattr(L, "mlp_b", None)
    _REF[id(mod)] = (ref_mlp, ref_mlp_b)

    def mlp(self, x):
        if not x.is_cuda:
            _decline(self, "not-on-cuda")
            return ref_mlp(self, x)
        shp = x.shape
        lay = _layer_of(mod, self)
        y = lay.forward(x.reshape(-1, mod.H).to(torch.bfloat16))
        self._b200_steps = getattr(self, "_b200_steps", 0) + 1
        return y.to(x.dtype).view(shp)

    def mlp_b(self, x):
        # the batched path: one MoE call over all B*s tokens (row-invariant kernels, so this equals
        # the per-stream calls bit for bit)
        return mlp(self, x)

    mlp._b200 = True
    L.mlp = mlp
    if ref_mlp_b is not None:
        L.mlp_b = mlp_b
    return True


def uninstall(mod) -> bool:
    L = mod.Layer
    if not getattr(L.mlp, "_b200", False):
        return False
    ref_mlp, ref_mlp_b = _REF.pop(id(mod))
    L.mlp = ref_mlp
    if ref_mlp_b is not None:
        L.mlp_b = ref_mlp_b
    return True
