"""Kimi-K3's routed experts on the B200, behind the seam the reference's K3 engine uses.

engines/kimi_k3/k3_moe_mxfp4.py replaces exactly one method, `KimiSparseMoeBlock.moe_infer(x,
topk_ids, topk_weight)` (:405-412): the reference keeps its own router (KimiMoEGate), latent down/up
projections, norm and shared experts (:12-17), and hands the routed experts to a W4A16 MXFP4 kernel
with K3's `situ` activation installed (:177-190). `install(mod)` rebinds the same method of the
reference module (vendor/kimi_k3_ref/modeling_kimi_linear.py) to the B200 forward: the block's
experts are laid out once (MXFP4, tensor-core layout) and every later call runs
sb_moe_forward_routed in K3 mode (bf16 activations, situ, routing weights applied to the expert
outputs, slot-order sum; modeling_kimi_linear.py:850-876). Calls on CPU tensors and expert-parallel
blocks (ep_size > 1) decline to the captured method, tallied.

The experts' weights are read as the module holds them: bf16 `nn.Linear` weights whose values are
MXFP4 numbers (a dequantised K3 checkpoint) are re-encoded to MXFP4, which reproduces the same values
exactly; linears that carry the checkpoint's packed form (`weight_packed` uint8 [out, in/2] and
`weight_scale` e8m0 [out, in/32], the compressed-tensors names k3_moe_mxfp4.py:47 reads) are taken
as they are.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import formats as F
from ._lib import lib
from .moe import MoELayer


def _mxfp4(lin):
    """(packed uint8 [out, in/2], e8m0 uint8 [out, in/32]) of one expert linear."""
    wp = getattr(lin, "weight_packed", None)
    if wp is not None:
        return wp.view(torch.uint8), lin.weight_scale.view(torch.uint8)
    p, s = F.quant_mxfp4(lin.weight.detach().to(torch.bfloat16))
    return p, s


def layer_from_block(block, device: Optional[torch.device] = None) -> MoELayer:
    """Lay a reference KimiSparseMoeBlock's routed experts (modeling_kimi_linear.py:782-807) out as a
    K3-mode MoELayer: experts[i].w1 / w3 / w2 (KimiBlockSparseMLP, :242-270), the situ parameters of
    their act_fn, top_k."""
    experts = list(block.experts)
    e0 = experts[0]
    dev = device or e0.w1.weight.device
    act = e0.act_fn
    beta, linear_beta = float(getattr(act, "beta", 1.0)), getattr(act, "linear_beta", None)
    w13, w13_s, w2, w2_s = [], [], [], []
    for ex in experts:
        p1, s1 = _mxfp4(ex.w1)
        p3, s3 = _mxfp4(ex.w3)
        p2, s2 = _mxfp4(ex.w2)
        w13.append(torch.cat([p1, p3]).to(dev))
        w13_s.append(torch.cat([s1, s3]).to(dev))
        w2.append(p2.to(dev))
        w2_s.append(s2.to(dev))
    hidden, inter = e0.w1.in_features, e0.w1.out_features
    return MoELayer(hidden=hidden, inter=inter, n_experts=len(experts), topk=block.top_k, expert_fmt=F.FMT_MXFP4,
                    gate_w=None, w13=torch.stack(w13), w13_s=torch.stack(w13_s), w2=torch.stack(w2),
                    w2_s=torch.stack(w2_s), mode="k3", situ_beta=beta,
                    situ_linear_beta=None if linear_beta is None else float(linear_beta))


# ── the seam ───────────────────────────────────────────────────────────────────────────────────

_REF_INFER = None
_MOD = None


def _decline(block, why, x, topk_ids, topk_weight):
    tally = getattr(block, "_b200_declined", None)
    if tally is None:
        tally = block._b200_declined = {}
    tally[why] = tally.get(why, 0) + 1
    return _REF_INFER(block, x, topk_ids, topk_weight)


@torch.no_grad()
def b200_moe_infer(self, x, topk_ids, topk_weight):
    """KimiSparseMoeBlock.moe_infer(self, x [T, D] bf16, topk_ids [T, k], topk_weight [T, k]) -> [T, D]
    on the B200."""
    if int(getattr(self, "ep_size", 1) or 1) > 1:
        return _decline(self, "ep_size>1", x, topk_ids, topk_weight)
    if not x.is_cuda:
        return _decline(self, "not-on-cuda", x, topk_ids, topk_weight)
    layer = getattr(self, "_b200_layer", None)
    if layer is None:
        layer = self._b200_layer = layer_from_block(self, x.device)
    y = layer.forward_routed(x.to(torch.bfloat16), topk_ids, topk_weight)
    self._b200_steps = getattr(self, "_b200_steps", 0) + 1
    return y.to(x.dtype)


def install(mod) -> bool:
    """Rebind mod.KimiSparseMoeBlock.moe_infer to the B200 forward; the previous method becomes the
    fallback. Idempotent. Fails loudly if a CUDA device is present but the library is not."""
    global _REF_INFER, _MOD
    cls = mod.KimiSparseMoeBlock
    if getattr(cls.moe_infer, "_b200", False):
        return False
    if torch.cuda.is_available():
        lib()
    _REF_INFER = cls.moe_infer
    _MOD = mod
    b200_moe_infer._b200 = True
    cls.moe_infer = b200_moe_infer
    return True


def uninstall(mod) -> bool:
    global _REF_INFER
    cls = mod.KimiSparseMoeBlock
    if not getattr(cls.moe_infer, "_b200", False):
        return False
    cls.moe_infer = _REF_INFER
    _REF_INFER = None
    return True


def coverage(module):
    """{id: (steps on the B200, {decline reason: count})} for every KimiSparseMoeBlock under `module`."""
    out = {}
    for m in module.modules() if hasattr(module, "modules") else [module]:
        if hasattr(m, "experts") and hasattr(m, "moe_infer") and hasattr(m, "top_k"):
            out[len(out)] = (getattr(m, "_b200_steps", 0), dict(getattr(m, "_b200_declined", {})))
    return out
