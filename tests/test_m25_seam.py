"""The MiniMax-M2.5 MoE seam (shard_b200.m25): a stand-in with the shape of
engines/minimax_m25/m25_stage.py (module-level `raw`, `E/K/H/I`, `NORM_TOPK`, `ROUTED_SCALE`, and a
`Layer` whose `mlp`/`mlp_b` call the MoE), filled with a synthetic ModelOpt-NVFP4 checkpoint.

CPU: install/uninstall and the decline of CPU tensors to the previous method.
GPU: the B200 MoE behind Layer.mlp against the oracle restating the M2.5 routing (bf16 router
logits, sigmoid, e_score_correction_bias for selection, renormalise per norm_topk_prob, times
routed_scaling_factor): top-k bit-exact, outputs within max relative error 1e-2."""
import types

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from shard_b200 import formats as F
from shard_b200 import m25

TOL = 1e-2


def checkpoint(h, e, i, seed, li=0):
    g = torch.Generator().manual_seed(seed)
    ck = {}
    pm = f"model.layers.{li}.block_sparse_moe."
    ck[pm + "gate.weight"] = (torch.randn(e, h, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    pop = 1.0 / np.arange(1, e + 1) ** 1.1
    ck[pm + "e_score_correction_bias"] = torch.from_numpy((0.05 * np.log(pop / pop.sum())).astype(np.float32))
    for x in range(e):
        for name, (n, k) in (("w1", (i, h)), ("w3", (i, h)), ("w2", (h, i))):
            w = (torch.randn(n, k, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)
            p, s, ts = F.quant_nvfp4(w)
            base = f"{pm}experts.{x}.{name}."
            ck[base + "weight"] = p
            ck[base + "weight_scale"] = s.view(torch.float8_e4m3fn) if s.dtype == torch.uint8 else s
            ck[base + "weight_scale_2"] = torch.tensor(ts, dtype=torch.float32)
            ck[base + "input_scale"] = torch.tensor(1.0, dtype=torch.float32)
    return ck


def stage_module(ck, h, e, k, i, norm_topk=True, routed_scale=1.0, device="cpu"):
    mod = types.ModuleType("m25_stage")
    mod.raw = lambda n: ck[n]
    mod.E, mod.K, mod.H, mod.I = e, k, h, i
    mod.NORM_TOPK, mod.ROUTED_SCALE = norm_topk, routed_scale

    class Layer:
        def __init__(self, li):
            self.li = li
            self.gate = mod.raw(f"model.layers.{li}.block_sparse_moe.gate.weight").to(torch.bfloat16).to(device)

        def mlp(self, x):
            return x * 3 - 1            # the stand-in for vLLM's FusedMoE path

        def mlp_b(self, x):
            return x * 3 - 1

    mod.Layer = Layer
    return mod


def oracle_layer(ck, h, e, k, i, norm_topk, routed_scale, li=0):
    pm = f"model.layers.{li}.block_sparse_moe."

    def expert(x):
        t = [ck[f"{pm}experts.{x}.{n}.{s}"] for n in ("w1", "w3", "w2") for s in ("weight", "weight_scale",
                                                                                   "weight_scale_2")]
        u8 = lambda z: z.view(torch.uint8).numpy()
        return (np.concatenate([u8(t[0]), u8(t[3])]), np.concatenate([u8(t[1]), u8(t[4])]),
                np.array([float(t[2]), float(t[5])], np.float32), u8(t[6]), u8(t[7]),
                np.array([float(t[8])], np.float32))

    return O.OracleLayer(hidden=h, inter=i, topk=k, score_func="sigmoid", route_scale=routed_scale,
                         swiglu_limit=0.0, expert_fmt=O.FMT_NVFP4, gate_w=ck[pm + "gate.weight"].float().numpy(),
                         gate_b=ck[pm + "e_score_correction_bias"].numpy(), expert=expert, pow2=True,
                         logits_bf16=True, renormalize=norm_topk)


def test_install_declines_cpu_tensors_and_uninstalls():
    h, e, k, i = 256, 8, 2, 128
    mod = stage_module(checkpoint(h, e, i, seed=3), h, e, k, i)
    ref = mod.Layer.mlp
    assert m25.install(mod) and not m25.install(mod)
    layer = mod.Layer(0)
    x = torch.randn(1, 3, h).to(torch.bfloat16)
    assert torch.equal(layer.mlp(x), x * 3 - 1)
    assert layer._b200_declined == {"not-on-cuda": 1}
    assert m25.uninstall(mod) and mod.Layer.mlp is ref and not m25.uninstall(mod)


@pytest.mark.gpu
@pytest.mark.parametrize("dims,norm,scale,m", [((512, 32, 8, 256), True, 2.5, 6),
                                                ((512, 32, 4, 256), False, 1.0, 9),
                                                ((3072, 256, 8, 1536), True, 1.0, 4)])
def test_m25_mlp_matches_the_oracle(dims, norm, scale, m):
    h, e, k, i = dims
    ck = checkpoint(h, e, i, seed=h + e)
    mod = stage_module(ck, h, e, k, i, norm_topk=norm, routed_scale=scale, device="cuda")
    m25.install(mod)
    try:
        layer = mod.Layer(0)
        g = torch.Generator().manual_seed(m)
        x = torch.randn(1, m, h, generator=g, dtype=torch.float32).to(torch.bfloat16)
        y = layer.mlp(x.cuda())
        yb = layer.mlp_b(x.cuda())
        lay = layer._b200_moe
        _, w, idx = lay.forward(x.reshape(m, h).cuda(), routing=True)
        torch.cuda.synchronize()
        ref, rw, ridx = O.moe_forward(oracle_layer(ck, h, e, k, i, norm, scale), x.reshape(m, h).float().numpy())
        assert np.array_equal(idx.cpu().numpy(), ridx), "router top-k must be bit-exact"
        assert np.abs(w.cpu().numpy() - rw).max() < 1e-5
        err = O.max_rel_err(y.reshape(m, h).float().cpu().numpy(), ref)
        assert err < TOL, f"max rel err {err:.3e}"
        assert torch.equal(y, yb)
        assert lay.device_error() == 0
        # the same tokens through the prefill kernel and the tensor-core gate (bf16 router logits,
        # NORM_TOPK / ROUTED_SCALE, no shared expert)
        lay.prefill = 2
        y2, w2, idx2 = lay.forward(x.reshape(m, h).cuda(), routing=True)
        torch.cuda.synchronize()
        lay.prefill = 0
        assert np.array_equal(idx2.cpu().numpy(), ridx), "prefill path: router top-k must be bit-exact"
        assert np.abs(w2.cpu().numpy() - rw).max() < 1e-5
        err2 = O.max_rel_err(y2.float().cpu().numpy(), ref)
        assert err2 < TOL, f"prefill path: max rel err {err2:.3e}"
        assert lay.device_error() == 0
    finally:
        m25.uninstall(mod)
