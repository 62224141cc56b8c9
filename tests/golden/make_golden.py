"""Generate the golden vectors that pin the oracle (and through it the CUDA path) to the reference.

Run here, where the leyten/shard tree is readable, NEVER on the GPU box:

    python tests/golden/make_golden.py --ref <path to leyten/shard checkout>

It imports the reference's own CPU oracle (engines/deepseek_v4/v4_ref_cpu.load_ref, which executes
vendor/deepseek_v4_ref/inference/model.py on the engines/deepseek_v4/v4_kernels_cpu stand-ins),
builds reference `MoE` modules, fills them with the seeded weights of `shard_b200.synth`, and records
the reference's outputs for the same seeded inputs:

  moe_<case>.npz   y (bf16 bits), routing weights, top-k indices, gate logits, and the SHA-256 of the
                   inputs and of every expert's quantised bytes (so a consumer can prove it
                   regenerated the same bytes before comparing outputs).
  kat_formats.npz  the reference's act_quant / fp4_act_quant / fp4_gemm / fp8_gemm on small inputs.

NVFP4 experts have no in-tree reference kernel. For those cases the script rebinds the reference
module's `fp4_gemm` to the CPU stand-in's own structure (dequant -> fp32 matmul -> default dtype)
with only the weight dequant swapped to e2m1 * e4m3(scale per 16) * fp32 tensor scale; every other
operation is the reference's.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, REPO)

from shard_b200 import formats as F  # noqa: E402
from shard_b200 import synth as S  # noqa: E402

CASES = {
    # name: (base config, overrides, M, x scale, layer id, act scale format)
    "c0_nvfp4_m8": ("c0", {}, 8, 1.0, "ue8m0"),
    "c0_mxfp4_m8": ("c0", {"expert_fmt": F.FMT_MXFP4}, 8, 1.0, "ue8m0"),
    "c0_mxfp4_m1": ("c0", {"expert_fmt": F.FMT_MXFP4}, 1, 1.0, "ue8m0"),
    "c0_nvfp4_m33": ("c0", {}, 33, 1.0, "ue8m0"),
    "c0_mxfp4_fp32scale_m8": ("c0", {"expert_fmt": F.FMT_MXFP4}, 8, 1.0, None),
    "v4route_nvfp4_m8": ("c0", {"score_func": "sqrtsoftplus", "route_scale": 1.5, "swiglu_limit": 10.0,
                                "gate_init": "normal"}, 8, 24.0, "ue8m0"),
    "softmax_mxfp4_m5": ("c0", {"score_func": "softmax", "expert_fmt": F.FMT_MXFP4, "swiglu_limit": 10.0},
                         5, 24.0, "ue8m0"),
    "small_fp8_noshared_m16": ("c0", {"hidden": 256, "inter": 128, "n_shared": 0, "expert_fmt": F.FMT_FP8,
                                      "zipf_s": 1.1, "gate_init": "normal", "seed": 7}, 16, 1.0, "ue8m0"),
    "c1_nvfp4_m4": ("c1", {}, 4, 1.0, "ue8m0"),
    "c3_fp8_m2": ("c3", {}, 2, 1.0, "ue8m0"),
    # a c4-shaped layer with 16 experts: 128 routed tokens per expert on average (Zipf-skewed, some
    # experts over one 128-token pass), the shape where the prefill kernel is the default choice
    "c4e16_nvfp4_m256": ("c4", {"n_experts": 16}, 256, 1.0, "ue8m0"),
}

# Cases whose reference module is also recorded as a seam fixture (seam_<case>.json): the module's
# structure, attributes, parameter dtypes and shapes, and the SHA-256 of every parameter's bytes.
SEAM_CASES = ("c0_mxfp4_m8", "c0_nvfp4_m8", "small_fp8_noshared_m16")


def case_config(name):
    base, over, m, xscale, sfmt = CASES[name]
    cfg = S.CONFIGS[base].replace(**over)
    return cfg, m, xscale, sfmt


def case_inputs(cfg, m, xscale):
    x, ids = S.make_inputs(cfg, m)
    if xscale != 1.0:
        x = (x.float() * xscale).to(torch.bfloat16)
    return x, ids


def _load_reference(ref_root):
    eng = os.path.join(ref_root, "engines", "deepseek_v4")
    sys.path.insert(0, eng)
    os.environ.setdefault("V4_KERNELS", "cpu")
    import v4_ref_cpu  # noqa: E402  (the reference's own loader)
    import v4_kernels_cpu  # noqa: E402
    mod = v4_ref_cpu.load_ref()
    return mod, v4_kernels_cpu


def _patch_nvfp4(mod, K):
    """Rebind the reference module's fp4_gemm so an e4m3-scaled (NVFP4) weight dequantises as
    e2m1 * scale16 * tensor_scale; MXFP4 weights still go to the reference stand-in."""
    orig = mod.fp4_gemm

    def fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32):
        if b_s.dtype != torch.float8_e4m3fn:
            return orig(a, a_s, b, b_s, scale_dtype)
        k, n = a.size(-1), b.size(0)
        da = K._dequant(a.reshape(-1, k), a_s.reshape(-1, a_s.size(-1)), 128)
        db = K.unpack_fp4(b).float() * b_s.float().repeat_interleave(16, -1)[:, :k]
        db = db * b.tensor_scale
        c = da @ db.t()
        return c.view(*a.shape[:-1], n).to(torch.get_default_dtype())

    mod.fp4_gemm = fp4_gemm
    return orig


def _fill_linear(lin, fmt, packed, scale, ts):
    with torch.no_grad():
        lin.weight.data.view(torch.uint8).copy_(packed)
        if fmt == F.FMT_MXFP4:
            lin.scale.data.view(torch.uint8).copy_(scale)
        elif fmt == F.FMT_NVFP4:
            p = torch.nn.Parameter(scale.clone().view(torch.float8_e4m3fn), requires_grad=False)
            lin.weight.scale = lin.scale = p
            lin.weight.tensor_scale = float(ts)
        else:
            lin.scale.data.view(torch.uint8).copy_(F.e8m0_encode(scale))


def _fill_expert(expert, fmt, ew, inter):
    if fmt == F.FMT_FP8:
        bi = inter // 128
        _fill_linear(expert.w1, fmt, ew.w13[:inter], ew.w13_s[:bi], 1.0)
        _fill_linear(expert.w3, fmt, ew.w13[inter:], ew.w13_s[bi:], 1.0)
    else:
        _fill_linear(expert.w1, fmt, ew.w13[:inter], ew.w13_s[:inter], ew.w13_ts[0])
        _fill_linear(expert.w3, fmt, ew.w13[inter:], ew.w13_s[inter:], ew.w13_ts[1])
    _fill_linear(expert.w2, fmt, ew.w2, ew.w2_s, ew.w2_ts[0])


def _sha(t):
    import hashlib
    return hashlib.sha256(t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def seam_record(mod, moe):
    """What shard_b200.moe.layer_from_module and b200_moe_forward read from a reference MoE module
    (model.py:129-158 Linear, :569-589 Gate, :592-611 Expert, :614-632 MoE) and from the module that
    defines it, with every parameter's dtype, shape and byte hash."""
    def lin(l):
        return {"in_features": l.in_features, "out_features": l.out_features,
                "weight_scale_is_scale": getattr(l.weight, "scale", None) is l.scale,
                "tensor_scale": getattr(l.weight, "tensor_scale", None)}

    g = moe.gate
    rec = {
        "module": {"world_size": mod.world_size, "rank": mod.rank, "scale_fmt": mod.scale_fmt,
                   "scale_dtype": str(mod.scale_dtype), "block_size": mod.block_size,
                   "fp4_block_size": mod.fp4_block_size},
        "moe": {"layer_id": moe.layer_id, "dim": moe.dim, "n_routed_experts": moe.n_routed_experts,
                "n_activated_experts": moe.n_activated_experts, "experts_start_idx": moe.experts_start_idx,
                "experts_end_idx": moe.experts_end_idx},
        "gate": {"dim": g.dim, "topk": g.topk, "score_func": g.score_func, "route_scale": g.route_scale,
                 "hash": g.hash},
        "swiglu_limit": moe.shared_experts.swiglu_limit,
        "linears": {},
        "params": {},
    }
    for name, sub in moe.named_modules():
        if hasattr(sub, "in_features") and hasattr(sub, "weight"):
            rec["linears"][name] = lin(sub)
    for name, p in moe.named_parameters():
        rec["params"][name] = {"dtype": str(p.dtype), "shape": list(p.shape), "sha": _sha(p)}
    return rec


def run_case(mod, K, name, out_dir):
    cfg, m, xscale, sfmt = case_config(name)
    x, ids = case_inputs(cfg, m, xscale)
    h, e, k, i = cfg.hidden, cfg.n_experts, cfg.topk, cfg.inter
    mod.world_size, mod.rank = 1, 0
    mod.default_dtype = torch.float8_e4m3fn
    mod.scale_fmt = sfmt
    mod.scale_dtype = torch.float8_e8m0fnu if sfmt else torch.float32
    args = mod.ModelArgs(dim=h, moe_inter_dim=i, n_routed_experts=e, n_activated_experts=k,
                         n_shared_experts=1, n_hash_layers=0, score_func=cfg.score_func,
                         route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit, dtype="fp8",
                         scale_fmt=sfmt, scale_dtype="fp8" if sfmt else "fp32",
                         expert_dtype=None if cfg.expert_fmt == F.FMT_FP8 else "fp4")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        moe = mod.MoE(0, args)
        gw, gb = S.make_gate(cfg)
        with torch.no_grad():
            moe.gate.weight.data.copy_(gw)
            moe.gate.bias.data.copy_(gb)
        # Route first (the gate is cheap) and materialise only the routed experts at full size.
        with torch.no_grad():
            _, idx0 = moe.gate(x.view(-1, h), ids)
        routed = sorted(set(idx0.flatten().tolist())) if e > 32 else list(range(e))
        shas = {}
        mx_match = True
        for ex in routed:
            ew = S.make_expert(cfg, 0, ex)
            _fill_expert(moe.experts[ex], cfg.expert_fmt, ew, i)
            shas[str(ex)] = S.tensor_sha(ew.w13, ew.w13_s, ew.w13_ts, ew.w2, ew.w2_s, ew.w2_ts)
            if cfg.expert_fmt == F.FMT_MXFP4:
                w1, _, _ = S.expert_bf16(cfg, 0, ex)
                rp, rs = K.fp4_act_quant(w1, 32)
                mx_match &= torch.equal(rp.view(torch.uint8), ew.w13[:i]) and \
                    torch.equal(rs.view(torch.uint8), ew.w13_s[:i])
        assert mx_match, "shard_b200.formats.quant_mxfp4 disagrees with the reference fp4_act_quant"
        if cfg.n_shared:
            sh = S.make_expert(cfg, 0, -1, F.FMT_FP8)
            _fill_expert(moe.shared_experts, F.FMT_FP8, sh, i)
            shas["shared"] = S.tensor_sha(sh.w13, sh.w13_s, sh.w13_ts, sh.w2, sh.w2_s, sh.w2_ts)
        else:
            # The reference asserts exactly one shared expert (model.py:631). "No shared expert" is a
            # zero-weight shared expert: its output is +0, and adding +0 in fp32 is the identity.
            with torch.no_grad():
                for lin in (moe.shared_experts.w1, moe.shared_experts.w3, moe.shared_experts.w2):
                    lin.weight.data.view(torch.uint8).zero_()
                    lin.scale.data.view(torch.uint8).fill_(127)
        with torch.no_grad():
            logits = torch.nn.functional.linear(x.view(-1, h).float(), moe.gate.weight.float())
            wts, idx = moe.gate(x.view(-1, h), ids)
            y = moe(x.view(1, m, h), ids.view(1, m)).view(m, h)
    finally:
        torch.set_default_dtype(prev)
    if name in SEAM_CASES:
        rec = seam_record(mod, moe)
        rec["case"] = name
        with open(os.path.join(out_dir, f"seam_{name}.json"), "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)
    meta = dict(case=name, config=cfg.name, overrides=CASES[name][1], m=m, x_scale=xscale,
                scale_fmt=sfmt, layer=0, reference="leyten/shard model.py MoE.forward on v4_kernels_cpu")
    np.savez_compressed(
        os.path.join(out_dir, f"moe_{name}.npz"),
        meta=json.dumps(meta), x_sha=S.tensor_sha(x), expert_sha=json.dumps(shas),
        y_bits=y.contiguous().view(torch.int16).numpy().astype(np.uint16),
        weights=wts.float().numpy(), indices=idx.numpy().astype(np.int64),
        logits=logits.numpy())
    print(f"{name}: M={m} experts routed={len(set(idx.flatten().tolist()))} |y|max={y.float().abs().max():.4f}")


# Kimi-K3 routed-expert cases: the reference's KimiSparseMoeBlock (vendor/kimi_k3_ref/
# modeling_kimi_linear.py:782-876) with MXFP4 experts (the K3 checkpoint format, k3_moe_mxfp4.py:1-9)
# held as their exact bf16 values; its own KimiMoEGate routes, its moe_infer runs.
K3_CASES = {
    # name: (hidden, experts, top-k, intermediate, seed, M, situ beta, situ linear_beta)
    "k3_mxfp4_m8": (512, 16, 4, 256, 11, 8, 2.0, 4.0),
    "k3_mxfp4_nolb_m37": (512, 16, 4, 256, 12, 37, 1.0, None),
}


def k3_config(name):
    h, e, k, i, seed, m, beta, lb = K3_CASES[name]
    cfg = S.MoEConfig(name, h, e, k, i, n_shared=0, expert_fmt=F.FMT_MXFP4, gate_init="normal", seed=seed)
    return cfg, m, beta, lb


def _load_k3(ref_root):
    """The reference's K3 modules, imported the way its K3 engine imports them (engines/kimi_k3/
    k3_stage.py:115-141: the CPU `fla` stand-in first, then the one moved transformers symbol)."""
    import importlib
    for p in (os.path.join(ref_root, "engines", "kimi_k3"), os.path.join(ref_root, "vendor"), ref_root):
        sys.path.insert(0, p)
    import k3_kda_cpu  # noqa: E402
    k3_kda_cpu.install()
    generic = importlib.import_module("transformers.utils.generic")
    if not hasattr(generic, "OutputRecorder"):
        generic.OutputRecorder = importlib.import_module("transformers.utils.output_capturing").OutputRecorder
    from kimi_k3_ref import modeling_kimi_linear as MK  # noqa: E402
    from kimi_k3_ref.configuration_kimi_k3 import KimiLinearConfig  # noqa: E402
    return MK, KimiLinearConfig


def k3_seam_record(block):
    rec = {"top_k": block.top_k, "num_experts": block.num_experts, "ep_size": block.ep_size,
           "ep_rank": block.ep_rank, "experts_per_rank": block.experts_per_rank,
           "moe_hidden_size": block.moe_hidden_size,
           "act": {"beta": block.experts[0].act_fn.beta, "linear_beta": block.experts[0].act_fn.linear_beta},
           "linears": {}, "params": {}}
    for name, sub in block.named_modules():
        if isinstance(sub, torch.nn.Linear):
            rec["linears"][name] = {"in_features": sub.in_features, "out_features": sub.out_features}
    for name, p in block.named_parameters():
        if name.startswith("experts."):
            rec["params"][name] = {"dtype": str(p.dtype), "shape": list(p.shape), "sha": _sha(p)}
    return rec


def run_k3_case(MK, KimiLinearConfig, name, out_dir):
    cfg, m, beta, lb = k3_config(name)
    h, e, k, i = cfg.hidden, cfg.n_experts, cfg.topk, cfg.inter
    kc = KimiLinearConfig(hidden_size=h, num_experts=e, num_experts_per_token=k, moe_intermediate_size=i,
                          hidden_act="situ", activation_situ_beta=beta, activation_situ_linear_beta=lb,
                          num_shared_experts=None, moe_renormalize=True, routed_scaling_factor=2.5,
                          moe_router_activation_func="sigmoid")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        block = MK.KimiSparseMoeBlock(kc).eval()
        gw, gb = S.make_gate(cfg)
        shas = {}
        with torch.no_grad():
            block.gate.weight.copy_(gw)
            block.gate.e_score_correction_bias.copy_(gb)
            for ex in range(e):
                ew = S.make_expert(cfg, 0, ex)
                deq = [F.dequant_weight(F.FMT_MXFP4, ew.w13[:i], ew.w13_s[:i]),
                       F.dequant_weight(F.FMT_MXFP4, ew.w13[i:], ew.w13_s[i:]),
                       F.dequant_weight(F.FMT_MXFP4, ew.w2, ew.w2_s)]
                for lin, w in zip((block.experts[ex].w1, block.experts[ex].w3, block.experts[ex].w2), deq):
                    assert torch.equal(w.to(torch.bfloat16).float(), w), "MXFP4 values must be exact in bf16"
                    lin.weight.copy_(w.to(torch.bfloat16))
                shas[str(ex)] = S.tensor_sha(ew.w13, ew.w13_s, ew.w2, ew.w2_s)
        x, _ = S.make_inputs(cfg, m)
        with torch.no_grad():
            topk_idx, topk_weight = block.gate(x.view(1, m, h))
            y = block.moe_infer(x, topk_idx, topk_weight)
    finally:
        torch.set_default_dtype(prev)
    meta = dict(case=name, hidden=h, experts=e, topk=k, inter=i, seed=cfg.seed, m=m, situ_beta=beta,
                situ_linear_beta=lb, reference="leyten/shard vendor/kimi_k3_ref KimiSparseMoeBlock.moe_infer")
    np.savez_compressed(
        os.path.join(out_dir, f"{name}.npz"), meta=json.dumps(meta), x_sha=S.tensor_sha(x),
        expert_sha=json.dumps(shas), topk_idx=topk_idx.numpy().astype(np.int64),
        topk_weight=topk_weight.float().numpy(), y_bits=y.contiguous().view(torch.int16).numpy().astype(np.uint16))
    rec = k3_seam_record(block)
    rec["case"] = name
    with open(os.path.join(out_dir, f"seam_{name}.json"), "w") as f:
        json.dump(rec, f, indent=1, sort_keys=True)
    print(f"{name}: M={m} |y|max={y.float().abs().max():.4f} experts used={len(set(topk_idx.flatten().tolist()))}")


def run_kats(mod, K, out_dir):
    torch.manual_seed(11)
    a_bf = (torch.randn(5, 256) * 2).bfloat16()
    q_p2, s_p2 = K.act_quant(a_bf, 128, "ue8m0", torch.float32)
    q_f, s_f = K.act_quant(a_bf, 128, None, torch.float32)
    w_bf = (torch.randn(384, 256) * 0.02).bfloat16()
    wp, ws = K.fp4_act_quant(w_bf, 32)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        c4 = K.fp4_gemm(q_p2, s_p2, wp, ws)
        w8 = (torch.randn(384, 256) * 2).bfloat16().to(torch.float8_e4m3fn)
        w8s = (torch.rand(3, 2, dtype=torch.float32) + 0.5)
        c8 = K.fp8_gemm(q_f, s_f, w8, w8s)
    finally:
        torch.set_default_dtype(prev)
    exact = torch.zeros(13, 128, dtype=torch.bfloat16)
    for r, kk in enumerate(range(-6, 7)):
        exact[r, 0] = 448.0 * 2.0 ** kk
    _, s_exact = K.act_quant(exact, 128, "ue8m0")
    np.savez_compressed(
        os.path.join(out_dir, "kat_formats.npz"),
        a_bits=a_bf.view(torch.int16).numpy().astype(np.uint16),
        q_pow2=q_p2.view(torch.uint8).numpy(), s_pow2=s_p2.float().numpy(),
        q_fp32=q_f.view(torch.uint8).numpy(), s_fp32=s_f.float().numpy(),
        w_bits=w_bf.view(torch.int16).numpy().astype(np.uint16),
        w_packed=wp.view(torch.uint8).numpy(), w_scale=ws.view(torch.uint8).numpy(),
        c_fp4_bits=c4.view(torch.int16).numpy().astype(np.uint16),
        w8=w8.view(torch.uint8).numpy(), w8s=w8s.numpy(),
        c_fp8_bits=c8.view(torch.int16).numpy().astype(np.uint16),
        exact_bits=exact.view(torch.int16).numpy().astype(np.uint16), s_exact=s_exact.float().numpy())
    print("kat_formats: act_quant / fp4_act_quant / fp4_gemm / fp8_gemm recorded")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to the leyten/shard checkout")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*")
    a = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    only = a.only or (list(CASES) + list(K3_CASES))
    if any(n in CASES for n in only):
        mod, K = _load_reference(a.ref)
        _patch_nvfp4(mod, K)
        run_kats(mod, K, a.out)
        for name in only:
            if name in CASES:
                run_case(mod, K, name, a.out)
    if any(n in K3_CASES for n in only):
        MK, KC = _load_k3(a.ref)
        for name in only:
            if name in K3_CASES:
                run_k3_case(MK, KC, name, a.out)


if __name__ == "__main__":
    main()
