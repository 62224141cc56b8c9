"""The operator seam on the reference's own MoE module layout (model.py:614-649), rebuilt from the
recorded seam fixtures (tests/seam_mirror.py): `shard_b200.moe.install(mod)` rebinds MoE.forward,
and the installed forward reads the module's float4_e2m1fn_x2 / float8_e4m3fn weights, its
float8_e8m0fnu / e4m3 `.weight.scale` and NVFP4 `weight.tensor_scale` (layout via
layer_from_module), as the reference's levers do (engines/deepseek_v4/v4_moe_grouped.py:736-755;
hardware tests tests/test_v4_moe_grouped.py:1061-1153)."""
import numpy as np
import pytest
import torch

import seam_mirror
from cases import case_config, case_inputs, load_golden
from oracle import moe_oracle as O
from shard_b200 import moe as sbm

CASES = ["c0_mxfp4_m8", "c0_nvfp4_m8", "small_fp8_noshared_m16"]
TOL = 1e-2


@pytest.mark.parametrize("case", CASES)
def test_fixture_rebuilds_the_reference_module(case):
    """Every parameter of the rebuilt module has the recorded dtype, shape and bytes (checked inside
    build), and on CPU tensors the installed forward declines to the captured forward, tallied."""
    mod, moe = seam_mirror.build(case)
    cfg, m, xs, _ = case_config(case)
    assert sbm.install(mod)
    try:
        assert not sbm.install(mod), "a second install must be refused"
        x, ids = case_inputs(cfg, m, xs)
        before = seam_mirror.MoE.fallback_calls
        y = moe(x.view(1, m, cfg.hidden), ids.view(1, m))
        assert seam_mirror.MoE.fallback_calls == before + 1
        assert torch.equal(y, torch.zeros_like(y))
        assert sbm.coverage(moe) == {0: (0, {"not-on-cuda": 1})}
    finally:
        assert sbm.uninstall(mod)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_installed_forward_on_the_reference_module(case):
    """The drop-in itself: install(mod), move the module to the B200, call MoE.forward. Top-k indices
    bit-exact and y within 1e-2 of the reference's own MoE.forward output recorded for the case;
    coverage shows the step ran on the B200 with no declines."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = load_golden(case)
    mod, moe = seam_mirror.build(case)
    moe.cuda()
    cfg, m, xs, _ = case_config(case)
    x, ids = case_inputs(cfg, m, xs)
    assert sbm.install(mod)
    try:
        before = seam_mirror.MoE.fallback_calls
        with torch.no_grad():
            y = moe(x.view(1, m, cfg.hidden).cuda(), ids.view(1, m).cuda())
        torch.cuda.synchronize()
        assert y.shape == (1, m, cfg.hidden) and y.dtype == torch.bfloat16 and y.is_cuda
        assert seam_mirror.MoE.fallback_calls == before, "the reference forward must not run"
        assert sbm.coverage(moe) == {0: (1, {})}
        layer = moe._b200_layer
        assert layer.device_error() == 0
        w, idx = layer.route(x.cuda())
        assert np.array_equal(idx.cpu().numpy(), g["indices"]), "router top-k indices must be bit-exact"
        assert np.abs(w.cpu().numpy() - g["weights"]).max() < 1e-5
        err = O.max_rel_err(y.view(m, cfg.hidden).float().cpu().numpy(), O.bf16_from_bits(g["y_bits"]))
        assert err < TOL, f"{case}: max rel err {err:.3e}"
        # a second call reuses the laid-out layer
        with torch.no_grad():
            y2 = moe(x.view(1, m, cfg.hidden).cuda(), ids.view(1, m).cuda())
        assert torch.equal(y, y2)
        assert sbm.coverage(moe) == {0: (2, {})}
    finally:
        assert sbm.uninstall(mod)
