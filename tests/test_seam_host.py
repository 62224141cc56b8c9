"""The drop-in seams on the host: shard_b200.moe.install rebinds a reference-shaped module's
MoE.forward and declines (tallied, like v4_moe_grouped._decline, v4_moe_grouped.py:736-755) the cases
the B200 forward does not take: world_size > 1 and CPU tensors; the kernel seam exposes the
reference `kernel` module's entry points with its argument names (kernel.py:105-125, 257-273,
518-536). No GPU work."""
import inspect
import types

import pytest
import torch

from shard_b200 import moe as M
from shard_b200 import ops


def _reference_shaped_module():
    mod = types.ModuleType("model")

    class MoE(torch.nn.Module):
        def __init__(self, layer_id):
            super().__init__()
            self.layer_id = layer_id
            self.dim = 8
            self.experts = torch.nn.ModuleList()
            self.experts_start_idx, self.experts_end_idx = 0, 0

        def forward(self, x, input_ids):
            return x * 2 + 1

    mod.MoE = MoE
    mod.world_size = 1
    mod.scale_fmt = "ue8m0"
    return mod


@pytest.fixture()
def seam():
    mod = _reference_shaped_module()
    ref = mod.MoE.forward
    assert M.install(mod)
    yield mod, ref
    M.uninstall(mod)


def test_install_rebinds_and_is_idempotent(seam):
    mod, ref = seam
    assert mod.MoE.forward is not ref
    assert getattr(mod.MoE.forward, "_b200", False)
    assert not M.install(mod)         # second install is a no-op


def test_uninstall_restores_the_previous_forward():
    mod = _reference_shaped_module()
    ref = mod.MoE.forward
    assert M.install(mod)
    assert M.uninstall(mod)
    assert mod.MoE.forward is ref
    assert not M.uninstall(mod)


def test_cpu_tensors_decline_to_the_previous_forward(seam):
    mod, _ = seam
    layer = mod.MoE(3)
    x = torch.randn(2, 5, 8)
    y = layer(x, torch.zeros(2, 5, dtype=torch.long))
    assert torch.equal(y, x * 2 + 1)
    assert M.coverage(layer) == {3: (0, {"not-on-cuda": 1})}


def test_world_size_above_one_declines(seam):
    mod, _ = seam
    mod.world_size = 2
    layer = mod.MoE(0)
    x = torch.randn(1, 3, 8)
    for _ in range(2):
        assert torch.equal(layer(x, torch.zeros(1, 3, dtype=torch.long)), x * 2 + 1)
    assert M.coverage(layer) == {0: (0, {"world_size>1": 2})}


def test_kernel_seam_signatures_match_the_reference():
    # names and order of the reference's parameters (kernel.py:105, :257, :518)
    assert list(inspect.signature(ops.act_quant).parameters) == ["x", "block_size", "scale_fmt", "scale_dtype",
                                                                 "inplace"]
    assert list(inspect.signature(ops.fp8_gemm).parameters) == ["a", "a_s", "b", "b_s", "scale_dtype"]
    assert list(inspect.signature(ops.fp4_gemm).parameters) == ["a", "a_s", "b", "b_s", "scale_dtype"]


def test_kernel_seam_rejects_non_contiguous_inputs():
    a = torch.zeros(4, 256, dtype=torch.float8_e4m3fn).t()
    b = torch.zeros(256, 128, dtype=torch.float8_e4m3fn)
    s = torch.ones(1, 1)
    with pytest.raises(AssertionError):
        ops.fp8_gemm(a, s, b, s)
