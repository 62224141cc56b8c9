"""The C-ABI library on the host (no GPU work): it loads, exports every entry point the public header
declares, and validates shapes, pointers and workspaces before any launch, returning the documented
status codes (include/shard_b200.h). Every call here returns before touching the device."""
import ctypes
import os
import re

import pytest

from shard_b200 import _lib
from shard_b200 import formats as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "shard_b200.h")
FAKE = ctypes.c_void_p(1 << 12)   # an aligned address that is never dereferenced by these calls


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(sb_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_with_matching_abi():
    L = _lib.lib()
    assert L.sb_abi_version() == _lib.ABI_VERSION


def test_every_declared_entry_point_is_exported_and_bound():
    names = header_functions()
    assert len(names) >= 15, names
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in the header but not exported"
        assert n in _lib.SIGNATURES, f"{n} exported but has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_tiled_sizes_match_the_canonical_sizes():
    L = _lib.lib()
    n, k = 4096, 2048
    assert L.sb_tiled_bytes(F.FMT_NVFP4, n, k) == n * k // 2
    assert L.sb_tiled_bytes(F.FMT_MXFP4, n, k) == n * k // 2
    assert L.sb_tiled_bytes(F.FMT_FP8, n, k) == n * k
    assert L.sb_tiled_scale_bytes(F.FMT_NVFP4, 0, n, k) == n * k // 16
    assert L.sb_tiled_scale_bytes(F.FMT_MXFP4, 0, n, k) == n * k // 32
    # FP8 block scales: tensor-core layout keeps 16 bytes per 128x128 block (2 scales + 2 pads)
    assert L.sb_tiled_scale_bytes(F.FMT_FP8, _lib.KIND_TC, n, k) == (n // 128) * (k // 128) * 16


def _layer(layout=_lib.LAYOUT_TC, hidden=4096, inter=2048, n_experts=256, topk=8, fmt=F.FMT_NVFP4):
    d = _lib.SbMoeLayer()
    d.hidden, d.inter, d.n_experts, d.topk = hidden, inter, n_experts, topk
    d.expert_fmt, d.has_shared, d.score_func, d.act_pow2 = fmt, 1, 1, 1
    d.route_scale, d.swiglu_limit = 1.0, 0.0
    for f in ("gate_w", "w13", "w13_s", "w13_ts", "w2", "w2_s", "w2_ts", "sh_w13", "sh_w13_s", "sh_w2", "sh_w2_s"):
        setattr(d, f, FAKE.value)
    d.layout = layout
    return d


def test_workspace_sizes_grow_with_m_and_reject_bad_layers():
    L = _lib.lib()
    for layout in (_lib.LAYOUT_FRAGMENT, _lib.LAYOUT_TC):
        d = _layer(layout)
        sizes = [L.sb_moe_workspace_bytes(ctypes.byref(d), m) for m in (1, 16, 64, 256)]
        assert all(s > 0 for s in sizes) and sizes == sorted(sizes)
    bad = _layer(hidden=100)
    assert L.sb_moe_workspace_bytes(ctypes.byref(bad), 16) == 0
    assert L.sb_qgemm_workspace_bytes(F.FMT_FP8, _lib.LAYOUT_FRAGMENT, 4096, 4096, 16) == 0
    # the dense GEMM's workspace serves every m' <= m (its narrow batches split K and add fp32
    # partials), so it never shrinks as m grows
    for fmt in (F.FMT_NVFP4, F.FMT_FP8):
        for n, k in ((4096, 4096), (512, 7168), (32768, 1024)):
            sizes = [L.sb_qgemm_workspace_bytes(fmt, _lib.LAYOUT_TC, n, k, m) for m in range(1, 100)]
            assert sizes[0] > 0 and sizes == sorted(sizes), (fmt, n, k)
            assert L.sb_qgemm_workspace_bytes(fmt, _lib.LAYOUT_TC, n, k, 1024) >= sizes[-1]


def test_workspace_serves_every_smaller_batch_across_the_prefill_switch():
    """A workspace sized for m serves every m' <= m: under the default kernel choice the size at m
    covers the verify kernel's largest batch below the switch to the hybrid dispatch and the hybrid
    dispatch at m; the hybrid dispatch's own size covers the batches before its shared expert moves
    to the prefill kernel."""
    L = _lib.lib()
    for e, k in ((16, 4), (256, 8), (384, 8)):
        d = _layer(n_experts=e, topk=k)
        sizes = {}
        top = max(16 * e // k, 512) + 40
        for mode in (0, 1, 2, 3):
            d.prefill = mode
            sizes[mode] = [L.sb_moe_workspace_bytes(ctypes.byref(d), m) for m in range(1, top)]
            assert all(s > 0 for s in sizes[mode])
            assert sizes[mode] == sorted(sizes[mode]), (e, k, mode)
        switch = -(-4 * e // k)                          # first m the default sends to the hybrid dispatch
        for m in range(1, len(sizes[0]) + 1):
            below = max(sizes[1][:min(m, switch - 1)] or [0])
            assert sizes[0][m - 1] >= below
            assert sizes[0][m - 1] >= (sizes[3][m - 1] if m >= switch else sizes[1][m - 1])
    d = _layer()
    d.prefill = 4
    assert L.sb_moe_workspace_bytes(ctypes.byref(d), 16) == 0
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, None) == -1


def _msg():
    return _lib.lib().sb_last_error().decode()


def test_forward_validates_before_launching():
    L = _lib.lib()
    st = None
    d = _layer(hidden=100)
    rc = L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, st)
    assert rc == -2 and "hidden" in _msg()
    d = _layer(topk=0)
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, st) == -2
    d = _layer(fmt=7)
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, st) == -3
    d = _layer()
    d.layout = 5
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, st) == -1
    d = _layer()
    d.w13 = None
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, 1 << 30, st) == -1
    d = _layer()
    need = L.sb_moe_workspace_bytes(ctypes.byref(d), 16)
    rc = L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, need - 1, st)
    assert rc == -4 and "workspace" in _msg()
    rc = L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, None, need, st)
    assert rc == -4
    # hash routing needs token ids
    d.tid2eid, d.vocab = FAKE.value, 1000
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 16, None, FAKE, None, None, FAKE, need, st) == -1
    # m == 0 is a no-op
    d = _layer()
    assert L.sb_moe_forward(ctypes.byref(d), FAKE, 0, None, FAKE, None, None, None, 0, st) == 0
    # misaligned activations
    d = _layer()
    assert L.sb_moe_forward(ctypes.byref(d), ctypes.c_void_p((1 << 12) + 4), 16, None, FAKE, None, None, FAKE,
                            need, st) == -1


def test_kernel_seam_entry_points_validate():
    L = _lib.lib()
    # qgemm: n must be a multiple of 32, the tensor-core layout a multiple of 128 and a workspace
    assert L.sb_qgemm(F.FMT_FP8, _lib.LAYOUT_FRAGMENT, FAKE, FAKE, None, 100, 512, FAKE, FAKE, 4, FAKE, None, 0,
                      None) == -2
    assert L.sb_qgemm(F.FMT_NVFP4, _lib.LAYOUT_FRAGMENT, FAKE, FAKE, None, 256, 512, FAKE, FAKE, 4, FAKE, None, 0,
                      None) == -1   # NVFP4 without its tensor scale
    assert L.sb_qgemm(F.FMT_FP8, _lib.LAYOUT_TC, FAKE, FAKE, None, 160, 512, FAKE, FAKE, 4, FAKE, FAKE, 1 << 20,
                      None) == -2
    assert L.sb_qgemm(F.FMT_FP8, _lib.LAYOUT_TC, FAKE, FAKE, None, 256, 512, FAKE, FAKE, 4, FAKE, FAKE, 16,
                      None) == -4
    assert L.sb_qgemm(9, _lib.LAYOUT_TC, FAKE, FAKE, None, 256, 512, FAKE, FAKE, 4, FAKE, FAKE, 1 << 20, None) == -3
    # act_quant: k must be a multiple of 128
    assert L.sb_act_quant(FAKE, 4, 100, 1, FAKE, FAKE, None) == -2
    assert L.sb_act_quant(FAKE, 0, 128, 1, FAKE, FAKE, None) == 0
    # tiling: unknown kind, W13 with an odd intermediate size, TC layout with n % 128 != 0
    assert L.sb_tile_weights(F.FMT_FP8, 2, FAKE, FAKE, 1, 256, 512, None) == -1
    assert L.sb_tile_weights(F.FMT_FP8, _lib.MAT_W13, FAKE, FAKE, 1, 96, 512, None) == -2
    assert L.sb_tile_weights(F.FMT_FP8, _lib.MAT_PLAIN | _lib.KIND_TC, FAKE, FAKE, 1, 96, 512, None) == -2
    assert L.sb_tile_scales(F.FMT_NVFP4, _lib.MAT_PLAIN, None, FAKE, 1, 256, 512, None) == -1
    assert L.sb_selftest_formats(None, None) == -1


@pytest.mark.parametrize("call", ["route", "forward"])
def test_bad_m_is_rejected(call):
    L = _lib.lib()
    d = _layer()
    f = L.sb_moe_route if call == "route" else None
    if call == "route":
        rc = f(ctypes.byref(d), FAKE, -1, None, None, None, FAKE, 1 << 30, None)
    else:
        rc = L.sb_moe_forward(ctypes.byref(d), FAKE, -1, None, FAKE, None, None, FAKE, 1 << 30, None)
    assert rc == -2


def _host_layer(shared_scale, fp8_experts=False, prefill=0):
    """A MoELayer over host tensors in the tiled form (its constructor makes no library call then)."""
    import torch
    from shard_b200.moe import MoELayer
    e, h, i = 4, 256, 128
    u8 = lambda n: torch.zeros(n, dtype=torch.uint8)
    sc = torch.full((16,), shared_scale, dtype=torch.float32).view(torch.uint8)
    fmt = F.FMT_FP8 if fp8_experts else F.FMT_NVFP4
    ex_s = sc.repeat(e) if fp8_experts else u8(64)
    return MoELayer(hidden=h, inter=i, n_experts=e, topk=2, expert_fmt=fmt, gate_w=torch.zeros(e, h),
                    w13=u8(64), w13_s=ex_s, w2=u8(64), w2_s=ex_s, w13_ts=torch.ones(e, 2), w2_ts=torch.ones(e),
                    shared=(u8(64), sc, u8(64), sc), tiled=True, prefill=prefill)


def test_non_power_of_two_fp8_scales_keep_the_verify_kernel():
    """The prefill kernel's bf16 weight operand is exact only for power-of-two FP8 block scales: the
    default choice resolves to the verify kernel otherwise; an explicit choice stands."""
    assert _host_layer(2.0 ** -7).prefill == 0
    lay = _host_layer(0.3)
    assert not lay.prefill_exact and lay.prefill == 1
    assert _host_layer(0.3, prefill=2).prefill == 2
    assert _host_layer(0.3, fp8_experts=True).prefill == 1
    lay = _host_layer(0.25, fp8_experts=True)
    assert lay.prefill_exact and lay.prefill == 0
    with pytest.raises(ValueError):
        lay.prefill = 4


def _k3_layer():
    d = _layer(hidden=512, inter=256, n_experts=16, topk=4, fmt=F.FMT_MXFP4)
    d.has_shared = 0
    d.mode = _lib.MODE_K3
    d.situ_beta, d.situ_linear_beta = 2.0, 4.0
    d.gate_w = None   # K3 takes the caller's routing: no gate needed
    return d


def test_k3_mode_is_validated_before_launching():
    """sb_moe_forward_routed (KimiSparseMoeBlock.moe_infer's seam): the layer and the call are checked
    on the host, with no device work; each refusal names its reason."""
    L = _lib.lib()
    d = _k3_layer()
    need = L.sb_moe_workspace_bytes(ctypes.byref(d), 8)
    assert need > 0
    # a V4-mode layer does not take the caller's routing, a K3-mode one only takes it
    v4 = _layer()
    rc = L.sb_moe_forward_routed(ctypes.byref(v4), FAKE, 8, FAKE, FAKE, FAKE, FAKE, 1 << 30, None)
    assert rc == -6 and "K3-mode layers" in _msg()
    rc = L.sb_moe_forward(ctypes.byref(d), FAKE, 8, None, FAKE, None, None, FAKE, 1 << 30, None)
    assert rc == -6 and "sb_moe_forward_routed" in _msg()
    # K3 needs routing weights
    rc = L.sb_moe_forward_routed(ctypes.byref(d), FAKE, 8, FAKE, None, FAKE, FAKE, 1 << 30, None)
    assert rc == -1
    # the layer constraints: MXFP4 experts, no shared expert, situ_beta > 0, linear beta >= 0
    for field, value in (("expert_fmt", F.FMT_NVFP4), ("has_shared", 1), ("situ_beta", 0.0),
                         ("situ_linear_beta", -1.0)):
        bad = _k3_layer()
        setattr(bad, field, value)
        if field == "has_shared":
            for f in ("sh_w13", "sh_w13_s", "sh_w2", "sh_w2_s"):
                setattr(bad, f, FAKE.value)
        assert L.sb_moe_workspace_bytes(ctypes.byref(bad), 8) == 0, field
        rc = L.sb_moe_forward_routed(ctypes.byref(bad), FAKE, 8, FAKE, FAKE, FAKE, FAKE, 1 << 30, None)
        assert rc == -6 and "K3 mode" in _msg(), field
    # a mode that does not exist
    bad = _k3_layer()
    bad.mode = 7
    assert L.sb_moe_workspace_bytes(ctypes.byref(bad), 8) == 0
    # the workspace bound is checked like sb_moe_forward's
    rc = L.sb_moe_forward_routed(ctypes.byref(d), FAKE, 8, FAKE, FAKE, FAKE, FAKE, need - 1, None)
    assert rc == -4 and "workspace" in _msg()
