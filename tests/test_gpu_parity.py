"""Parity of the CUDA path (through the C ABI) with the oracle and the reference's golden vectors.

Bars (the north star's): router top-k indices bit-exact; outputs within max relative error 1e-2,
measured as max|got - ref| / max|ref| over the compared tensor; act_quant bit-exact."""
import numpy as np
import pytest
import torch

from cases import CASES, SeededLayer, case_config, case_inputs, load_golden
from oracle import moe_oracle as O
from shard_b200 import formats as F
from shard_b200 import synth as S

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from shard_b200 import _lib
    _lib.lib()


def _np(t):
    return t.detach().float().cpu().numpy()


def test_device_format_decoding_matches_host_tables():
    from shard_b200._lib import check, lib, stream_ptr
    out = torch.zeros(64, dtype=torch.float32, device="cuda")
    check(lib().sb_selftest_formats(out.data_ptr(), stream_ptr()), "selftest")
    o = out.cpu().numpy()
    assert np.array_equal(o[:16], O.E2M1_SIGNED)
    e4 = np.array([0x00, 0x01, 0x07, 0x08, 0x30, 0x38, 0x3C, 0x40, 0x7E, 0x80, 0xB8, 0xFE, 0x11, 0x22, 0x55, 0x66])
    assert np.array_equal(o[16:32], O.E4M3[e4])
    e8 = np.array([127, 126, 128, 120, 134, 1, 254, 100])
    assert np.array_equal(o[32:40], np.ldexp(np.float32(1), e8 - 127).astype(np.float32))
    px = np.array([1.0, 1.5, 0.75, 1.0, 3.0e-3, 2.0, 1.0e-4 / 448.0, 0.1], dtype=np.float32)
    assert np.array_equal(o[40:48], O.pow2_ceil(px, np.float32(1.0)))
    qx = np.array([0.1, -3.3, 447.0, 17.0, 0.0009765625, -0.3, 250.0, 1.0 / 3.0], dtype=np.float32)
    assert np.array_equal(o[48:56], O.E4M3[O.e4m3_encode(qx)])


@pytest.mark.parametrize("pow2", [True, False])
@pytest.mark.parametrize("m,k", [(1, 128), (7, 512), (64, 4096)])
def test_act_quant_is_bit_exact(m, k, pow2):
    from shard_b200 import ops
    g = torch.Generator().manual_seed(m * 1000 + k)
    x = (torch.randn(m, k, generator=g) * 3).to(torch.bfloat16)
    x[0, :128] = 0                                            # an all-zero block
    if m > 2:
        x[1, 5] = 448.0 * 4                                   # a block amax at exactly 448 * 2^k
    q, s = ops.act_quant(x.cuda(), 128, "ue8m0" if pow2 else None)
    qo, so = O.act_quant(x.float().numpy(), 128, pow2)
    assert np.array_equal(s.float().cpu().numpy(), so)
    assert np.array_equal(O.E4M3[q.view(torch.uint8).cpu().numpy()], O.E4M3[qo])


LAYOUTS = [1, 0]   # tensor-core (tcgen05) layout, mma.sync fragment layout


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("fmt", [F.FMT_NVFP4, F.FMT_MXFP4, F.FMT_FP8])
@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (5, 4096, 2048), (37, 512, 4096), (8, 7168, 2048),
                                   (3, 384, 896), (64, 128, 1024)])
def test_quantised_gemm_matches_oracle(fmt, m, n, k, layout):
    """The kernel-level seam: fp4_gemm / fp8_gemm (kernel.py:257-273, 518-536). On the tensor-core
    layout every one of these narrow shapes splits K across CTAs (k = 896: a last piece of 3
    stages, an odd count)."""
    from shard_b200 import ops
    g = torch.Generator().manual_seed(n + k + fmt)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    if fmt == F.FMT_NVFP4:
        p, s, ts = F.quant_nvfp4(w)
        wdq = O.dequant_weight(O.FMT_NVFP4, p.numpy(), s.numpy(), ts)
    elif fmt == F.FMT_MXFP4:
        p, s = F.quant_mxfp4(w)
        ts = 1.0
        wdq = O.dequant_weight(O.FMT_MXFP4, p.numpy(), s.numpy())
    else:
        p, s = F.quant_fp8_block(w)
        ts = 1.0
        wdq = O.dequant_weight(O.FMT_FP8, p.numpy(), s.numpy())
    qx, sx = ops.act_quant(x.cuda(), 128, "ue8m0")
    y = ops.quantised_gemm(fmt, p.cuda(), s.cuda(), ts, qx, sx, layout=layout)
    ref = O.qlinear(x.float().numpy(), wdq, True)
    assert O.max_rel_err(_np(y), ref) < TOL
    # and nearly every element is the same bf16 word
    assert (_np(y) != ref).mean() < 0.02


# (layout, prefill): the tensor-core layout's verify kernel, prefill kernel and hybrid dispatch (at
# these sizes every routed expert is cold: the verify kernel with h in the prefill kernel's padded
# rows, and prefill launches with no items), the fragment layout
KERNELS = {"tc_verify": (1, 1), "tc_prefill": (1, 2), "tc_hybrid": (1, 3), "fragment": (0, 0)}


def _golden_layer(name, layout=None, prefill=0):
    g = load_golden(name)
    cfg, m, xs, sfmt = case_config(name)
    seeded = None if cfg.n_experts <= 32 else sorted(set(g["indices"].ravel().tolist()))
    lay = S.device_layer(cfg, 0, "cuda", seeded=seeded, act_pow2=sfmt is not None, layout=layout, prefill=prefill)
    x, ids = case_inputs(cfg, m, xs)
    return g, cfg, lay, x, ids, sfmt


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("name", list(CASES))
def test_forward_matches_reference_golden(name, kernel):
    g, cfg, lay, x, ids, sfmt = _golden_layer(name, *KERNELS[kernel])
    y, w, idx = lay.forward(x.cuda(), ids.cuda(), routing=True)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), g["indices"]), "router top-k indices must be bit-exact"
    assert np.abs(w.cpu().numpy() - g["weights"]).max() < 1e-5
    yref = O.bf16_from_bits(g["y_bits"])
    err = O.max_rel_err(_np(y), yref)
    assert err < TOL, f"{name}: max rel err {err:.3e}"
    assert lay.device_error() == 0


@pytest.mark.parametrize("name", ["c0_nvfp4_m8", "c0_mxfp4_m8", "small_fp8_noshared_m16", "v4route_nvfp4_m8"])
def test_forward_matches_oracle(name):
    g, cfg, lay, x, ids, sfmt = _golden_layer(name)
    y = lay.forward(x.cuda(), ids.cuda())
    yo, _, _ = O.moe_forward(SeededLayer(cfg, pow2=sfmt is not None).oracle(), x.float().numpy())
    assert O.max_rel_err(_np(y), yo) < TOL


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("cname,m", [("c1", 1), ("c1", 8), ("c1", 32), ("c1", 64), ("c3", 16), ("c3", 64),
                                     ("c4", 256), ("c4", 1024)])
def test_full_size_forward(cname, m, layout):
    """Full configuration shapes. The oracle checks a sample of tokens (its cost grows with the experts
    they route to); the whole batch is checked for row invariance: every token's output equals the
    same token run alone through the same kernel, bit for bit. The tensor-core layout runs both of
    its expert kernels (verify and prefill) and the hybrid dispatch (not row-invariant: an expert's
    kernel depends on its batch), and the default choice must equal the one it picks."""
    cfg = S.CONFIGS[cname]
    x, ids = S.make_inputs(cfg, m)
    gw, gb = S.make_gate(cfg)
    _, idx_o, _ = O.gate(x.float().numpy(), gw.float().numpy(), gb.numpy(), cfg.score_func, cfg.route_scale, cfg.topk)
    sample = sorted(set([0, m // 2, m - 1]))[:3]
    seeded = sorted(set(idx_o[sample].ravel().tolist()))
    lay = S.device_layer(cfg, 0, "cuda", seeded=seeded, layout=layout)
    sl = SeededLayer(cfg)
    yo, _, _ = O.moe_forward(sl.oracle(), x[sample].float().numpy(), workers=8)
    modes = [1, 2] if layout == 1 else [0]
    ys = {}
    for mode in modes:
        lay.prefill = mode
        y, w, idx = lay.forward(x.cuda(), ids.cuda(), routing=True)
        assert np.array_equal(idx.cpu().numpy(), idx_o), "router top-k indices must be bit-exact"
        err = O.max_rel_err(_np(y[sample]), yo)
        assert err < TOL, f"{cname} M={m} prefill={mode}: max rel err {err:.3e}"
        for t in sample:
            alone = lay.forward(x[t:t + 1].cuda(), ids[t:t + 1].cuda())
            assert torch.equal(alone, y[t:t + 1]), "a token's output must not depend on its batch"
        assert torch.isfinite(y.float()).all()
        assert lay.device_error() == 0
        ys[mode] = y
    if layout == 1:
        lay.prefill = 3
        y3, w3, idx3 = lay.forward(x.cuda(), ids.cuda(), routing=True)
        assert np.array_equal(idx3.cpu().numpy(), idx_o), "router top-k indices must be bit-exact"
        err = O.max_rel_err(_np(y3[sample]), yo)
        assert err < TOL, f"{cname} M={m} hybrid: max rel err {err:.3e}"
        assert torch.isfinite(y3.float()).all()
        assert lay.device_error() == 0
        assert torch.equal(lay.forward(x.cuda(), ids.cuda()), y3), "the hybrid dispatch is deterministic"
        lay.prefill = 0
        auto = lay.forward(x.cuda(), ids.cuda())
        hybrid = m * cfg.topk >= 4 * cfg.n_experts and cfg.expert_fmt != F.FMT_FP8
        assert torch.equal(auto, y3 if hybrid else ys[1])
        # the kernels sum in different orders; they agree to well within the parity bar
        assert O.max_rel_err(_np(ys[1]), _np(ys[2])) < TOL
        assert O.max_rel_err(_np(ys[1]), _np(y3)) < TOL


@pytest.mark.parametrize("cname,m", [("c1", 64), ("c3", 64), ("c4", 256), ("c4", 1024)])
def test_full_size_forward_every_token(cname, m):
    """Every token of a full-size batch against the oracle, through both tensor-core expert kernels
    and the hybrid dispatch (at c4 sizes its hot experts run on the prefill kernel, the rest on the
    verify kernel).
    The layer's experts are N(0, 0.02) draws quantised on the device (the benchmark's layers); the
    oracle regenerates the bytes of each routed expert it needs and runs its C dequant-GEMM."""
    import threading
    cfg = S.CONFIGS[cname]
    x, ids = S.make_inputs(cfg, m)
    lay = S.device_layer(cfg, 0, "cuda", seeded=[], fill="normal")
    gw, gb = S.make_gate(cfg)
    lock = threading.Lock()

    def expert(e):
        with lock:
            ew = S.normal_expert(cfg, 0, e, "cuda")
            return tuple(t.cpu().numpy() for t in (ew.w13, ew.w13_s, ew.w13_ts, ew.w2, ew.w2_s, ew.w2_ts))

    sh = S.make_expert(cfg, 0, -1, F.FMT_FP8) if cfg.n_shared else None
    ol = O.OracleLayer(hidden=cfg.hidden, inter=cfg.inter, topk=cfg.topk, score_func=cfg.score_func,
                       route_scale=cfg.route_scale, swiglu_limit=cfg.swiglu_limit, expert_fmt=cfg.expert_fmt,
                       gate_w=gw.float().numpy(), gate_b=gb.numpy(), expert=expert,
                       shared=None if sh is None else tuple(t.numpy() for t in (sh.w13, sh.w13_s, sh.w13_ts, sh.w2,
                                                                                   sh.w2_s, sh.w2_ts)))
    yo, wo, io = O.moe_forward(ol, x.float().numpy(), workers=16)
    for mode in (1, 2, 3):
        lay.prefill = mode
        y, w, idx = lay.forward(x.cuda(), ids.cuda(), routing=True)
        torch.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), io), "router top-k indices must be bit-exact"
        assert np.abs(w.cpu().numpy() - wo).max() < 1e-5
        yg = _np(y)
        # the parity bar over the whole batch: max|got - ref| / max|ref| over all M tokens
        err = O.max_rel_err(yg, yo)
        assert err < TOL, f"{cname} M={m} prefill={mode}: max rel err {err:.3e}"
        # and token by token, each row against its own max: h is re-quantised to e4m3 per 128
        # before w2, so an fp32 summation-order difference that moves one h value across an e4m3
        # rounding boundary changes it by up to 2^-4 relative; a few such flips in one row can put
        # that row's own relative error near the bar. At least 99% of the tokens stay under it
        # and none above twice it.
        rows = np.array([O.max_rel_err(yg[t], yo[t]) for t in range(m)])
        worst = int(np.argmax(rows))
        assert (rows < TOL).mean() >= 0.99, f"{cname} M={m} prefill={mode}: {(rows >= TOL).sum()} tokens over"
        assert rows[worst] < 2 * TOL, f"{cname} M={m} prefill={mode}: token {worst} max rel err {rows[worst]:.3e}"
        assert lay.device_error() == 0


@pytest.mark.parametrize("prefill", [1, 2])
def test_merged_chunks_equal_unmerged(prefill):
    """Row invariance across batch composition: two chunks run together equal each run alone."""
    cfg = S.CONFIGS["c0"]
    lay = S.device_layer(cfg, 0, "cuda", prefill=prefill)
    a, _ = S.make_inputs(cfg, 16, step=1)
    b, _ = S.make_inputs(cfg, 16, step=2)
    ya, yb = lay.forward(a.cuda()), lay.forward(b.cuda())
    yab = lay.forward(torch.cat([a, b]).cuda())
    assert torch.equal(torch.cat([ya, yb]), yab)


@pytest.mark.parametrize("prefill", [1, 2, 3])
def test_hash_routing_drops_earlier_duplicate_slots(prefill):
    """Hash layers (model.py:581-582): ids from tid2eid, repeated ids keep only the last slot
    (the reference's `y[idx] +=` semantics, v4_moe_grouped.py:98-118); through the verify kernel
    and through the prefill kernel (whose batches take the tensor-core gate for the weights)."""
    cfg = S.CONFIGS["c0"]
    sl = SeededLayer(cfg)
    lay = S.device_layer(cfg, 0, "cuda")
    vocab = 64
    tab = torch.randint(0, cfg.n_experts, (vocab, cfg.topk), generator=torch.Generator().manual_seed(3)).int()
    tab[5] = torch.tensor([3, 3, 9, 3], dtype=torch.int32)
    from shard_b200.moe import MoELayer
    hl = MoELayer(hidden=lay.hidden, inter=lay.inter, n_experts=lay.n_experts, topk=lay.topk,
                  expert_fmt=lay.expert_fmt, gate_w=lay.gate_w, gate_bias=None, tid2eid=tab.cuda(),
                  score_func="sqrtsoftplus", route_scale=1.5, w13=lay.w13, w13_s=lay.w13_s, w13_ts=lay.w13_ts,
                  w2=lay.w2, w2_s=lay.w2_s, w2_ts=lay.w2_ts, shared=lay.shared, tiled=True, prefill=prefill)
    x, _ = S.make_inputs(cfg, 8)
    ids = torch.tensor([5, 1, 2, 5, 7, 9, 11, 63])
    y, w, idx = hl.forward(x.cuda(), ids.cuda(), routing=True)
    assert torch.equal(idx.cpu(), tab[ids].long())
    ol = sl.oracle()
    ol.score_func, ol.route_scale = "sqrtsoftplus", 1.5
    # the oracle's gate on a hash layer: indices from the table, weights from the unbiased scores
    logits = x.float().numpy() @ sl.gate_w.float().numpy().T
    sp = np.where(logits > 20, logits, np.log1p(np.exp(np.minimum(logits, 20)))).astype(np.float32)
    scores = np.sqrt(sp).astype(np.float32)
    ti = tab[ids].long().numpy()
    ww = np.take_along_axis(scores, ti, 1)
    ww = (ww / ww.sum(-1, keepdims=True) * np.float32(1.5)).astype(np.float32)
    assert np.abs(w.cpu().numpy() - ww).max() < 1e-5
    yo = np.zeros((8, cfg.hidden), np.float32)
    for e in sorted(set(ti.ravel().tolist())):
        rows, slots = np.nonzero(ti == e)
        out = O.expert_forward(x.float().numpy()[rows], cfg.expert_fmt, ol.expert(e), 0.0, ww[rows, slots][:, None])
        yo[rows] = yo[rows] + out                          # repeated rows: the last write wins
    yo = O.bf16_round(yo + O.expert_forward(x.float().numpy(), F.FMT_FP8, ol.shared, 0.0))
    assert O.max_rel_err(_np(y), yo) < TOL


@pytest.mark.parametrize("fmt", [F.FMT_FP8, F.FMT_NVFP4])
def test_kernel_seam_retiles_a_new_weight_at_a_freed_address(fmt):
    """The kernel seam caches each weight's tiled copy on the weight tensor. A weight freed and
    replaced by a same-shape tensor (which the caching allocator hands the same address) must give
    the new weight's result, not the old tiled copy's; an in-place change of a weight retiles too."""
    from shard_b200 import ops
    n, k, m = 512, 1024, 4
    g = torch.Generator().manual_seed(99 + fmt)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    qx, sx = ops.act_quant(x.cuda(), 128, "ue8m0")

    def quant(seed):
        w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02).to(torch.bfloat16)
        if fmt == F.FMT_NVFP4:
            p, s, ts = F.quant_nvfp4(w)
            return p, s, ts, O.dequant_weight(O.FMT_NVFP4, p.numpy(), s.numpy(), ts)
        p, s = F.quant_fp8_block(w)
        return p, s, 1.0, O.dequant_weight(O.FMT_FP8, p.numpy(), s.numpy())

    def run(pw, ps, ts):
        return ops.quantised_gemm(fmt, pw, ps, ts, qx, sx)

    p1, s1, t1, d1 = quant(1)
    w1, ws1 = p1.cuda(), s1.cuda()
    y1 = run(w1, ws1, t1)
    addr = w1.data_ptr()
    del w1, ws1
    p2, s2, t2, d2 = quant(2)
    w2, ws2 = p2.cuda(), s2.cuda()
    y2 = run(w2, ws2, t2)
    r1 = O.qlinear(x.float().numpy(), d1, True)
    r2 = O.qlinear(x.float().numpy(), d2, True)
    assert O.max_rel_err(_np(y1), r1) < TOL
    assert O.max_rel_err(_np(y2), r2) < TOL, \
        f"stale tiled copy (same address: {addr == w2.data_ptr()})"
    # in place: the weight's version counter moves and the next call retiles
    w2.copy_(p1.cuda())
    ws2.copy_(s1.cuda())
    y3 = run(w2, ws2, t1)
    assert O.max_rel_err(_np(y3), r1) < TOL
