"""The oracle is pinned before it is trusted: restated known-answer tests of the reference's format
arithmetic, the reference's own recorded kernel outputs, and the reference's own MoE.forward outputs
for every golden case (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from cases import CASES, SeededLayer, case_config, case_inputs, expert_shas, load_golden
from oracle import moe_oracle as O
from shard_b200 import formats as F
from shard_b200 import synth as S

KAT = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "kat_formats.npz"))


# ── restated KATs (tests/test_v4_ref_cpu.py:41-151 of the reference) ─────────────────────────────

def test_pow2_scale_exact_at_powers_of_two():
    """amax = 448 * 2^k must give exactly 2^k (the frexp rule), for the oracle and the host quantiser."""
    ks = np.arange(-6, 7)
    amax = (448.0 * 2.0 ** ks).astype(np.float32)[:, None]
    assert np.array_equal(O.pow2_ceil(amax, np.float32(1) / O.FP8_MAX)[:, 0], (2.0 ** ks).astype(np.float32))
    got = F.pow2_ceil_scale(torch.from_numpy(amax), 1.0 / 448.0)[:, 0].numpy()
    assert np.array_equal(got, (2.0 ** ks).astype(np.float32))
    # and the reference kernel's own scales for the same blocks
    exact = O.bf16_from_bits(KAT["exact_bits"])
    _, s = O.act_quant(exact, 128, pow2=True)
    assert np.array_equal(s, KAT["s_exact"])


def test_act_quant_matches_reference_kernel():
    a = O.bf16_from_bits(KAT["a_bits"])
    for pow2, qk, sk in ((True, "q_pow2", "s_pow2"), (False, "q_fp32", "s_fp32")):
        q, s = O.act_quant(a, 128, pow2=pow2)
        assert np.array_equal(s, KAT[sk])
        assert np.array_equal(O.E4M3[q], O.E4M3[KAT[qk]])


def test_act_quant_zero_block_is_safe():
    q, s = O.act_quant(np.zeros((1, 128), np.float32), 128, True)
    assert np.all(O.E4M3[q] == 0) and np.all(np.isfinite(s)) and s[0, 0] > 0


def test_e2m1_ties_to_even():
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0])
    want = [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0]
    for sign in (1.0, -1.0):
        codes = F.e2m1_encode(mids * sign)
        vals = O.E2M1_SIGNED[codes.numpy()]
        assert vals.tolist() == [sign * v for v in want]


def test_nibble_order_low_first():
    packed = np.array([[0x71, 0x0F]], dtype=np.uint8)      # k0=code1(0.5) k1=code7(6) k2=code15(-6) k3=0
    assert O.unpack_fp4(packed).tolist() == [[0.5, 6.0, -6.0, 0.0]]
    t = F.pack_fp4(torch.tensor([[1, 7, 15, 0]]))
    assert t.tolist() == [[0x71, 0x0F]]


def test_e4m3_encode_matches_torch_cast():
    x = torch.linspace(-448, 448, 20001, dtype=torch.float32)
    x = torch.cat([x, torch.tensor([0.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 464.0 / 2, 0.001953125])])
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = O.e4m3_encode(x.numpy())
    assert np.array_equal(O.E4M3[got], O.E4M3[ref])


def test_bf16_round_matches_torch():
    x = torch.randn(100000) * 100
    ref = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(x.numpy()), ref)


def test_mxfp4_quantiser_matches_reference_fp4_act_quant():
    w = O.bf16_from_bits(KAT["w_bits"])
    p, s = F.quant_mxfp4(torch.from_numpy(w).to(torch.bfloat16))
    assert np.array_equal(p.numpy(), KAT["w_packed"])
    assert np.array_equal(s.numpy(), KAT["w_scale"])


def test_fp4_and_fp8_gemm_match_reference_stand_ins():
    """fp4_gemm / fp8_gemm: dequant -> fp32 matmul -> bf16, against the reference stand-ins' bytes."""
    da = O.dequant_act(KAT["q_pow2"], KAT["s_pow2"])
    wd = O.dequant_weight(O.FMT_MXFP4, KAT["w_packed"], KAT["w_scale"])
    c = O.bf16_round(da @ wd.T)
    ref = O.bf16_from_bits(KAT["c_fp4_bits"])
    assert O.max_rel_err(c, ref) < 1e-2
    da8 = O.dequant_act(KAT["q_fp32"], KAT["s_fp32"])
    wd8 = O.dequant_weight(O.FMT_FP8, KAT["w8"], KAT["w8s"])
    c8 = O.bf16_round(da8 @ wd8.T)
    assert O.max_rel_err(c8, O.bf16_from_bits(KAT["c_fp8_bits"])) < 1e-2


def test_nvfp4_roundtrip_is_on_grid_and_close():
    w = (torch.randn(64, 256) * 0.02).bfloat16()
    p, s, ts = F.quant_nvfp4(w)
    dq = O.dequant_weight(O.FMT_NVFP4, p.numpy(), s.numpy(), ts)
    err = np.abs(dq - w.float().numpy()).max() / np.abs(w.float().numpy()).max()
    assert err < 1.0 / 6.0 + 1e-3          # half the widest e2m1 gap (4 -> 6) of the block max
    # the host dequant and the oracle dequant agree bit for bit
    assert np.array_equal(F.dequant_weight(F.FMT_NVFP4, p, s, ts).numpy(), dq)


# ── the reference's own MoE.forward outputs ─────────────────────────────────────────────────────

FAST = [c for c in CASES if not c.startswith(("c1", "c3"))]


@pytest.mark.parametrize("name", FAST + ["c3_fp8_m2", "c1_nvfp4_m4"])
def test_oracle_matches_reference_moe_forward(name):
    g = load_golden(name)
    cfg, m, xs, sfmt = case_config(name)
    x, _ = case_inputs(cfg, m, xs)
    assert S.tensor_sha(x) == str(g["x_sha"]), "the seeded inputs drifted from the golden's"
    layer = SeededLayer(cfg, pow2=sfmt is not None)
    shas = expert_shas(g)
    y, w, idx = O.moe_forward(layer.oracle(), x.float().numpy(), workers=4)
    for e in sorted(set(idx.ravel().tolist()))[:4]:
        ew = layer.expert(e)
        assert S.tensor_sha(ew.w13, ew.w13_s, ew.w13_ts, ew.w2, ew.w2_s, ew.w2_ts) == shas[str(e)]
    assert np.array_equal(idx, g["indices"]), "router top-k must be bit-exact"
    assert np.abs(w - g["weights"]).max() < 1e-5
    yref = O.bf16_from_bits(g["y_bits"])
    assert O.max_rel_err(y, yref) < 1e-2
    # nearly every element is the same bf16 word; the rest are fp32 summation-order ulps
    assert (y != yref).mean() < 0.01


def test_permutation_is_grouped_by_ascending_expert_then_token():
    idx = np.array([[3, 1], [1, 0], [3, 2]])
    counts, offs, tok, slot, active = O.permutation(idx, 5)
    assert counts.tolist() == [1, 2, 1, 2, 0]
    assert offs.tolist() == [0, 1, 3, 4, 6, 6]
    assert tok.tolist() == [1, 0, 1, 2, 0, 2]
    assert slot.tolist() == [1, 1, 0, 1, 0, 0]
    assert active.tolist() == [0, 1, 2, 3]
