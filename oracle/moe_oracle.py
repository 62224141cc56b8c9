"""CPU oracle for the MoE stage forward: a numpy restatement of the reference's arithmetic.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this module: only tests/, the
`smoke()` check in __graft_entry__.py and bench.py's CPU-baseline leg may call it, and there only as
the checker (or as the timed CPU baseline), never as the thing measured on the GPU.

What it restates, and from where (paths are relative to the leyten/shard tree):
  act_quant         vendor/deepseek_v4_ref/inference/kernel.py:40-125, engines/deepseek_v4/v4_kernels_cpu.py:89-104
  pow2 scale rule   kernel.py:22-37, v4_kernels_cpu.py:65-75
  fp4/fp8 GEMMs     v4_kernels_cpu.py:158-173 (dequant to fp32, fp32 matmul, round to bf16)
  e2m1 table        v4_kernels_cpu.py:61-62, nibble order v4_kernels_cpu.py:141-155
  Gate.forward      vendor/deepseek_v4_ref/inference/model.py:569-589
  Expert.forward    model.py:601-611
  MoE.forward       model.py:634-649 (fp32 accumulator, ascending expert id, shared expert last)
  linear dispatch   model.py:114-126
  K3 moe_infer      vendor/kimi_k3_ref/modeling_kimi_linear.py:64-82 (situ), :242-270 (expert),
                    :850-876 (moe_infer), with MXFP4 experts in bf16 (the engine's W4A16 seam,
                    engines/kimi_k3/k3_moe_mxfp4.py:405-412)
NVFP4 (no in-tree reference): the weight dequant is e2m1[nibble] * e4m3(scale per 16) * fp32 tensor
scale, left to right; everything around it is the reference's order of operations.

Parity is pinned by tests/test_oracle.py against (a) the reference's own known-answer tests,
restated, and (b) tests/golden/*.npz, which tests/golden/make_golden.py produced by running the
reference's own MoE.forward on its CPU kernel stand-ins for the same seeded inputs.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

FP8_MAX = np.float32(448.0)
FP4_MAX = np.float32(6.0)
FMT_NVFP4, FMT_MXFP4, FMT_FP8 = 1, 2, 3

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_SIGNED = np.concatenate([E2M1, -E2M1]).astype(np.float32)


# ── number formats ─────────────────────────────────────────────────────────────────────────────

def _e4m3_table() -> np.ndarray:
    """All 256 e4m3fn codes -> fp32 (0x7f/0xff are NaN)."""
    out = np.zeros(256, dtype=np.float32)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 0x7
        if e == 0xF and m == 0x7:
            out[c] = np.nan
        elif e == 0:
            out[c] = s * (m / 8.0) * 2.0 ** -6
        else:
            out[c] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return out


E4M3 = _e4m3_table()
_E4M3_POS = E4M3[:127]                                      # codes 0..126, increasing
_E4M3_MID = ((_E4M3_POS[:-1].astype(np.float64) + _E4M3_POS[1:]) / 2).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 (torch's `.to(bfloat16)`)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (r.astype(np.uint32) << 16).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Values already on the bf16 grid -> their uint16 bit patterns."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(u: np.ndarray) -> np.ndarray:
    return (u.astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 (already clamped to +-448) -> e4m3 codes, nearest with ties to the even code."""
    a = np.abs(x).astype(np.float32)
    lo = np.searchsorted(_E4M3_MID, a, side="left")
    hi = np.searchsorted(_E4M3_MID, a, side="right")
    code = lo + ((hi != lo) & (lo % 2 == 1))
    return (code | (np.signbit(x) * 0x80)).astype(np.uint8)


def pow2_ceil(amax: np.ndarray, max_inv: np.float32) -> np.ndarray:
    """2^ceil(log2(amax * max_inv)), exact at powers of two (kernel.py:22-37, v4_kernels_cpu.py:65-75)."""
    x = (amax.astype(np.float32) * np.float32(max_inv)).astype(np.float32)
    mant, exp = np.frexp(x)
    exp = np.where(mant == 0.5, exp - 1, exp)
    return np.ldexp(np.float32(1.0), exp).astype(np.float32)


def act_quant(x: np.ndarray, block: int = 128, pow2: bool = True):
    """[M, K] fp32 (bf16 values) -> (e4m3 codes uint8 [M, K], fp32 scales [M, K/block]).

    kernel.py:40-125: per row per block, amax floored at 1e-4; scale = pow2 rule (scale_fmt
    'ue8m0') or amax/448; q = e4m3(clamp(x / s, +-448))."""
    m, k = x.shape
    assert k % block == 0
    z = x.astype(np.float32).reshape(m, k // block, block)
    amax = np.maximum(np.abs(z).max(-1, keepdims=True), np.float32(1e-4)).astype(np.float32)
    if pow2:
        s = pow2_ceil(amax, np.float32(1.0) / FP8_MAX)
    else:
        s = (amax * (np.float32(1.0) / FP8_MAX)).astype(np.float32)
    q = np.clip((z / s).astype(np.float32), -FP8_MAX, FP8_MAX)
    return e4m3_encode(q).reshape(m, k), s.reshape(m, k // block)


def dequant_act(q: np.ndarray, s: np.ndarray, block: int = 128) -> np.ndarray:
    return (E4M3[q] * np.repeat(s, block, axis=-1)).astype(np.float32)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    """[N, K/2] bytes -> [N, K] fp32 e2m1 values, low nibble first (v4_kernels_cpu.py:141-155)."""
    lo = E2M1_SIGNED[packed & 0x0F]
    hi = E2M1_SIGNED[packed >> 4]
    return np.stack([lo, hi], axis=-1).reshape(packed.shape[0], -1)


_CLIB = None


def _clib():
    """oracle/dequant.c through ctypes (built on first use), or None without a C compiler."""
    global _CLIB
    if _CLIB is None:
        import ctypes
        import os
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        try:
            import build_oracle
            lib = ctypes.CDLL(build_oracle.build())
        except Exception:  # noqa: BLE001  (the numpy path below is the same arithmetic)
            _CLIB = False
            return None
        finally:
            sys.path.pop(0)
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.oracle_dequant_fp4.argtypes = [ctypes.c_int, vp, vp, ctypes.c_float, i64, i64, vp]
        lib.oracle_dequant_fp8.argtypes = [vp, vp, i64, i64, vp]
        lib.oracle_qgemm.argtypes = [ctypes.c_int, vp, vp, ctypes.c_float, i64, i64, vp, i64, vp, vp]
        _CLIB = lib
    return _CLIB or None


def dequant_weight(fmt: int, packed: np.ndarray, scale: np.ndarray, ts: float = 1.0) -> np.ndarray:
    """One weight matrix -> fp32 [N, K], in the reference dequant order (v4_kernels_cpu.py:141-173).

    Runs oracle/dequant.c when it is available (the same products in fp32, computed per element),
    else the numpy expression below it."""
    lib = _clib()
    if lib is not None:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        n = packed.shape[0]
        k = packed.shape[1] * (1 if fmt == FMT_FP8 else 2)
        out = np.empty((n, k), dtype=np.float32)
        if fmt == FMT_FP8:
            sc = np.ascontiguousarray(scale, dtype=np.float32)
            rc = lib.oracle_dequant_fp8(packed.ctypes.data, sc.ctypes.data, n, k, out.ctypes.data)
        else:
            sc = np.ascontiguousarray(scale, dtype=np.uint8)
            rc = lib.oracle_dequant_fp4(fmt, packed.ctypes.data, sc.ctypes.data, float(np.float32(ts)), n, k,
                                        out.ctypes.data)
        if rc != 0:
            raise ValueError(fmt)
        return out
    return dequant_weight_np(fmt, packed, scale, ts)


def dequant_weight_np(fmt: int, packed: np.ndarray, scale: np.ndarray, ts: float = 1.0) -> np.ndarray:
    """dequant_weight in numpy."""
    if fmt == FMT_FP8:
        n, k = packed.shape
        s = np.repeat(np.repeat(scale.astype(np.float32), 128, 0)[:n], 128, 1)[:, :k]
        return (E4M3[packed] * s).astype(np.float32)
    v = unpack_fp4(packed)
    if fmt == FMT_MXFP4:
        s = np.ldexp(np.float32(1.0), scale.astype(np.int32) - 127).astype(np.float32)
        return (v * np.repeat(s, 32, axis=-1)).astype(np.float32)
    if fmt == FMT_NVFP4:
        s = E4M3[scale]
        return ((v * np.repeat(s, 16, axis=-1)).astype(np.float32) * np.float32(ts)).astype(np.float32)
    raise ValueError(fmt)


def qlinear(x: np.ndarray, wdq: np.ndarray, pow2: bool = True) -> np.ndarray:
    """model.py:114-126 for a quantised weight: act_quant(x) then dequant-GEMM, bf16 out
    (v4_kernels_cpu.py:158-173: C = dequant(A) @ dequant(B)^T in fp32, then to bf16)."""
    q, s = act_quant(x, 128, pow2)
    da = dequant_act(q, s)
    return bf16_round((da @ wdq.T).astype(np.float32))


# Activation batches up to this many rows take oracle/dequant.c's fused dequant-and-dot (no
# dequantised copy of the weight); wider ones dequantise once and multiply with BLAS.
QGEMM_C_ROWS = 64


def qlinear_packed(x: np.ndarray, fmt: int, packed: np.ndarray, scale: np.ndarray, ts: float = 1.0,
                   pow2: bool = True) -> np.ndarray:
    """qlinear with the weight still quantised: the same arithmetic, the dequantisation done per
    weight row inside the GEMM for narrow batches."""
    lib = _clib()
    if lib is None or x.shape[0] > QGEMM_C_ROWS:
        return qlinear(x, dequant_weight(fmt, packed, scale, ts), pow2)
    q, s = act_quant(x, 128, pow2)
    da = np.ascontiguousarray(dequant_act(q, s), dtype=np.float32)
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    n = packed.shape[0]
    k = da.shape[1]
    sc = np.ascontiguousarray(scale, dtype=np.float32 if fmt == FMT_FP8 else np.uint8)
    y = np.empty((da.shape[0], n), dtype=np.float32)
    row = np.empty(k, dtype=np.float32)
    rc = lib.oracle_qgemm(fmt, packed.ctypes.data, sc.ctypes.data, float(np.float32(ts)), n, k, da.ctypes.data,
                          da.shape[0], y.ctypes.data, row.ctypes.data)
    if rc != 0:
        raise ValueError(fmt)
    return bf16_round(y)


# ── the MoE ────────────────────────────────────────────────────────────────────────────────────

def _sigmoid(x):
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gate(x: np.ndarray, w: np.ndarray, bias, score_func: str, route_scale: float, topk: int,
         logits_bf16: bool = False, renormalize: bool = True):
    """Gate.forward (model.py:569-589): fp32 logits, score, bias for selection only, sorted top-k,
    weights gathered from the unbiased scores, renormalised unless softmax, times route_scale.
    Ties in the biased score go to the lower expert id.

    logits_bf16 / renormalize=False restate the MiniMax-M2.5 router (engines/minimax_m25/
    m25_stage.py:412-416: a bf16 F.linear; :299-303: FusedMoE renormalize=norm_topk_prob)."""
    logits = (x.astype(np.float32) @ w.astype(np.float32).T).astype(np.float32)
    if logits_bf16:
        logits = bf16_round(logits)
    if score_func == "softmax":
        z = logits - logits.max(-1, keepdims=True)
        ez = np.exp(z).astype(np.float32)
        scores = (ez / ez.sum(-1, keepdims=True)).astype(np.float32)
    elif score_func == "sigmoid":
        scores = _sigmoid(logits)
    else:
        sp = np.where(logits > 20, logits, np.log1p(np.exp(np.minimum(logits, 20)))).astype(np.float32)
        scores = np.sqrt(sp).astype(np.float32)
    sel = scores + bias.astype(np.float32) if bias is not None else scores
    e = scores.shape[-1]
    order = np.lexsort((np.broadcast_to(np.arange(e), sel.shape), -sel), axis=-1)
    idx = order[:, :topk].astype(np.int64)
    wts = np.take_along_axis(scores, idx, axis=-1).astype(np.float32)
    if score_func != "softmax" and renormalize:
        wts = (wts / wts.sum(-1, keepdims=True)).astype(np.float32)
    wts = (wts * np.float32(route_scale)).astype(np.float32)
    return wts, idx, logits


def expert_forward(x: np.ndarray, fmt: int, ew, swiglu_limit: float, weight=None, pow2: bool = True):
    """Expert.forward (model.py:601-611) for rows x [m, H] (bf16 values as fp32).

    ew = (w13 packed, w13 scale, w13 tensor scales [2], w2 packed, w2 scale, w2 tensor scale [1])
    with w13 = w1 rows then w3 rows."""
    w13, w13_s, w13_ts, w2, w2_s, w2_ts = ew
    i2 = w13.shape[0]
    inter = i2 // 2
    if fmt == FMT_FP8:
        bi = inter // 128
        g = qlinear_packed(x, fmt, w13[:inter], w13_s[:bi], 1.0, pow2)
        u = qlinear_packed(x, fmt, w13[inter:], w13_s[bi:], 1.0, pow2)
    else:
        g = qlinear_packed(x, fmt, w13[:inter], w13_s[:inter], float(w13_ts[0]), pow2)
        u = qlinear_packed(x, fmt, w13[inter:], w13_s[inter:], float(w13_ts[1]), pow2)
    if swiglu_limit > 0:
        lim = np.float32(swiglu_limit)
        u = np.clip(u, -lim, lim)
        g = np.minimum(g, lim)
    h = (g * _sigmoid(g)).astype(np.float32) * u
    h = h.astype(np.float32)
    if weight is not None:
        h = (weight.astype(np.float32) * h).astype(np.float32)
    h = bf16_round(h)
    return qlinear_packed(h, fmt, w2, w2_s, float(w2_ts[0]), pow2)


class OracleLayer:
    """A MoE layer as the oracle sees it: numpy arrays plus an expert accessor.

    `expert(e)` returns the 6-tuple expert_forward takes; it is a callable so that full-size layers
    can materialise only the experts a batch routes to."""

    def __init__(self, *, hidden, inter, topk, score_func, route_scale, swiglu_limit, expert_fmt,
                 gate_w, gate_b, expert, shared=None, shared_fmt=FMT_FP8, pow2=True, logits_bf16=False,
                 renormalize=True):
        self.hidden, self.inter, self.topk = hidden, inter, topk
        self.score_func, self.route_scale, self.swiglu_limit = score_func, route_scale, swiglu_limit
        self.expert_fmt, self.shared_fmt = expert_fmt, shared_fmt
        self.gate_w, self.gate_b = gate_w, gate_b
        self.expert, self.shared = expert, shared
        self.pow2 = pow2
        self.logits_bf16, self.renormalize = logits_bf16, renormalize


def moe_forward(layer: OracleLayer, x: np.ndarray, workers: int = 1):
    """MoE.forward (model.py:634-649). x: [M, H] fp32 holding bf16 values.

    Returns (y [M, H] fp32 on the bf16 grid, routing weights [M, k], indices [M, k]).
    Duplicate ids in one row (hash layers) follow the reference's `y[idx] +=` semantics: the last
    slot naming an expert wins, the earlier ones are dropped."""
    wts, idx, _ = gate(x, layer.gate_w, layer.gate_b, layer.score_func, layer.route_scale, layer.topk,
                       getattr(layer, "logits_bf16", False), getattr(layer, "renormalize", True))
    y = np.zeros_like(x, dtype=np.float32)
    experts = sorted(set(idx.ravel().tolist()))

    def run(e):
        rows, slots = np.nonzero(idx == e)
        out = expert_forward(x[rows], layer.expert_fmt, layer.expert(e), layer.swiglu_limit,
                             wts[rows, slots][:, None], layer.pow2)
        return rows, out

    if workers > 1:
        with ThreadPoolExecutor(workers) as pool:
            results = list(pool.map(run, experts))
    else:
        results = [run(e) for e in experts]
    for rows, out in results:                     # ascending expert id: the reference's loop order
        cur = y[rows] + out
        y[rows] = cur                             # repeated rows: the last write wins, as in torch
    if layer.shared is not None:
        y = (y + expert_forward(x, layer.shared_fmt, layer.shared, layer.swiglu_limit, None,
                                layer.pow2)).astype(np.float32)
    return bf16_round(y), wts, idx


def permutation(idx: np.ndarray, n_experts: int):
    """The token permutation the grouped forward builds: per expert (ascending id), its (token, slot)
    pairs in ascending token order. Returns (counts [E], offsets [E+1], pair_token, pair_slot,
    active expert ids)."""
    m, k = idx.shape
    flat = idx.ravel()
    order = np.lexsort((np.arange(m * k), flat))
    counts = np.bincount(flat, minlength=n_experts).astype(np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return counts, offsets, (order // k).astype(np.int32), (order % k).astype(np.int32), \
        np.nonzero(counts)[0].astype(np.int32)


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref|: the tolerance metric of the parity tests."""
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64)).max()
    r = np.abs(ref.astype(np.float64)).max()
    return float(d / r) if r > 0 else float(d)


# ── Kimi-K3's routed experts (KimiSparseMoeBlock.moe_infer) ─────────────────────────────────────

def situ(g: np.ndarray, u: np.ndarray, beta: float, linear_beta) -> np.ndarray:
    """SituAndMul (vendor/kimi_k3_ref/modeling_kimi_linear.py:64-82) on fp32 gate / up values:
    beta * tanh(gate / beta) * sigmoid(gate) * up, up -> linear_beta * tanh(up / linear_beta) when
    linear_beta is set."""
    b = np.float32(beta)
    a = (b * np.tanh((g / b).astype(np.float32)).astype(np.float32)).astype(np.float32)
    a = (a * _sigmoid(g)).astype(np.float32)
    if linear_beta:
        lb = np.float32(linear_beta)
        u = (lb * np.tanh((u / lb).astype(np.float32))).astype(np.float32)
    return (a * u).astype(np.float32)


def bf16_linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """nn.Linear on bf16 tensors: the products of bf16 values summed in fp32, the result in bf16."""
    return bf16_round((x.astype(np.float32) @ w.astype(np.float32).T).astype(np.float32))


def k3_moe_infer(x: np.ndarray, topk_ids: np.ndarray, topk_weight: np.ndarray, expert, beta: float,
                 linear_beta=None) -> np.ndarray:
    """KimiSparseMoeBlock.moe_infer (modeling_kimi_linear.py:850-876) for x [T, D] (bf16 values as
    fp32), distinct topk_ids [T, k] per token, topk_weight [T, k] fp32, with MXFP4 experts:
    expert(e) = (w13 packed [2I, D/2], w13 e8m0 [2I, D/32], w2 packed [D, I/2], w2 e8m0 [D, I/32]),
    w1 rows then w3 rows. Each expert (KimiBlockSparseMLP.forward, :262-270): w1 and w3 in bf16,
    situ in fp32 -> bf16, w2 in bf16; then, per token, the fp32 sum over its slots of the bf16
    expert output times the slot's weight, rounded to bf16."""
    t, k = topk_ids.shape
    out = np.zeros((t, k, x.shape[1]), dtype=np.float32)
    for e in sorted(set(topk_ids.ravel().tolist())):
        rows, slots = np.nonzero(topk_ids == e)
        w13, w13_s, w2, w2_s = expert(e)
        inter = w13.shape[0] // 2
        w1 = dequant_weight(FMT_MXFP4, w13[:inter], w13_s[:inter])
        w3 = dequant_weight(FMT_MXFP4, w13[inter:], w13_s[inter:])
        g = bf16_linear(x[rows], w1)
        u = bf16_linear(x[rows], w3)
        h = bf16_round(situ(g, u, beta, linear_beta))
        out[rows, slots] = bf16_linear(h, dequant_weight(FMT_MXFP4, w2, w2_s))
    acc = np.zeros((t, x.shape[1]), dtype=np.float32)
    for j in range(k):                      # the slots in order
        acc = (acc + out[:, j] * topk_weight[:, j:j + 1].astype(np.float32)).astype(np.float32)
    return bf16_round(acc)
