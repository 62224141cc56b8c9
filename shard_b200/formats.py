"""Weight and activation formats of the MoE stage, as host-side (load-time) quantizers.

These run once per weight at load time, never on the forward path. They are written with torch ops
so the same code quantizes on the CPU (fixtures, tests) and on the GPU (synthetic bench weights).

Formats (all 4-bit data packed two per byte, LOW NIBBLE FIRST: byte i of a row holds logical K
positions 2i (bits 0-3) and 2i+1 (bits 4-7), as `unpack_fp4` in
engines/deepseek_v4/v4_kernels_cpu.py:141-155 and vendor/deepseek_v4_ref/inference/convert.py read it):

  MXFP4   e2m1 values, one e8m0 (power-of-two) scale per 32 K-elements.  This is the reference's
          own routed-expert format (model.py:135-141; fp4_quant_kernel kernel.py:128-200).
  NVFP4   e2m1 values, one e4m3 scale per 16 K-elements, one fp32 tensor scale per matrix.
          The reference has no in-tree NVFP4 arithmetic; the dequant is e2m1 * e4m3 * tensor_scale,
          the order the MoE oracle states it in.
  FP8     e4m3 values, one fp32 scale per 128x128 block of [N, K] (model.py:143-147; the
          reference stores the scale as e8m0, which holds exactly the power-of-two values
          produced here).

Rounding rules shared with the reference quantizers (v4_kernels_cpu.py:30-45):
  * power-of-two scale = 2^ceil(log2(amax * (1/max))), exact at powers of two (frexp, not log2);
  * e2m1 rounds to nearest with ties to the EVEN code (0.25->0, 0.75->1, 1.25->1, 1.75->2,
    2.5->2, 3.5->4, 5->4);
  * e4m3 rounds to nearest even (torch's cast), after a clamp to +-448.
"""
from __future__ import annotations

import torch

FP8_MAX = 448.0
FP4_MAX = 6.0
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)

# Format ids shared with include/shard_b200.h (SB_FMT_*).
FMT_NVFP4 = 1
FMT_MXFP4 = 2
FMT_FP8 = 3
FMT_NAMES = {FMT_NVFP4: "nvfp4", FMT_MXFP4: "mxfp4", FMT_FP8: "fp8"}
FMT_IDS = {v: k for k, v in FMT_NAMES.items()}


def pow2_ceil_scale(amax: torch.Tensor, max_inv: float) -> torch.Tensor:
    """2^ceil(log2(amax * max_inv)) in fp32, exact at powers of two.

    Follows kernel.py:22-37 (fast_log2_ceil / fast_pow2 on the IEEE bits) and its CPU transcription
    v4_kernels_cpu.py:65-75: frexp gives x = m * 2^e with m in [0.5, 1), so ceil(log2 x) is e-1 when
    m == 0.5 and e otherwise. `max_inv` is multiplied, not divided, as the kernel folds 1/max into a
    constant."""
    x = amax.float() * torch.tensor(max_inv, dtype=torch.float32)
    mant, exp = torch.frexp(x)
    return torch.ldexp(torch.ones_like(x), torch.where(mant == 0.5, exp - 1, exp))


def e2m1_encode(a: torch.Tensor) -> torch.Tensor:
    """Signed fp32 in [-6, 6] -> 4-bit e2m1 code (uint8), nearest value, ties to the even code.

    Same rule as v4_kernels_cpu._e2m1 (v4_kernels_cpu.py:107-116): bucketize left/right agree except
    exactly on a midpoint, where the even code is chosen."""
    mag = a.abs()
    mid = torch.tensor(E2M1_MID, dtype=torch.float32, device=a.device)
    lo = torch.bucketize(mag, mid, right=False)
    hi = torch.bucketize(mag, mid, right=True)
    code = lo + ((hi != lo) & (lo % 2 == 1)).to(lo.dtype)
    sign = (a < 0).to(code.dtype) * 8
    return (code | sign).to(torch.uint8)


def pack_fp4(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] 4-bit codes -> [..., K/2] bytes, low nibble first."""
    c = codes.to(torch.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).contiguous()


def unpack_fp4_values(packed: torch.Tensor) -> torch.Tensor:
    """[..., K/2] bytes -> [..., K] fp32 e2m1 values, low nibble first."""
    table = torch.tensor(E2M1 + tuple(-v for v in E2M1), dtype=torch.float32, device=packed.device)
    u = packed.to(torch.uint8)
    lo = table[(u & 0x0F).long()]
    hi = table[(u >> 4).long()]
    return torch.stack([lo, hi], dim=-1).flatten(-2)


def e4m3_encode(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3 bytes (round to nearest even; the caller clamps to +-448 first)."""
    return x.float().to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_decode(u: torch.Tensor) -> torch.Tensor:
    return u.view(torch.float8_e4m3fn).float()


def e8m0_encode(pow2: torch.Tensor) -> torch.Tensor:
    """Exact powers of two (fp32) -> e8m0 bytes (biased exponent)."""
    _, exp = torch.frexp(pow2.float())
    return (exp - 1 + 127).clamp(0, 254).to(torch.uint8)


def e8m0_decode(u: torch.Tensor) -> torch.Tensor:
    return torch.ldexp(torch.ones(u.shape, dtype=torch.float32, device=u.device),
                       u.to(torch.int32) - 127)


def quant_mxfp4(w: torch.Tensor):
    """bf16 [N, K] -> (packed uint8 [N, K/2], e8m0 uint8 [N, K/32]).

    The reference's fp4_act_quant (kernel.py:128-200, v4_kernels_cpu.py:119-136): per 32 along K,
    amax floored at 6*2^-126, power-of-two scale for max 6.0, e2m1 of clamp(x/s, +-6)."""
    n, k = w.shape
    assert k % 32 == 0, "MXFP4 needs K % 32 == 0"
    z = w.float().reshape(n, k // 32, 32)
    amax = z.abs().amax(-1, keepdim=True).clamp_min(FP4_MAX * 2.0 ** -126)
    s = pow2_ceil_scale(amax, 1.0 / FP4_MAX)
    q = (z / s).clamp(-FP4_MAX, FP4_MAX)
    codes = e2m1_encode(q).reshape(n, k)
    return pack_fp4(codes), e8m0_encode(s.squeeze(-1))


def quant_nvfp4(w: torch.Tensor):
    """bf16 [N, K] -> (packed uint8 [N, K/2], e4m3 uint8 [N, K/16], fp32 tensor scale).

    NVFP4 two-level scaling: the tensor scale maps the matrix amax onto the largest product of an
    e4m3 block scale and an e2m1 value (448 * 6); each 16-block gets the e4m3 scale
    amax_block / (6 * ts) rounded to nearest even; values are e2m1 of x / (s16 * ts), clamped to
    +-6. An all-zero block gets scale 0 and codes 0."""
    n, k = w.shape
    assert k % 16 == 0, "NVFP4 needs K % 16 == 0"
    z = w.float().reshape(n, k // 16, 16)
    tmax = float(z.abs().max())
    ts = (tmax / (FP8_MAX * FP4_MAX)) if tmax > 0 else 1.0
    ts = float(torch.tensor(ts, dtype=torch.float32))
    amax = z.abs().amax(-1, keepdim=True)
    s16 = e4m3_encode((amax / (FP4_MAX * ts)).clamp(max=FP8_MAX))
    sdq = e4m3_decode(s16) * ts
    q = torch.where(sdq > 0, z / torch.where(sdq > 0, sdq, torch.ones_like(sdq)), torch.zeros_like(z))
    q = q.clamp(-FP4_MAX, FP4_MAX)
    codes = e2m1_encode(q).reshape(n, k)
    return pack_fp4(codes), s16.squeeze(-1).contiguous(), ts


def quant_fp8_block(w: torch.Tensor, block: int = 128):
    """bf16 [N, K] -> (e4m3 uint8 [N, K], fp32 [ceil(N/128), ceil(K/128)] power-of-two scales).

    The weight layout fp8_gemm reads (kernel.py:203-273): one scale per 128x128 tile. The scale is
    the power of two 2^ceil(log2(amax/448)) (amax floored at 1e-4), i.e. what an e8m0 scale holds."""
    n, k = w.shape
    nb, kb = -(-n // block), -(-k // block)
    pad = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    pad[:n, :k] = w.float()
    b = pad.reshape(nb, block, kb, block)
    amax = b.abs().amax(dim=(1, 3)).clamp_min(1e-4)
    s = pow2_ceil_scale(amax, 1.0 / FP8_MAX)
    q = (b / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).reshape(nb * block, kb * block)[:n, :k]
    return e4m3_encode(q).contiguous(), s.contiguous()


def dequant_weight(fmt: int, packed: torch.Tensor, scale: torch.Tensor, tscale: float = 1.0):
    """Host-side dequant of one weight matrix to fp32 [N, K] (for tests and diagnostics)."""
    if fmt == FMT_FP8:
        n, k = packed.shape
        s = scale.repeat_interleave(128, 0)[:n].repeat_interleave(128, 1)[:, :k]
        return e4m3_decode(packed) * s
    vals = unpack_fp4_values(packed)
    if fmt == FMT_MXFP4:
        return vals * e8m0_decode(scale).repeat_interleave(32, -1)
    if fmt == FMT_NVFP4:
        return vals * e4m3_decode(scale).repeat_interleave(16, -1) * torch.tensor(tscale, dtype=torch.float32)
    raise ValueError(f"unknown format {fmt}")


def weight_bytes(fmt: int, n: int, k: int) -> int:
    """Algorithmic bytes of one [N, K] weight matrix (values + scales)."""
    if fmt == FMT_NVFP4:
        return n * k // 2 + n * k // 16 + 4
    if fmt == FMT_MXFP4:
        return n * k // 2 + n * k // 32
    if fmt == FMT_FP8:
        return n * k + (-(-n // 128)) * (-(-k // 128)) * 4
    raise ValueError(fmt)
