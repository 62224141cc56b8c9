"""The kernel-level seam: the reference `kernel` module's quantise/GEMM entry points on the B200.

Same names, argument meaning and errors as vendor/deepseek_v4_ref/inference/kernel.py (act_quant
:105-125, fp8_gemm :257-273, fp4_gemm :518-536): inputs must be contiguous (AssertionError
otherwise), the wrapper allocates its output, the result is in torch's default dtype... here always
bf16, the dtype the reference runs in. Installing this module as `sys.modules["kernel"]` before the
reference model.py is executed routes every quantised `linear()` through these kernels.

Weights arrive in the reference's canonical layout and are tiled on first use. The tiled copy (and,
for NVFP4, the tensor scale as a device scalar) is cached as an attribute of the weight tensor
itself, so it lives and dies with that tensor: a new tensor that happens to reuse a freed weight's
address never sees the old copy, and an in-place change of the weight (its version counter) or a
different scale tensor retiles it.
"""
from __future__ import annotations

import torch

from . import _lib
from . import formats as F
from ._lib import check, lib, ptr, stream_ptr


def act_quant(x: torch.Tensor, block_size: int = 128, scale_fmt=None, scale_dtype=torch.float32,
              inplace: bool = False):
    """Block-wise e4m3 quantisation, one scale per row per 128 along the last dim (kernel.py:105-125).
    scale_fmt not None selects the power-of-two scale. Returns (e4m3 tensor, fp32 or e8m0 scales)."""
    if inplace:
        raise NotImplementedError("act_quant(inplace=True) is the attention QAT path, not the MoE stage")
    n = x.size(-1)
    assert n % block_size == 0 and block_size == 128, "act_quant: last dim must be a multiple of 128"
    assert x.dtype == torch.bfloat16, "act_quant: bf16 input"
    z = x.contiguous()
    m = z.numel() // n
    y = torch.empty(*z.shape, dtype=torch.float8_e4m3fn, device=z.device)
    s = torch.empty(*z.shape[:-1], n // block_size, dtype=torch.float32, device=z.device)
    check(lib().sb_act_quant(ptr(z), m, n, 1 if scale_fmt is not None else 0, ptr(y), ptr(s), stream_ptr()),
          "sb_act_quant")
    if scale_dtype == torch.float8_e8m0fnu:
        s = F.e8m0_encode(s).view(torch.float8_e8m0fnu)
    return y, s


_CACHE_ATTR = "_sb_tiled"


def _tiled(fmt, b, b_s, layout, tensor_scale=None):
    """(tiled values, tiled scales, NVFP4 tensor scale on the device or None), cached on `b`."""
    key = (fmt, layout, b.data_ptr(), b._version, id(b_s), b_s.data_ptr(), b_s._version, tuple(b.shape),
           None if tensor_scale is None else float(tensor_scale))
    hit = getattr(b, _CACHE_ATTR, None)
    if hit is not None and hit[0] == key:
        return hit[1]
    from .moe import tile
    n = b.size(0)
    k = b.size(1) * (2 if fmt != F.FMT_FP8 else 1)
    if fmt == F.FMT_FP8:
        s = F.e8m0_decode(b_s.view(torch.uint8)) if b_s.dtype == torch.float8_e8m0fnu else b_s.float()
    else:
        s = b_s.view(torch.uint8)
    wt, st = tile(fmt, _lib.MAT_PLAIN, b.view(torch.uint8), s, 1, n, k, layout)
    ts = None
    if fmt == F.FMT_NVFP4:
        ts = torch.tensor([float(tensor_scale)], dtype=torch.float32).to(b.device)
    val = (wt, st, ts)
    setattr(b, _CACHE_ATTR, (key, val))
    return val


def _act_scales_f32(a_s):
    return F.e8m0_decode(a_s.view(torch.uint8)) if a_s.dtype == torch.float8_e8m0fnu else a_s.float()


def quantised_gemm(fmt: int, w, w_s, tensor_scale, a, a_s, layout=None):
    """y bf16 [M, N] = dequant(a, a_s) @ dequant(w, w_s, tensor_scale)^T, canonical weights."""
    from .moe import DEFAULT_LAYOUT
    layout = DEFAULT_LAYOUT if layout is None else layout
    assert a.is_contiguous() and w.is_contiguous(), "Input tensors must be contiguous"
    k = a.size(-1)
    m = a.numel() // k
    n = w.size(0)
    wt, st, ts = _tiled(fmt, w, w_s, layout, tensor_scale if fmt == F.FMT_NVFP4 else None)
    sa = _act_scales_f32(a_s).contiguous()
    y = torch.empty(*a.shape[:-1], n, dtype=torch.bfloat16, device=a.device)
    L = lib()
    wsb = L.sb_qgemm_workspace_bytes(fmt, layout, n, k, m)
    ws = torch.empty(wsb, dtype=torch.uint8, device=a.device) if wsb else None
    check(L.sb_qgemm(fmt, layout, ptr(wt), ptr(st), ptr(ts), n, k, ptr(a.view(torch.uint8)), ptr(sa), m,
                     ptr(y), ptr(ws), wsb, stream_ptr()), "sb_qgemm")
    return y


def fp8_gemm(a, a_s, b, b_s, scale_dtype=torch.float32):
    """C[M,N] = A[M,K] @ B[N,K]^T, A scaled per 1x128, B per 128x128 (kernel.py:257-273)."""
    assert a.is_contiguous() and b.is_contiguous(), "Input tensors must be contiguous"
    assert a_s.is_contiguous() and b_s.is_contiguous(), "Scaling factor tensors must be contiguous"
    return quantised_gemm(F.FMT_FP8, b, b_s, 1.0, a, a_s)


def fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32):
    """C[M,N] = A_fp8[M,K] @ B_fp4[N,K]^T (kernel.py:518-536). B packed [N, K/2], low nibble first;
    b_s e8m0 [N, K/32] (MXFP4) or e4m3 [N, K/16] with `b.tensor_scale` (NVFP4)."""
    assert a.is_contiguous() and b.is_contiguous(), "Input tensors must be contiguous"
    assert a_s.is_contiguous() and b_s.is_contiguous(), "Scaling factor tensors must be contiguous"
    if b_s.dtype == torch.float8_e4m3fn:
        return quantised_gemm(F.FMT_NVFP4, b, b_s, getattr(b, "tensor_scale", 1.0), a, a_s)
    return quantised_gemm(F.FMT_MXFP4, b, b_s, 1.0, a, a_s)
