"""The stage-boundary FP8 activation wire on the B200: the reference's `_pack_t` / `_unpack_t`
(engines/deepseek_v4/v4_pipe.py:335-384) as CUDA kernels behind the C ABI.

pack(t)         [..., dim] bf16 -> (e4m3 [..., dim], bf16 scale [...]); one scale per row of the last
                dim, so each position's wire bytes depend on its own values only (the property the
                reference keeps for speculative decoding: the same position packs to the same bytes in
                chunks of any length)
unpack(q, s)    -> bf16 [..., dim] = q * s in bf16

Same names, shapes, dtypes and results as the reference functions (bit-exact). CUDA tensors only;
there is no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._lib import check, lib, ptr, stream_ptr


def pack(t: torch.Tensor, stream=None):
    assert t.is_cuda and t.dtype == torch.bfloat16, "pack: bf16 CUDA tensor"
    x = t.contiguous()
    dim = x.shape[-1]
    rows = x.numel() // dim
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(x.shape[:-1], dtype=torch.bfloat16, device=x.device)
    check(lib().sb_wire_pack(ptr(x), rows, dim, ptr(q), ptr(s), stream_ptr(stream)), "sb_wire_pack")
    return q, s


def unpack(q: torch.Tensor, scale: torch.Tensor, stream=None) -> torch.Tensor:
    assert q.is_cuda and scale.is_cuda and scale.dtype == torch.bfloat16, "unpack: CUDA e4m3 + bf16 scale"
    q = q.contiguous()
    scale = scale.contiguous()
    dim = q.shape[-1]
    rows = q.numel() // dim
    assert scale.numel() == rows
    y = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    check(lib().sb_wire_unpack(ptr(q), ptr(scale), rows, dim, ptr(y), stream_ptr(stream)), "sb_wire_unpack")
    return y


def residual_rmsnorm(x: torch.Tensor, y: Optional[torch.Tensor] = None, weight: Optional[torch.Tensor] = None,
                     eps: float = 1e-6, norm: bool = True, stream=None) -> Optional[torch.Tensor]:
    """The block around the MoE operator (model.py:701-706, hyper-connections aside): x (bf16, the
    residual stream, updated in place) += y when given; returns RMSNorm(x) (model.py:197-202) in bf16,
    or None when norm is False (the add alone)."""
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous(), "residual_rmsnorm: contiguous bf16 CUDA x"
    dim = x.shape[-1]
    rows = x.numel() // dim
    if y is not None:
        assert y.dtype == torch.bfloat16 and y.shape == x.shape
        y = y.contiguous()
    w = None if weight is None else weight.float().contiguous()
    out = torch.empty_like(x) if norm else None
    check(lib().sb_residual_rmsnorm(ptr(x), ptr(y), rows, dim, ptr(w), float(eps), ptr(out), stream_ptr(stream)),
          "sb_residual_rmsnorm")
    return out


# the reference's names (v4_pipe.py:335, :379)
_pack_t = pack
_unpack_t = unpack
