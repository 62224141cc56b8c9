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


# the reference's names (v4_pipe.py:335, :379)
_pack_t = pack
_unpack_t = unpack
