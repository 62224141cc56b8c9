"""CPU oracle for the FP8 activation wire: a numpy restatement of the reference's stage-boundary codec.

TEST INFRASTRUCTURE ONLY: only tests/ (and, as the checker, smoke()) use it; the product path is the
CUDA codec in libshard_b200.so.

Restates engines/deepseek_v4/v4_pipe.py (paths relative to the leyten/shard tree):
  pack    `_pack_t`   :335-376  one scale per row of the last dim: amax in fp32, scale =
                                clamp(amax / 448, 1e-8, bf16 max) rounded to bf16, q = e4m3(clamp(x /
                                scale, +-448)) with the division by that same rounded scale
  unpack  `_unpack_t` :379-384  q -> bf16 times the bf16 scale, in bf16 (one rounding of the exact
                                fp32 product)

Pinned by tests/test_wire.py against tests/golden/wire_*.npz, which tests/golden/make_wire_golden.py
recorded from the reference's own _pack_t / _unpack_t.
"""
from __future__ import annotations

import numpy as np

from oracle.moe_oracle import E4M3, bf16_round, e4m3_encode

BF16_MAX = np.float32(3.3895313892515355e38)


def pack(x: np.ndarray):
    """x: [..., dim] fp32 holding bf16 values -> (e4m3 codes uint8 [..., dim], fp32 scales [...] on
    the bf16 grid)."""
    f = np.asarray(x, dtype=np.float32)
    amax = np.abs(f).max(-1, keepdims=True).astype(np.float32)
    scale = (amax / np.float32(448.0)).astype(np.float32)
    scale = np.clip(scale, np.float32(1e-8), BF16_MAX).astype(np.float32)
    scale = bf16_round(scale)
    q = np.clip((f / scale).astype(np.float32), np.float32(-448.0), np.float32(448.0))
    return e4m3_encode(q), scale[..., 0]


def unpack(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """(e4m3 codes [..., dim], bf16-valued fp32 scales [...]) -> fp32 holding the bf16 result."""
    with np.errstate(over="ignore"):   # an inf in x saturates to 448 and decodes to 448 * bf16 max = inf
        return bf16_round((E4M3[q] * np.asarray(scale, dtype=np.float32)[..., None]).astype(np.float32))
