"""Generate the golden vectors of the FP8 activation wire (the stage-boundary codec).

Run here, where the leyten/shard tree is readable, NEVER on the GPU box:

    python tests/golden/make_wire_golden.py --ref <path to leyten/shard checkout>

It imports the reference's own codec, engines/deepseek_v4/v4_pipe.py `_pack_t` (e4m3 with one bf16
scale per (position, stream), the amax over the last dim) and `_unpack_t` (fp8 * scale in bf16), and
records their outputs on seeded inputs that cover the edge cases the codec's docstring names:

  wire_<case>.npz   x (bf16 bits, [..., dim]), q (e4m3 bytes), scale (bf16 bits, [...]),
                    y = _unpack_t(q, scale) (bf16 bits)

Cases: N(0,1) tokens at the V4 boundary shape [b, s, hc=4, dim=4096]; the c1/c3/c4 hidden sizes as
[M, H] stage activations; a row of zeros (the 1e-8 clamp), a row holding +inf (the bf16-max clamp:
the inf saturates to 448 and the rest of the row stays finite), rows of huge, tiny and subnormal
magnitudes, and a row of exact ties for the e4m3 rounding.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t):
    return t.contiguous().view(torch.int16).numpy().copy()


def cases():
    g = torch.Generator().manual_seed(11)
    out = {}
    out["v4_boundary"] = torch.randn(1, 3, 4, 4096, generator=g, dtype=torch.float32).to(torch.bfloat16)
    out["c1_m16"] = (torch.randn(16, 4096, generator=g, dtype=torch.float32) * 3.0).to(torch.bfloat16)
    out["c3_m5"] = torch.randn(5, 3072, generator=g, dtype=torch.float32).to(torch.bfloat16)
    out["c4_m3"] = (torch.randn(3, 7168, generator=g, dtype=torch.float32) * 0.01).to(torch.bfloat16)
    e = torch.randn(8, 4096, generator=g, dtype=torch.float32)
    e[0] = 0.0                                   # all-zero row: scale clamps to 1e-8
    e[1, 17] = float("inf")                      # one inf: saturates, the row stays finite
    e[2] *= 1e30                                 # huge magnitudes
    e[3] *= 1e-30                                # tiny magnitudes
    e[4] = torch.linspace(-448.0, 448.0, 4096)   # amax exactly 448: scale 1, values on and between codes
    e[5, :] = 0.0
    e[5, :64] = torch.tensor([2.0 ** -9 * k for k in range(64)])   # e4m3 subnormal range after scaling
    e[6] = -e[6].abs()                           # all negative
    e[7, ::2] = -0.0                             # signed zeros among values
    out["edges"] = e.to(torch.bfloat16)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to a leyten/shard checkout")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "engines", "deepseek_v4"))
    sys.path.insert(0, args.ref)
    import v4_pipe  # the reference's stage transport module
    for name, x in cases().items():
        q, s = v4_pipe._pack_t(x)
        y = v4_pipe._unpack_t(q, s)
        np.savez_compressed(os.path.join(HERE, f"wire_{name}.npz"), x=bits(x), q=q.view(torch.uint8).numpy(),
                            scale=bits(s), y=bits(y), shape=np.array(x.shape))
        print(name, tuple(x.shape), "finite y:", bool(torch.isfinite(y.float()).all()))


if __name__ == "__main__":
    main()
