"""Pipeline-partitioned MoE layer stack over the GPUs of one node.

The reference shards a model into contiguous layer blocks, one stage per GPU/process
(engines/deepseek_v4/v4_pipe.py:2286-2298 even_tiling, :2521-2557 split_stages_to_gpus), and moves
activations between stages as host frames over TCP (v4_pipe.py:424-460, shard/transport.py:143-175).
Here each stage is one rank of a torch.distributed NCCL group, and the hop is an NCCL send/recv of
the bf16 activation [M, H] device to device over NVLink. Several verify chunks stream through the
stages back to back, so stage r works on chunk j while stage r+1 works on chunk j-1; each hop is
enqueued without a host sync (the host runs ahead and the streams order the work).

With wire="fp8" a hop carries the reference's FP8 activation wire instead (v4_pipe.py:320-384:
e4m3 + one bf16 scale per row, half the bytes): the stage's last MoE layer emits it from its combine
kernel (MoELayer.forward_wire) and the next stage unpacks it before its first layer.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def even_tiling(n_layers: int, n_stages: int) -> List[range]:
    """Contiguous layer blocks, the first n_layers % n_stages blocks one layer longer
    (the front-loaded split of v4_pipe.py:2286-2298)."""
    base, extra = divmod(n_layers, n_stages)
    out, lo = [], 0
    for s in range(n_stages):
        hi = lo + base + (1 if s < extra else 0)
        out.append(range(lo, hi))
        lo = hi
    return out


class StageStack:
    """The layers one stage owns, run in order. Each layer is a MoELayer (or anything callable
    x -> y with the same [M, H] bf16 shape)."""

    def __init__(self, layers: Sequence):
        self.layers = list(layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self.layers:
            x = layer.forward(x)
        return x

    __call__ = forward

    def forward_wire(self, x: torch.Tensor, pack):
        """The stack's output in the FP8 wire form: the last layer emits it directly when it can,
        otherwise `pack` is applied to the output."""
        for layer in self.layers[:-1]:
            x = layer.forward(x)
        last = self.layers[-1] if self.layers else None
        if last is not None and hasattr(last, "forward_wire"):
            return last.forward_wire(x)
        return pack(last.forward(x) if last is not None else x)


class Pipeline:
    """One rank's view of the pipeline: receive a chunk from the previous stage (or take it from the
    caller on stage 0), run the stage's layers, send it on (or hand it back on the last stage)."""

    def __init__(self, stack: StageStack, m: int, hidden: int, rank: int = 0, world: int = 1,
                 device: Optional[torch.device] = None, depth: int = 4, wire: str = "bf16", codec=None):
        """wire: "bf16" or "fp8". codec: (pack, unpack) for the fp8 wire; shard_b200.wire's CUDA
        codec by default."""
        assert wire in ("bf16", "fp8")
        self.stack, self.m, self.hidden = stack, m, hidden
        self.rank, self.world = rank, world
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.depth = depth
        self.wire = wire
        if wire == "fp8" and codec is None:
            from . import wire as _wire
            codec = (_wire.pack, _wire.unpack)
        self.codec = codec
        self.recv_bufs = [torch.empty(m, hidden, dtype=torch.bfloat16, device=self.device) for _ in range(depth)]
        if wire == "fp8":
            # the wire travels as raw bytes: e4m3 codes and bf16 scale bits
            self.recv_q = [torch.empty(m, hidden, dtype=torch.uint8, device=self.device) for _ in range(depth)]
            self.recv_s = [torch.empty(2 * m, dtype=torch.uint8, device=self.device) for _ in range(depth)]
        self._slot = 0

    @property
    def first(self) -> bool:
        return self.rank == 0

    @property
    def last(self) -> bool:
        return self.rank == self.world - 1

    def run_chunk(self, x: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Process one chunk. Stage 0 takes x; the last stage returns y; the others return None."""
        if self.first:
            assert x is not None
            h = x
        elif self.wire == "fp8":
            q, s = self.recv_q[self._slot], self.recv_s[self._slot]
            self._slot = (self._slot + 1) % self.depth
            dist.recv(q, src=self.rank - 1)
            dist.recv(s, src=self.rank - 1)
            h = self.codec[1](q.view(torch.float8_e4m3fn), s.view(torch.bfloat16))
        else:
            h = self.recv_bufs[self._slot]
            self._slot = (self._slot + 1) % self.depth
            dist.recv(h, src=self.rank - 1)
        if not self.last and self.wire == "fp8":
            q, s = self.stack.forward_wire(h, self.codec[0])
            dist.send(q.view(torch.uint8), dst=self.rank + 1)
            dist.send(s.contiguous().view(torch.uint8), dst=self.rank + 1)
            return None
        y = self.stack(h)
        if not self.last:
            dist.send(y, dst=self.rank + 1)
            return None
        return y

    def run(self, n: int, chunks: Optional[Sequence[torch.Tensor]] = None,
            outs: Optional[Sequence[torch.Tensor]] = None):
        """Stream n chunks through this stage (every rank calls this with the same n). Stage 0
        reads chunks[j]; the last stage copies each result into outs[j] (device or pinned host
        tensors) when given, else returns the results."""
        results = []
        for j in range(n):
            y = self.run_chunk(chunks[j] if self.first else None)
            if self.last:
                if outs is not None:
                    outs[j].copy_(y, non_blocking=True)
                else:
                    results.append(y)
        return results
