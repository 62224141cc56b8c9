"""Pipeline-partitioned MoE layer stack over the GPUs of one node.

The reference shards a model into contiguous layer blocks, one stage per GPU/process
(engines/deepseek_v4/v4_pipe.py:2286-2298 even_tiling, :2521-2557 split_stages_to_gpus), and moves
activations between stages as host frames over TCP (v4_pipe.py:424-460, shard/transport.py:143-175).
Here each stage is one rank of a torch.distributed NCCL group, and the hop is an NCCL send/recv of
the bf16 activation [M, H] device to device over NVLink. Several verify chunks stream through the
stages back to back, so stage r works on chunk j while stage r+1 works on chunk j-1. Every hop is
asynchronous and off the compute stream: a stage posts its receives `depth` chunks ahead on a
receive stream (each into a ring buffer the compute stream has released), issues each send on a send
stream once the compute stream has produced the chunk, and the compute stream waits only for the
receive of the chunk it is about to run. So a stage never waits for its successor's compute (a send
completes as soon as the successor's receive, posted long before, takes it), and the host never
blocks (the host runs ahead; events and stream waits order the work).

With wire="fp8" a hop carries the reference's FP8 activation wire instead (v4_pipe.py:320-384:
e4m3 + one bf16 scale per row, half the bytes): the stage's last MoE layer emits it from its combine
kernel (MoELayer.forward_wire) and the next stage unpacks it before its first layer.
"""
from __future__ import annotations

import collections
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
    x -> y with the same [M, H] bf16 shape).

    residual=False chains the operators (x <- layer(x)). residual=True runs each layer as the ffn half
    of the reference block (model.py:701-706, hyper-connections aside): x <- x + layer(RMSNorm(x)),
    with the add and the norm fused in one kernel (shard_b200.wire.residual_rmsnorm; CUDA tensors).
    Chained random-weight MoE layers drive every token onto the same experts within ~10 layers; the
    residual stream and the norm keep a synthetic stack's routing as spread as its first layer's."""

    def __init__(self, layers: Sequence, residual: bool = False, eps: float = 1e-6):
        self.layers = list(layers)
        self.residual = residual
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.residual:
            for layer in self.layers:
                x = layer.forward(x)
            return x
        from .wire import residual_rmsnorm
        x = x.clone()            # the residual stream; the caller's chunk is left as it is
        y = None
        for layer in self.layers:
            y = layer.forward(residual_rmsnorm(x, y, eps=self.eps))
        if y is not None:
            residual_rmsnorm(x, y, norm=False)
        return x

    __call__ = forward

    def forward_wire(self, x: torch.Tensor, pack):
        """The stack's output in the FP8 wire form: the last layer emits it directly when it can,
        otherwise `pack` is applied to the output."""
        if self.residual:
            return pack(self.forward(x))
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
        """depth: receives posted ahead (ring buffers) and sends kept in flight. wire: "bf16" or
        "fp8". codec: (pack, unpack) for the fp8 wire; shard_b200.wire's CUDA codec by default."""
        assert wire in ("bf16", "fp8") and depth >= 1
        self.stack, self.m, self.hidden = stack, m, hidden
        self.rank, self.world = rank, world
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.depth = depth
        self.wire = wire
        if wire == "fp8" and codec is None:
            from . import wire as _wire
            codec = (_wire.pack, _wire.unpack)
        self.codec = codec
        if wire == "fp8":
            # the wire travels as raw bytes: e4m3 codes and bf16 scale bits
            self.recv_bufs = [(torch.empty(m, hidden, dtype=torch.uint8, device=self.device),
                               torch.empty(2 * m, dtype=torch.uint8, device=self.device)) for _ in range(depth)]
        else:
            self.recv_bufs = [(torch.empty(m, hidden, dtype=torch.bfloat16, device=self.device),)
                              for _ in range(depth)]
        self.cuda = self.device.type == "cuda"
        if self.cuda:
            self.recv_stream = torch.cuda.Stream(self.device)
            self.send_stream = torch.cuda.Stream(self.device)
            self.free_ev = [None] * depth          # compute has finished reading ring slot i
        self._recvs = {}                          # chunk -> (works, buffers) posted, not yet used
        self._sends = collections.deque()         # (works, tensors kept alive) in flight

    @property
    def first(self) -> bool:
        return self.rank == 0

    @property
    def last(self) -> bool:
        return self.rank == self.world - 1

    def _post_recv(self, j: int):
        """Post the receive of chunk j (of the current run) into ring slot j % depth."""
        bufs = self.recv_bufs[j % self.depth]
        if self.cuda:
            with torch.cuda.stream(self.recv_stream):
                ev = self.free_ev[j % self.depth]
                if ev is not None:
                    self.recv_stream.wait_event(ev)
                works = [dist.irecv(b, src=self.rank - 1) for b in bufs]
        else:
            works = [dist.irecv(b, src=self.rank - 1) for b in bufs]
        self._recvs[j] = (works, bufs)

    def _take_recv(self, j: int):
        """The received tensors of chunk j, with the current (compute) stream made to wait for them."""
        works, bufs = self._recvs.pop(j)
        for w in works:
            w.wait()
        return bufs

    def _send(self, tensors):
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self.send_stream):
                self.send_stream.wait_event(ev)
                works = [dist.isend(t, dst=self.rank + 1) for t in tensors]
        else:
            works = [dist.isend(t, dst=self.rank + 1) for t in tensors]
        self._sends.append((works, tensors))
        while len(self._sends) > self.depth:
            self._retire_send()

    def _retire_send(self):
        works, _ = self._sends.popleft()
        for w in works:
            w.wait()                               # CUDA: the compute stream waits; host: blocks

    def flush(self):
        """Make the compute stream (on the host: the caller) wait for every send in flight."""
        while self._sends:
            self._retire_send()

    def _compute(self, h: torch.Tensor):
        """The stage's layers on one chunk: (y, tensors to send on or None)."""
        if not self.last and self.wire == "fp8":
            q, s = self.stack.forward_wire(h, self.codec[0])
            return None, (q.view(torch.uint8), s.contiguous().view(torch.uint8))
        y = self.stack(h)
        return y, (None if self.last else (y,))

    def run_chunk(self, x: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Process one chunk on its own (receive, compute, send). Stage 0 takes x; the last stage
        returns y; the others return None."""
        res = self.run(1, [x] if self.first else None)
        return res[0] if self.last else None

    def run(self, n: int, chunks: Optional[Sequence[torch.Tensor]] = None,
            outs: Optional[Sequence[torch.Tensor]] = None):
        """Stream n chunks through this stage (every rank calls this with the same n). Stage 0
        reads chunks[j]; the last stage copies each result into outs[j] (device or pinned host
        tensors) when given, else returns the results. Sends may still be in flight on return
        (flush() or a device synchronisation completes them); the last stage's copies are enqueued
        on the compute stream."""
        results = []
        if not self.first:
            for j in range(min(self.depth, n)):
                self._post_recv(j)
        for j in range(n):
            if self.first:
                h = chunks[j]
            else:
                bufs = self._take_recv(j)
                if self.wire == "fp8":
                    h = self.codec[1](bufs[0].view(torch.float8_e4m3fn), bufs[1].view(torch.bfloat16))
                else:
                    h = bufs[0]
            y, send = self._compute(h)
            if not self.first:
                # ring slot j % depth is free once this chunk's compute has read it
                if self.cuda:
                    ev = torch.cuda.Event()
                    ev.record()
                    self.free_ev[j % self.depth] = ev
                if j + self.depth < n:
                    self._post_recv(j + self.depth)
            if send is not None:
                self._send(send)
            elif self.last:
                if outs is not None:
                    outs[j].copy_(y, non_blocking=True)
                else:
                    results.append(y)
        if not self.cuda:
            self.flush()
        return results
