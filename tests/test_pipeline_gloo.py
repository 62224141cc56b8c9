"""Pipeline stages over torch.distributed on the host: world_size 2 with the gloo backend, each rank
owning a contiguous layer block (even_tiling, the split of v4_pipe.py:2286-2298) and passing bf16
activations with send/recv, as the NCCL path does between GPUs. The layers are stand-ins with the
MoE layer's x -> y contract, so the test checks the host logic: block assignment, chunk streaming
and ordering, and that the last stage's outputs equal the whole stack applied in order."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from shard_b200.pipeline import Pipeline, StageStack, even_tiling

HIDDEN, M, N_LAYERS, CHUNKS = 64, 4, 5, 6


class Affine:
    """A stand-in layer: y = bf16(x * a_l + b_l), distinct per layer so the order is observable."""

    def __init__(self, l):
        self.a, self.b = 1.0 + 0.25 * l, 0.5 * l - 1.0

    def forward(self, x):
        return (x.float() * self.a + self.b).to(torch.bfloat16)


def _inputs():
    g = torch.Generator().manual_seed(7)
    return [torch.randn(M, HIDDEN, generator=g).to(torch.bfloat16) for _ in range(CHUNKS)]


def _expected():
    outs = []
    for x in _inputs():
        for l in range(N_LAYERS):
            x = Affine(l).forward(x)
        outs.append(x)
    return outs


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_codec():
    """The FP8 wire on the host for these CPU stages: the oracle's restatement of the reference
    codec (the product codec is CUDA-only)."""
    from oracle import wire_oracle as W

    def pack(t):
        q, s = W.pack(t.float().numpy())
        return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.from_numpy(s).to(torch.bfloat16)

    def unpack(q, s):
        return torch.from_numpy(W.unpack(q.view(torch.uint8).numpy(), s.float().numpy())).to(torch.bfloat16)

    return pack, unpack


def _expected_fp8(world):
    """The whole stack with every stage boundary passing through the wire codec."""
    pack, unpack = _oracle_codec()
    blocks = even_tiling(N_LAYERS, world)
    outs = []
    for x in _inputs():
        for b, block in enumerate(blocks):
            for l in block:
                x = Affine(l).forward(x)
            if b < len(blocks) - 1:
                x = unpack(*pack(x))
        outs.append(x)
    return outs


def _rank_main(rank, world, port, out_path, wire="bf16", depth=4, runs=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        block = even_tiling(N_LAYERS, world)[rank]
        pipe = Pipeline(StageStack([Affine(l) for l in block]), M, HIDDEN, rank, world, torch.device("cpu"),
                        depth=depth, wire=wire, codec=_oracle_codec() if wire == "fp8" else None)
        all_outs = []
        for r in range(runs):
            chunks = [(x.float() + r).to(torch.bfloat16) for x in _inputs()] if rank == 0 else None
            outs = [torch.empty(M, HIDDEN, dtype=torch.bfloat16) for _ in range(CHUNKS)] if rank == world - 1 else None
            pipe.run(CHUNKS, chunks, outs)
            all_outs.append(outs)
        if rank == world - 1:
            torch.save(all_outs[0] if runs == 1 else all_outs, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_even_tiling_front_loads_the_remainder():
    assert [len(r) for r in even_tiling(48, 8)] == [6] * 8
    assert [list(r) for r in even_tiling(7, 3)] == [[0, 1, 2], [3, 4], [5, 6]]
    assert [len(r) for r in even_tiling(61, 8)] == [8, 8, 8, 8, 8, 7, 7, 7]
    assert sum(len(r) for r in even_tiling(5, 2)) == 5


def test_single_stage_runs_locally():
    pipe = Pipeline(StageStack([Affine(l) for l in range(N_LAYERS)]), M, HIDDEN, 0, 1, torch.device("cpu"))
    got = pipe.run(CHUNKS, _inputs())
    for g, e in zip(got, _expected()):
        assert torch.equal(g, e)


@pytest.mark.parametrize("world", [2])
def test_two_stage_gloo_pipeline_matches_the_whole_stack(world):
    with tempfile.TemporaryDirectory() as d:
        out_path = os.path.join(d, "outs.pt")
        mp.start_processes(_rank_main, args=(world, _free_port(), out_path), nprocs=world, join=True,
                           start_method="spawn")
        got = torch.load(out_path)
    for g, e in zip(got, _expected()):
        assert torch.equal(g, e)


def test_two_stage_gloo_pipeline_with_the_fp8_wire():
    """The hop carries e4m3 codes + bf16 scale bits; the result equals the stack with the codec
    applied at the stage boundary, and differs from the bf16 wire (the codec is lossy)."""
    with tempfile.TemporaryDirectory() as d:
        out_path = os.path.join(d, "outs.pt")
        mp.start_processes(_rank_main, args=(2, _free_port(), out_path, "fp8"), nprocs=2, join=True,
                           start_method="spawn")
        got = torch.load(out_path)
    exp = _expected_fp8(2)
    for g, e in zip(got, exp):
        assert torch.equal(g, e)
    assert any(not torch.equal(g, e) for g, e in zip(got, _expected()))


def test_three_stage_pipeline_streams_runs_back_to_back():
    """The middle stage both receives (posted `depth` chunks ahead into a ring of 2) and sends; two
    runs follow each other with no barrier between them, and every chunk of both arrives in order."""
    runs = 2
    with tempfile.TemporaryDirectory() as d:
        out_path = os.path.join(d, "outs.pt")
        mp.start_processes(_rank_main, args=(3, _free_port(), out_path, "bf16", 2, runs), nprocs=3, join=True,
                           start_method="spawn")
        got = torch.load(out_path)
    for r in range(runs):
        for j, x in enumerate(_inputs()):
            x = (x.float() + r).to(torch.bfloat16)
            for l in range(N_LAYERS):
                x = Affine(l).forward(x)
            assert torch.equal(got[r][j], x), f"run {r} chunk {j}"


class _Failing(Affine):
    """A stand-in layer that raises on its `at`-th call: a stage that dies mid-stream."""

    def __init__(self, l, at):
        super().__init__(l)
        self.calls, self.at = 0, at

    def forward(self, x):
        self.calls += 1
        if self.calls == self.at:
            raise RuntimeError("simulated stage failure")
        return super().forward(x)


def _failing_rank_main(rank, world, port, out_dir):
    """Rank world-1 dies on its second chunk; every other rank must leave its run with an error
    (the hop to the dead stage fails, or the process group's short timeout ends the wait) instead
    of waiting for good. Each rank records how its run ended."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    status = "ok"
    try:
        block = even_tiling(N_LAYERS, world)[rank]
        layers = [Affine(l) for l in block]
        if rank == world - 1:
            layers[0] = _Failing(block[0], at=2)
        pipe = Pipeline(StageStack(layers), M, HIDDEN, rank, world, torch.device("cpu"), depth=2)
        outs = [torch.empty(M, HIDDEN, dtype=torch.bfloat16) for _ in range(CHUNKS)] if rank == world - 1 else None
        for r in range(3):
            pipe.run(CHUNKS, _inputs() if rank == 0 else None, outs)
            pipe.flush()
        dist.barrier()
    except Exception as e:   # noqa: BLE001  (the test reads how each rank's run ended)
        status = f"error: {type(e).__name__}"
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write(status)
    if status == "ok":
        dist.destroy_process_group()
    os._exit(0)   # a failed group is not torn down: leave without waiting on it


def test_a_stage_that_dies_ends_the_other_ranks_runs_with_an_error():
    """Failure detection on the host: the stage that raised reports it, and its neighbour's run ends
    with an error within the process group's timeout rather than hanging."""
    import time
    world = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_failing_rank_main, args=(r, world, port, d)) for r in range(world)]
        t0 = time.time()
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        hung = [p.pid for p in procs if p.is_alive()]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert not hung, "a rank did not finish after its peer died"
        status = [open(os.path.join(d, f"rank{r}")).read() for r in range(world)]
        assert status[world - 1].startswith("error: RuntimeError"), status
        assert status[0].startswith("error"), status
        assert time.time() - t0 < 120
