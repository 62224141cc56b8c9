"""The bounded-wait failure path, exercised on the GPU without a fault or a hang.

The reference's failure story is host-side watchdogs (shard/coordinate.py:131-205). Here every wait
in the tensor-core kernels is bounded: a wait that runs out sets the workspace error flag, the CTA
drains its copies and MMAs in flight, frees its tensor memory and returns. sb_debug_set_wait_limit
shortens the consumer-side waits (on operands and accumulators) to one poll, which the first wait on
a copy still in flight cannot meet, so that wait runs out: the forward returns, the flag reads 1,
and the next forward with the normal limit on the same workspace is correct again."""
import numpy as np
import pytest
import torch

from cases import case_config, case_inputs, load_golden
from oracle import moe_oracle as O
from shard_b200 import _lib
from shard_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _restore_limit():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    _lib.check(_lib.lib().sb_debug_set_wait_limit(0), "sb_debug_set_wait_limit")


# the verify kernel (round-robin items), the prefill kernel, and the verify kernel on FP8 experts,
# whose items come from the launch's item counter through the producer's item queue
@pytest.mark.parametrize("name,prefill", [("c0_nvfp4_m8", 1), ("c0_nvfp4_m8", 2), ("small_fp8_noshared_m16", 1)])
def test_wait_that_runs_out_sets_the_flag_and_the_next_forward_recovers(name, prefill):
    g = load_golden(name)
    cfg, m, xs, _ = case_config(name)
    lay = S.device_layer(cfg, 0, "cuda", prefill=prefill)
    x, ids = case_inputs(cfg, m, xs)
    x = x.cuda()
    y0 = lay.forward(x)
    torch.cuda.synchronize()
    assert lay.device_error() == 0
    L = _lib.lib()
    _lib.check(L.sb_debug_set_wait_limit(1), "sb_debug_set_wait_limit")
    lay.forward(x)
    torch.cuda.synchronize()
    assert lay.device_error() == 1, "a consumer wait limited to one poll must run out"
    _lib.check(L.sb_debug_set_wait_limit(0), "sb_debug_set_wait_limit")
    y2 = lay.forward(x)
    torch.cuda.synchronize()
    assert lay.device_error() == 0
    assert torch.equal(y2, y0), "the forward after a timed-out one must be unchanged"
    err = O.max_rel_err(y2.float().cpu().numpy(), O.bf16_from_bits(g["y_bits"]))
    assert err < 1e-2
