"""Shared helpers: rebuild a golden case's seeded layer for the oracle and for the GPU path."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from make_golden import CASES, case_config, case_inputs  # noqa: F401  (case table lives with the generator)
from oracle import moe_oracle as O
from shard_b200 import formats as F
from shard_b200 import synth as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name):
    g = np.load(os.path.join(GOLDEN, f"moe_{name}.npz"))
    return {k: g[k] for k in g.files}


def np_expert(ew):
    return tuple(t.cpu().numpy() for t in (ew.w13, ew.w13_s, ew.w13_ts, ew.w2, ew.w2_s, ew.w2_ts))


class SeededLayer:
    """The seeded layer of a config: lazily generated experts, cached, plus the oracle view."""

    def __init__(self, cfg, layer=0, pow2=True):
        self.cfg, self.layer, self.pow2 = cfg, layer, pow2
        self.gate_w, self.gate_b = S.make_gate(cfg, layer)
        self._experts = {}
        self.shared = S.make_expert(cfg, layer, -1, F.FMT_FP8) if cfg.n_shared else None

    def expert(self, e):
        if e not in self._experts:
            self._experts[e] = S.make_expert(self.cfg, self.layer, e)
        return self._experts[e]

    def oracle(self):
        c = self.cfg
        return O.OracleLayer(
            hidden=c.hidden, inter=c.inter, topk=c.topk, score_func=c.score_func,
            route_scale=c.route_scale, swiglu_limit=c.swiglu_limit, expert_fmt=c.expert_fmt,
            gate_w=self.gate_w.float().numpy(), gate_b=self.gate_b.numpy(),
            expert=lambda e: np_expert(self.expert(e)),
            shared=np_expert(self.shared) if self.shared is not None else None, pow2=self.pow2)


def expert_shas(golden):
    return json.loads(str(golden["expert_sha"]))
