"""ctypes binding of libshard_b200.so (the C ABI in include/shard_b200.h).

The library is loaded from the package directory. There is no fallback: if it is missing or
fails to load, every entry point raises, so a forward can never silently run on something else.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libshard_b200.so")

SB_OK = 0
STATUS = {0: "SB_OK", -1: "SB_ERR_ARG", -2: "SB_ERR_SHAPE", -3: "SB_ERR_FORMAT", -4: "SB_ERR_WORKSPACE",
          -5: "SB_ERR_CUDA", -6: "SB_ERR_UNSUPPORTED"}

ABI_VERSION = 7
SCORE = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}
MAT_PLAIN, MAT_W13 = 0, 1
KIND_TC = 4                      # OR'ed into a tiling kind: the tensor-core (tcgen05) layout
LAYOUT_FRAGMENT, LAYOUT_TC = 0, 1
MODE_V4, MODE_K3 = 0, 1

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_fp = ctypes.POINTER(ctypes.c_float)


class SbMoeLayer(ctypes.Structure):
    """struct sb_moe_layer (include/shard_b200.h)."""
    _fields_ = [
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("n_experts", ctypes.c_int32),
        ("topk", ctypes.c_int32), ("expert_fmt", ctypes.c_int32), ("has_shared", ctypes.c_int32),
        ("score_func", ctypes.c_int32), ("act_pow2", ctypes.c_int32),
        ("route_scale", ctypes.c_float), ("swiglu_limit", ctypes.c_float),
        ("gate_w", _vp), ("gate_bias", _vp), ("tid2eid", _vp), ("vocab", ctypes.c_int64),
        ("w13", _vp), ("w13_s", _vp), ("w13_ts", _vp), ("w2", _vp), ("w2_s", _vp), ("w2_ts", _vp),
        ("sh_w13", _vp), ("sh_w13_s", _vp), ("sh_w2", _vp), ("sh_w2_s", _vp),
        ("layout", ctypes.c_int32), ("logits_bf16", ctypes.c_int32), ("no_renorm", ctypes.c_int32),
        ("prefill", ctypes.c_int32), ("fp8_pow2", ctypes.c_int32), ("mode", ctypes.c_int32),
        ("situ_beta", ctypes.c_float), ("situ_linear_beta", ctypes.c_float),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "sb_abi_version": (_int, []),
    "sb_last_error": (ctypes.c_char_p, []),
    "sb_tiled_bytes": (_sz, [_int, _i64, _i64]),
    "sb_tiled_scale_bytes": (_sz, [_int, _int, _i64, _i64]),
    "sb_tile_weights": (_int, [_int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sb_tile_scales": (_int, [_int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sb_act_quant": (_int, [_vp, _i64, _i64, _int, _vp, _vp, _vp]),
    "sb_qgemm_workspace_bytes": (_sz, [_int, _int, _i64, _i64, _i64]),
    "sb_qgemm": (_int, [_int, _int, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _sz, _vp]),
    "sb_qgemm_static": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "sb_qgemm_static_error": (_int, [ctypes.POINTER(ctypes.c_int), _vp]),
    "sb_moe_workspace_bytes": (_sz, [ctypes.POINTER(SbMoeLayer), _i64]),
    "sb_moe_forward": (_int, [ctypes.POINTER(SbMoeLayer), _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sb_moe_forward_profiled": (_int, [ctypes.POINTER(SbMoeLayer), _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp,
                                        ctypes.POINTER(_vp)]),
    "sb_moe_forward_routed": (_int, [ctypes.POINTER(SbMoeLayer), _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sb_moe_route": (_int, [ctypes.POINTER(SbMoeLayer), _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sb_moe_forward_wire": (_int, [ctypes.POINTER(SbMoeLayer), _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                   _vp]),
    "sb_wire_pack": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "sb_wire_unpack": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "sb_selftest_formats": (_int, [_vp, _vp]),
    "sb_debug_set_wait_limit": (_int, [_i64]),
    "sb_residual_rmsnorm": (_int, [_vp, _vp, _i64, _i64, _vp, ctypes.c_float, _vp, _vp]),
}

_LIB = None


class ShardB200Error(RuntimeError):
    pass


def lib():
    """The loaded library. Raises if it is missing: the CUDA path is the only path."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ShardB200Error(f"{LIB_PATH} is missing; build it with `python -m shard_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        if L.sb_abi_version() != ABI_VERSION:
            raise ShardB200Error(f"ABI version mismatch: library {L.sb_abi_version()}, binding {ABI_VERSION}")
        _LIB = L
    return _LIB


def check(rc: int, what: str):
    if rc != SB_OK:
        msg = lib().sb_last_error().decode(errors="replace")
        raise ShardB200Error(f"{what}: {STATUS.get(rc, rc)}: {msg}")


def ptr(t) -> int:
    """Device (or host) address of a tensor, or None for None."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
