"""ctypes binding of ``include/lewm_b200.h`` (``liblewm_b200.so``, built in-tree).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises. The library is the only compute path of this package.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "liblewm_b200.so"

STATUS = {
    0: "LEWM_OK",
    1: "LEWM_INVALID_ARG",
    2: "LEWM_UNSUPPORTED_SHAPE",
    3: "LEWM_DEVICE_TIMEOUT",
    4: "LEWM_NUMERIC_NAN",
    5: "LEWM_CUDA_ERROR",
    6: "LEWM_OUT_OF_MEMORY",
}
NORM_CODE = {"none": 0, "layernorm": 1, "batchnorm": 2}


class LewmError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.status_name = STATUS.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


class LewmInvalidArgument(LewmError, ValueError):
    """LEWM_INVALID_ARG: the reference raises ValueError for the same inputs."""


class ModelDescC(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "dim", "depth", "heads", "dim_head", "mlp_dim", "action_dim", "smoothed_dim", "embed_hidden",
        "num_frames", "pred_proj_hidden", "pred_proj_norm")]


class PlanDescC(C.Structure):
    _fields_ = [
        ("n_envs", C.c_int32), ("horizon", C.c_int32), ("history", C.c_int32), ("history_size", C.c_int32),
        ("num_samples", C.c_int32), ("topk", C.c_int32), ("n_steps", C.c_int32), ("sample_decay", C.c_double),
        ("bucket", C.c_int32), ("elite_retention", C.c_int32), ("beta", C.c_float), ("time_axis_raw", C.c_int32),
        ("action_block", C.c_int32), ("momentum_alpha", C.c_float), ("return_best_elite", C.c_int32),
        ("clip_actions", C.c_int32), ("seed", C.c_uint64), ("plan_index", C.c_uint64),
        ("sample_counts", C.POINTER(C.c_int32)),
    ]


class EncoderDescC(C.Structure):
    _fields_ = [("image_size", C.c_int32), ("patch_size", C.c_int32), ("channels", C.c_int32),
                ("hidden", C.c_int32), ("depth", C.c_int32), ("heads", C.c_int32), ("mlp_dim", C.c_int32),
                ("ln_eps", C.c_float), ("proj_hidden", C.c_int32), ("proj_out", C.c_int32),
                ("proj_norm", C.c_int32), ("proj_eps", C.c_float)]


class PlanTraceC(C.Structure):
    _fields_ = [("costs", C.c_void_p), ("topk_idx", C.c_void_p), ("topk_val", C.c_void_p),
                ("mean", C.c_void_p), ("std", C.c_void_p), ("candidates", C.c_void_p)]


_lib = None
ABI_VERSION = 3  # LEWM_ABI_VERSION of include/lewm_b200.h this binding follows

# name -> (restype, argtypes)
SIGNATURES = {
    "lewm_weight_count": (C.c_size_t, [C.POINTER(ModelDescC)]),
    "lewm_create": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(ModelDescC), C.c_void_p, C.c_size_t, C.c_int]),
    "lewm_destroy": (None, [C.c_void_p]),
    "lewm_last_error": (C.c_char_p, [C.c_void_p]),
    "lewm_model_cost": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                  C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "lewm_model_cost_grad": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                       C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p]),
    "lewm_sample_counts": (C.c_int, [C.POINTER(PlanDescC), C.c_void_p, C.c_int32, C.POINTER(C.c_int64)]),
    "lewm_plan": (C.c_int, [C.c_void_p, C.POINTER(PlanDescC), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                            C.POINTER(PlanTraceC), C.c_void_p]),
    "lewm_topk_refit": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                  C.c_int32, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p]),
    "lewm_sample_candidates": (C.c_int, [C.c_void_p, C.POINTER(PlanDescC), C.c_int32, C.c_int32, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "lewm_sample_candidates_noalloc": (C.c_int, [C.POINTER(PlanDescC), C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_int32, C.c_void_p]),
    "lewm_coloring_matrix": (C.c_int, [C.c_int32, C.c_double, C.c_void_p]),
    "lewm_sync_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lewm_set_wait_limit": (C.c_int, [C.c_void_p, C.c_uint64]),
    "lewm_set_model_cost_autocast": (C.c_int, [C.c_void_p, C.c_int32]),
    "lewm_wait_selftest": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lewm_abi_version": (C.c_int32, []),
    "lewm_profile_plan": (C.c_int, [C.c_void_p, C.POINTER(PlanDescC), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "lewm_encoder_weight_count": (C.c_size_t, [C.POINTER(EncoderDescC)]),
    "lewm_encoder_create": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(EncoderDescC), C.c_void_p, C.c_size_t,
                                      C.c_int]),
    "lewm_encode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "lewm_encode_u8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                 C.c_void_p, C.c_void_p]),
    "lewm_encoder_sync_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lewm_encoder_last_error": (C.c_char_p, [C.c_void_p]),
    "lewm_encoder_destroy": (None, [C.c_void_p]),
}
KERNEL_CLASSES = ("embed", "adaln", "qkv_attn", "out_proj", "fc1", "fc2", "final", "sample", "refit", "prep0", "ffn",
                  "ln_operand", "tile_call", "fp32_cost")


def lib():
    """Load liblewm_b200.so once. Raises if it is missing: there is no CPU fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing; build it with `python -m lewm_flash_b200.build` "
            "(the LeWM B200 path has no CPU fallback)")
    h = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(h, name)
        fn.restype = res
        fn.argtypes = args
    got = h.lewm_abi_version()
    if got != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH} has C ABI version {got}, this binding needs {ABI_VERSION}; rebuild it")
    _lib = h
    return h


def check(status: int, ctx=None) -> None:
    if status == 0:
        return
    msg = lib().lewm_last_error(ctx)
    text = msg.decode() if msg else ""
    if status == 1:
        raise LewmInvalidArgument(status, text)
    raise LewmError(status, text)


def check_encoder(status: int, enc=None) -> None:
    """``check`` for the encoder entry points (their error text lives on the encoder)."""
    if status == 0:
        return
    msg = lib().lewm_encoder_last_error(enc)
    text = msg.decode() if msg else ""
    if status == 1:
        raise LewmInvalidArgument(status, text)
    raise LewmError(status, text)
