"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

Loading fails loudly when the library has not been built: there is no fallback.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import os

# MOE_B200_LIB selects another build of the library (e.g. the MOE_TRACE build).
LIB_PATH = Path(os.environ.get("MOE_B200_LIB") or Path(__file__).resolve().with_name("libmoe_b200.so"))

OK = 0
ERR_ARG = 1
ERR_WORKSPACE = 2
ERR_CUDA = 3
ERR_DEVICE = 4
ERR_TIMEOUT = 5

EXPORTED = (
    "moe_b200_workspace_size",
    "moe_b200_workspace_layout",
    "moe_b200_workspace_init",
    "moe_b200_forward",
    "moe_b200_forward_routed",
    "moe_b200_forward_ep",
    "moe_b200_route",
    "moe_b200_device_status",
    "moe_b200_last_error",
    "moe_b200_last_launch_count",
    "moe_b200_timer_create",
    "moe_b200_timer_destroy",
    "moe_b200_forward_timed",
    "moe_b200_timer_read",
    "moe_b200_route_noalloc",
)


class MoeArgs(ctypes.Structure):
    _fields_ = [
        ("routing_logits", ctypes.c_void_p),
        ("routing_bias", ctypes.c_void_p),
        ("hidden_states", ctypes.c_void_p),
        ("hidden_states_scale", ctypes.c_void_p),
        ("gemm1_weights", ctypes.c_void_p),
        ("gemm1_weights_scale", ctypes.c_void_p),
        ("gemm2_weights", ctypes.c_void_p),
        ("gemm2_weights_scale", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int32),
        ("num_local_experts", ctypes.c_int32),
        ("local_expert_offset", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
    ]


MAX_RANKS = 8


class MoeEp(ctypes.Structure):
    """moe_b200_ep: expert parallelism over peer memory (include/moe_b200.h)."""
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("shard_tokens", ctypes.c_int32),
        ("epoch", ctypes.c_uint32),
        ("recv", ctypes.c_void_p * MAX_RANKS),
        ("signal", ctypes.c_void_p * MAX_RANKS),
        ("out_shard", ctypes.c_void_p),
        ("wait_limit_us", ctypes.c_uint32),
    ]


class MoeLayout(ctypes.Structure):
    _fields_ = [(name, ctypes.c_size_t) for name in (
        "plan", "topk_idx", "topk_w", "tok_nloc", "tok_rows", "e_count", "e_start", "row_token",
        "row_weight", "c_hi", "c_lo", "c_scale", "status", "trace", "r_max", "r_pad", "total")]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built; run `python -m moe_swarm_b200.build` "
            "(this package has no CPU or PyTorch fallback)")
    l = ctypes.CDLL(str(LIB_PATH))
    vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32
    l.moe_b200_workspace_size.argtypes = [i32, i32]
    l.moe_b200_workspace_size.restype = sz
    l.moe_b200_workspace_layout.argtypes = [i32, i32, ctypes.POINTER(MoeLayout)]
    l.moe_b200_workspace_layout.restype = ctypes.c_int
    l.moe_b200_workspace_init.argtypes = [vp, sz, i32, i32, vp]
    l.moe_b200_workspace_init.restype = ctypes.c_int
    l.moe_b200_forward.argtypes = [ctypes.POINTER(MoeArgs), vp, sz, vp]
    l.moe_b200_forward.restype = ctypes.c_int
    l.moe_b200_forward_routed.argtypes = [ctypes.POINTER(MoeArgs), vp, vp, vp, sz, vp]
    l.moe_b200_forward_routed.restype = ctypes.c_int
    l.moe_b200_forward_ep.argtypes = [ctypes.POINTER(MoeArgs), ctypes.POINTER(MoeEp), vp, sz, vp]
    l.moe_b200_forward_ep.restype = ctypes.c_int
    l.moe_b200_route.argtypes = [ctypes.POINTER(MoeArgs), vp, sz, vp]
    l.moe_b200_route.restype = ctypes.c_int
    l.moe_b200_device_status.argtypes = [vp, sz, i32, i32, vp, i32]
    l.moe_b200_device_status.restype = ctypes.c_int
    l.moe_b200_last_error.argtypes = []
    l.moe_b200_last_error.restype = ctypes.c_char_p
    l.moe_b200_last_launch_count.argtypes = []
    l.moe_b200_last_launch_count.restype = ctypes.c_int
    l.moe_b200_timer_create.argtypes = []
    l.moe_b200_timer_create.restype = vp
    l.moe_b200_timer_destroy.argtypes = [vp]
    l.moe_b200_timer_destroy.restype = None
    l.moe_b200_forward_timed.argtypes = [ctypes.POINTER(MoeArgs), vp, sz, vp, vp]
    l.moe_b200_forward_timed.restype = ctypes.c_int
    l.moe_b200_timer_read.argtypes = [vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32), i32]
    l.moe_b200_timer_read.restype = ctypes.c_int
    l.moe_b200_route_noalloc.argtypes = [ctypes.POINTER(MoeArgs), vp, vp, vp, vp, vp, vp]
    l.moe_b200_route_noalloc.restype = ctypes.c_int
    _lib = l
    return l


def last_error() -> str:
    return lib().moe_b200_last_error().decode(errors="replace")


def layout(T: int, E: int) -> MoeLayout:
    out = MoeLayout()
    rc = lib().moe_b200_workspace_layout(int(T), int(E), ctypes.byref(out))
    if rc != OK:
        raise ValueError(f"moe_b200_workspace_layout({T}, {E}) failed: {last_error()}")
    return out
