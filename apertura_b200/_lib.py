"""ctypes binding of libapt_moe.so (the C ABI declared in include/apt_moe.h).

The library is built in-tree by ``apertura_b200.build``.  There is no fallback:
if the shared object is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libapt_moe.so")

APT_OK = 0
STATUS_NAMES = {0: "APT_OK", 1: "APT_ERR_INVALID", 2: "APT_ERR_UNSUPPORTED", 3: "APT_ERR_CUDA",
                4: "APT_ERR_NCCL", 5: "APT_ERR_TIMEOUT", 6: "APT_ERR_STATE"}

# Every symbol include/apt_moe.h declares, in header order.
EXPORTED = [
    "apt_moe_config_from_json", "apt_moe_create", "apt_moe_destroy", "apt_moe_clone_shared", "apt_moe_last_error",
    "apt_moe_version", "apt_moe_load_router", "apt_moe_load_experts_bf16",
    "apt_moe_load_experts_quant", "apt_moe_route", "apt_moe_route_weights", "apt_moe_experts",
    "apt_moe_experts_dense", "apt_moe_forward", "apt_moe_layer_forward", "apt_moe_decoder_ff", "apt_moe_mlp_forward", "apt_moe_decoder_ff_full", "apt_moe_forward_host", "apt_moe_forward_host_async", "apt_moe_ep_dispatch",
    "apt_moe_ep_combine", "apt_moe_experts_grouped", "apt_moe_sync",
    "apt_moe_last_counts", "apt_moe_last_launches", "apt_moe_set_gemv_max_tokens",
    "apt_moe_set_sm_limit", "apt_moe_set_fused_decode", "apt_moe_set_q4_gemm",
    "apt_moe_set_timing", "apt_moe_stage_times", "apt_moe_route_noalloc",
    "apt_moe_nccl_unique_id", "apt_moe_create_ep", "apt_moe_ep_destroy", "apt_moe_ep_last_error",
    "apt_moe_ep_load_router", "apt_moe_ep_load_experts_bf16", "apt_moe_ep_forward",
    "apt_moe_ep_placement", "apt_moe_ep_stats", "apt_moe_selftest_wait",
    "apt_moe_ep_set_transport", "apt_moe_ep_get_transport", "apt_moe_ep_sync",
]

STAGES = ["router_scores", "router_select", "dispatch_count", "dispatch", "gather", "gate_up",
          "down", "combine"]


class AptMoeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int),
        ("num_experts", ctypes.c_int),
        ("top_k_experts", ctypes.c_int),
        ("moe_intermediate_size", ctypes.c_int),
        ("rms_norm_eps", ctypes.c_float),
        ("enable_moe_block", ctypes.c_int),
        ("moe_sparse", ctypes.c_int),
        ("quant_bits", ctypes.c_int),
        ("quant_group_size", ctypes.c_int),
        ("max_tokens", ctypes.c_int),
        ("device", ctypes.c_int),
    ]


class AptError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with `python -m apertura_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    P, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    cfgp = ctypes.POINTER(AptMoeConfig)
    hp = ctypes.c_void_p
    sig = {
        "apt_moe_config_from_json": ([ctypes.c_char_p, cfgp], i32),
        "apt_moe_create": ([cfgp, ctypes.POINTER(ctypes.c_void_p)], i32),
        "apt_moe_destroy": ([hp], i32),
        "apt_moe_clone_shared": ([hp, cfgp, ctypes.POINTER(ctypes.c_void_p)], i32),
        "apt_moe_last_error": ([hp], ctypes.c_char_p),
        "apt_moe_version": ([], ctypes.c_char_p),
        "apt_moe_load_router": ([hp, P, P, P, i32], i32),
        "apt_moe_load_experts_bf16": ([hp, P, P, i32], i32),
        "apt_moe_load_experts_quant": ([hp, P, P, P, P, P, P, i32, i32, i32], i32),
        "apt_moe_route": ([hp, P, i32, P, P, P], i32),
        "apt_moe_route_weights": ([hp, P, i32, P, P], i32),
        "apt_moe_experts": ([hp, P, P, P, i32, P, P], i32),
        "apt_moe_experts_dense": ([hp, P, P, i32, P, P], i32),
        "apt_moe_forward": ([hp, P, P, i32, P, P, P, P], i32),
        "apt_moe_forward_host": ([hp, P, i32, P, P], i32),
        "apt_moe_forward_host_async": ([hp, P, i32, P, P], i32),
        "apt_moe_layer_forward": ([hp, P, P, P, i32, P, P], i32),
        "apt_moe_decoder_ff": ([hp, P, P, P, P, P, P, i32, P, P], i32),
        "apt_moe_mlp_forward": ([hp, P, i32, P, P], i32),
        "apt_moe_decoder_ff_full": ([hp, hp, P, P, P, P, P, P, i32, P, P], i32),
        "apt_moe_ep_dispatch": ([hp, P, i32, P, P, P, P, P], i32),
        "apt_moe_ep_combine": ([hp, P, P, P, i32, P, P], i32),
        "apt_moe_experts_grouped": ([hp, P, i32, P, P, i32, P, P], i32),
        "apt_moe_sync": ([hp], i32),
        "apt_moe_last_counts": ([hp, P], i32),
        "apt_moe_last_launches": ([hp], i32),
        "apt_moe_set_gemv_max_tokens": ([hp, i32], i32),
        "apt_moe_set_fused_decode": ([hp, i32], i32),
        "apt_moe_set_q4_gemm": ([hp, i32], i32),
        "apt_moe_set_sm_limit": ([hp, i32], i32),
        "apt_moe_set_timing": ([hp, i32], i32),
        "apt_moe_stage_times": ([hp, P], i32),
        "apt_moe_route_noalloc": ([P, i32, P, P, P, i32, i32, i32, f32, P, P, P], i32),
        "apt_moe_nccl_unique_id": ([P], i32),
        "apt_moe_selftest_wait": ([hp, i32, P], i32),
        "apt_moe_create_ep": ([cfgp, P, i32, i32, P, i32, ctypes.POINTER(ctypes.c_void_p)], i32),
        "apt_moe_ep_destroy": ([P], i32),
        "apt_moe_ep_last_error": ([P], ctypes.c_char_p),
        "apt_moe_ep_load_router": ([P, P, P, P, i32], i32),
        "apt_moe_ep_load_experts_bf16": ([P, P, P, i32], i32),
        "apt_moe_ep_forward": ([P, P, i32, P, P], i32),
        "apt_moe_ep_placement": ([P, i32, i32, i32, P], i32),
        "apt_moe_ep_stats": ([P, ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
        "apt_moe_ep_set_transport": ([P, i32], i32),
        "apt_moe_ep_get_transport": ([P, ctypes.POINTER(i32)], i32),
        "apt_moe_ep_sync": ([P], i32),
    }
    for name, (argtypes, restype) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = L
    return L


def check(status: int, handle=None) -> None:
    if status != APT_OK:
        msg = ""
        if handle:
            raw = lib().apt_moe_last_error(handle)
            msg = raw.decode() if raw else ""
        raise AptError(status, msg)
