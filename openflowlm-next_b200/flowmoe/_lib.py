"""ctypes binding of libflowmoe.so (the C ABI in include/flowmoe.h).

The library is built in-tree by ``openflowlm-next_b200/build.py`` (``__graft_entry__.build()``). There
is no fallback: if the shared object is missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libflowmoe.so"

FM_OK = 0
FM_EINVAL_SHAPE = 1
FM_EINVAL_EXPERT = 2
FM_ECUDA = 3
FM_ENCCL = 4
FM_ETIMEOUT = 5
FM_EWORKSPACE = 6
FM_F32 = 0
FM_BF16 = 1

_STATUS = {FM_EINVAL_SHAPE: "FM_EINVAL_SHAPE", FM_EINVAL_EXPERT: "FM_EINVAL_EXPERT", FM_ECUDA: "FM_ECUDA",
           FM_ENCCL: "FM_ENCCL", FM_ETIMEOUT: "FM_ETIMEOUT", FM_EWORKSPACE: "FM_EWORKSPACE"}


class FmLayer(ctypes.Structure):
    """``fm_layer`` (include/flowmoe.h)."""
    _fields_ = [("hidden", ctypes.c_int32), ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("shared_ffn", ctypes.c_int32), ("e_begin", ctypes.c_int32),
                ("e_local", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("gate_up", ctypes.c_void_p), ("down", ctypes.c_void_p), ("shared_gate_up", ctypes.c_void_p),
                ("shared_down", ctypes.c_void_p), ("router", ctypes.c_void_p), ("router_bias", ctypes.c_void_p)]


FM_EP_MAX_RANKS = 16


class FmEpGroup(ctypes.Structure):
    """``fm_ep_group`` (include/flowmoe.h)."""
    _fields_ = [("rank", ctypes.c_int32), ("n_ranks", ctypes.c_int32), ("t_cap", ctypes.c_int32),
                ("timeout_ms", ctypes.c_int32), ("sym", ctypes.c_void_p * FM_EP_MAX_RANKS)]


P = ctypes.c_void_p
I32 = ctypes.c_int32
SZ = ctypes.c_size_t
LP = ctypes.POINTER(FmLayer)

# name -> argtypes; every entry point returns int
SIGNATURES = {
    "fm_last_error": [ctypes.c_char_p, SZ],
    "fm_version": [ctypes.c_char_p, SZ],
    "fm_q4_1_to_tiles": [P, I32, I32, P, P],
    "fm_pool_to_q4_1": [P, I32, I32, I32, I32, P, P, P],
    "fm_rmsnorm_bf16": [P, P, ctypes.c_float, I32, I32, P, P],
    "fm_tiles_to_q4_1": [P, I32, I32, P, P],
    "fm_gate_up_to_tiles": [P, P, I32, I32, P, P],
    "fm_tiles_narrow_scales": [P, ctypes.c_int64, P],
    "fm_router_pack": [P, P, I32, I32, P, P],
    "fm_workspace_size": [LP, I32, ctypes.POINTER(SZ)],
    "fm_router_topk": [LP, P, I32, I32, P, P, P, P, P, SZ, P],
    "fm_moe_block": [LP, P, I32, P, P, P, P, I32, I32, P, P, SZ, P],
    "fm_moe_layer": [LP, P, I32, P, I32, I32, P, P, P, P, SZ, P],
    "fm_moe_dispatch": [LP, P, I32, I32, P, P, P, P, P, SZ, P],
    "fm_moe_layer_norm": [LP, P, P, ctypes.c_float, I32, I32, P, P, P, P, SZ, P],
    "fm_moe_layer_noalloc": [LP, P, I32, P, I32, I32, P, P, P, P],
    "fm_q4_gemm_workspace_size": [I32, I32, I32, I32, ctypes.POINTER(SZ)],
    "fm_q4_gemm": [P, I32, I32, P, I32, I32, P, P, SZ, P],
    "fm_ep_workspace_size": [LP, I32, I32, I32, ctypes.POINTER(SZ)],
    "fm_ep_dispatch": [LP, P, I32, I32, I32, P, P, P, P, P, P, P, P, SZ, P],
    "fm_ep_experts": [LP, P, I32, P, I32, P, P, P, I32, I32, P, P, P, SZ, P],
    "fm_ep_combine": [LP, P, P, P, P, P, I32, I32, P],
    "fm_ep_peer_sizes": [LP, ctypes.c_void_p, ctypes.POINTER(SZ), ctypes.POINTER(SZ)],
    "fm_ep_peer_layer": [LP, ctypes.c_void_p, P, I32, P, I32, I32, P, P, P, P, SZ, P],
    "fm_ipc_alloc": [SZ, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p],
    "fm_ipc_open": [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)],
    "fm_ipc_close": [P],
    "fm_ipc_free": [P],
    "fm_moe_check": [P, P],
    "fm_launch_count": [ctypes.POINTER(ctypes.c_ulonglong)],
    "fm_profile": [I32],
    "fm_profile_read": [ctypes.POINTER(ctypes.c_double), I32],
}

STAGES = ("to_bf16", "router", "dispatch", "gather", "gate_up", "down", "combine")


class FlowMoeError(RuntimeError):
    """A non-zero status from libflowmoe (the reference raises std::runtime_error in these cases)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS.get(code, code)}: {msg}")
        self.code = code


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python openflowlm-next_b200/build.py` "
                          "(or __graft_entry__.build()); flowmoe has no CPU fallback")
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    return lib


lib = _load()


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib.fm_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != FM_OK:
        raise FlowMoeError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))


def launch_count() -> int:
    n = ctypes.c_ulonglong(0)
    call("fm_launch_count", ctypes.byref(n))
    return n.value


def profile(enable: bool) -> None:
    call("fm_profile", 1 if enable else 0)


def profile_read() -> dict:
    """Summed ms per stage since the last read (synchronises on the recorded events)."""
    buf = (ctypes.c_double * len(STAGES))()
    call("fm_profile_read", buf, len(STAGES))
    return {n: buf[i] for i, n in enumerate(STAGES)}
