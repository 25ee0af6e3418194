"""ctypes binding of libminiep_b200.so (the C ABI in include/miniep_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises. Build it with ``python -m miniep_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libminiep_b200.so"

MEP_OK = 0
MEP_F32 = 0
MEP_BF16 = 1
IPC_HANDLE_BYTES = 64
# step-timeline slots (MEP_TL_* of include/miniep_b200.h): name -> slot; a
# stage name has its start at the slot and its end at slot + 1
TL_SLOTS = 24
TL_STAGES = {"norm": 1, "router": 3, "route": 5, "dispatch": 9, "fanout": 12, "gemm1": 14,
             "gemm2": 16, "combine": 19}
TL_MARKS = {"barrier_end": 0, "counts_sent": 7, "layout": 8, "data_in": 11, "results_in": 18,
            "route_hist": 21, "route_sync": 22}

_P = C.c_void_p
_I64 = C.c_int64
_I = C.c_int

# name -> argtypes (every function returns int unless listed in _RESTYPES)
SIGNATURES = {
    "mep_version": [],
    "mep_last_error": [_P],
    "mep_ctx_create": [_I, _I, _I, _I, _I, _I, _I, _I, _I64, _I, _I64, C.POINTER(_P)],
    "mep_ctx_destroy": [_P],
    "mep_ipc_handle": [_P, _P],
    "mep_ipc_open": [_P, _I, _P],
    "mep_set_placement": [_P, _I, _P, _P, _I],
    "mep_reset_rr": [_P, _P],
    "mep_dest_ranks": [_P, _I, _P, _I64, _P, _P],
    "mep_router_topk": [_P, _P, _P, _P, _I64, _P, _P, _P, _P],
    "mep_moe_forward": [_P, _I, _P, _P, _P, _P, _I64, _P, _P, _I, _P, _P],
    "mep_moe_block": [_P, _I, _P, _P, _P, _P, _P, _I64, _P, _P, _I, C.c_float, _P, _P, _P, _P],
    "mep_rmsnorm": [_P, _P, _P, C.c_float, _I64, _P, _P],
    "mep_moe_block_from_h": [_P, _I, _P, _P, C.c_float, _P, _P, _P, _I64, _P, _P, _I, C.c_float,
                             _P, _P, _P, _P, _P],
    "mep_route": [_P, _I, _P, _P, _I64, _I, _P],
    "mep_dispatch": [_P, _P, _P, _I64, _P],
    "mep_expert_ffn": [_P, _P, _P, _I, _P],
    "mep_combine": [_P, _P, _P, _I64, _P, C.c_float, _P, _P, _P],
    "mep_read_stats": [_P, _P, _P, _P],
    "mep_reset_stats": [_P, _P],
    "mep_last_recv_rows": [_P, C.POINTER(_I64), _P],
    "mep_check": [_P],
    "mep_set_option": [_P, C.c_char_p, _I64],
    "mep_debug_wait": [_P, C.c_uint32, _I64, _P],
    "mep_barrier": [_P, _P],
    "mep_read_timeline": [_P, _P, _P],
    "mep_dest_ranks_noalloc": [_I, _I, _P, _P, _I, _P, _P, _I64, _P, _P],
}
_RESTYPES = {"mep_last_error": C.c_char_p}

_lib = None
_lock = threading.Lock()


class MEPError(RuntimeError):
    """A libminiep_b200 call failed (bad argument, CUDA error or device error)."""


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise MEPError(f"{LIB_PATH} is missing: build it with "
                               f"`python -m miniep_b200.build` (nvcc, sm_100a)")
            l = C.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(l, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = l
    return _lib


def last_error(ctx) -> str:
    msg = lib().mep_last_error(ctx)
    return msg.decode() if msg else ""


def check(rc: int, ctx=None, what: str = "") -> None:
    if rc != MEP_OK:
        raise MEPError(f"{what or 'libminiep_b200'} failed (code {rc}): {last_error(ctx)}")


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()
