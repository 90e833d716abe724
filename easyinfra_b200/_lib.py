"""ctypes binding of libb200moe.so (the C ABI declared in include/b200moe.h).

The library is loaded from the package directory, where ``easyinfra_b200.build``
writes it.  There is no fallback: if the library is missing or the current device is
not an sm_100 part, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libb200moe.so")
_lock = threading.Lock()
_lib = None

c_int, c_int64, c_float, c_size_t = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
c_void_p, c_char_p = ctypes.c_void_p, ctypes.c_char_p

DTYPE_BF16 = 0
DTYPE_F32 = 1

STATUS_NAMES = {0: "ok", 1: "timeout", 2: "capacity", 3: "bad_index"}

# name -> (restype, argtypes); mirrors include/b200moe.h one for one.
SIGNATURES = {
    "b200moe_abi_version": (c_int, []),
    "b200moe_last_error": (c_char_p, []),
    "b200moe_tokens_per_block": (c_int, [c_int]),
    "b200moe_router_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "b200moe_router": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
         c_int, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_size_t, c_void_p, c_void_p],
    ),
    "b200moe_add_rmsnorm_router": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_float, c_int64, c_void_p, c_void_p, c_int64, c_int,
         c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p,
         c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "b200moe_add_rmsnorm_router_permute": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_float, c_int64, c_void_p, c_void_p, c_int64, c_int,
         c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p,
         c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "b200moe_router_sigmoid_grouped": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "b200moe_router_noalloc": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
         c_int, c_float, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "b200moe_router_from_logits": (
        c_int,
        [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p, c_void_p,
         c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "b200moe_permute": (
        c_int,
        [c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "b200moe_grouped_swiglu": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_int64, c_void_p, c_void_p],
    ),
    "b200moe_grouped_down": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_int64, c_void_p, c_void_p, c_void_p],
    ),
    "b200moe_grouped_swiglu_ex": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_int64, c_void_p, c_void_p],
    ),
    "b200moe_grouped_down_ex": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_int64, c_void_p, c_void_p, c_void_p],
    ),
    "b200moe_grouped_swiglu_f32": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int64,
         c_void_p],
    ),
    "b200moe_grouped_down_f32": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int64,
         c_void_p, c_void_p],
    ),
    "b200moe_combine": (
        c_int,
        [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
         c_int64, c_void_p, c_void_p, c_int64, c_void_p],
    ),
    "b200moe_add_rmsnorm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_int64, c_void_p, c_void_p,
         c_int64, c_void_p],
    ),
    "b200moe_gather_segments": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_void_p,
         c_void_p],
    ),
    "b200moe_ep_layout": (
        c_int, [c_int, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "b200moe_ep_alloc": (c_int, [c_size_t, c_void_p, c_void_p]),
    "b200moe_ep_open": (c_int, [c_void_p, c_void_p]),
    "b200moe_ep_close": (c_int, [c_void_p]),
    "b200moe_ep_free": (c_int, [c_void_p]),
    "b200moe_ep_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "b200moe_ep_collect": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "b200moe_ep_combine_send": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "b200moe_ep_wait_combine": (c_int, [c_void_p, c_void_p]),
    "b200moe_ep_permute_dispatch": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
         c_void_p, c_size_t, c_void_p]),
    "b200moe_ep_grouped_down_send": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p,
         c_void_p, c_void_p]),
    "b200moe_ep_grouped_swiglu_recv": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "b200moe_ep_grouped_down_send_recv": (
        c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "b200moe_ep_combine": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p,
         c_int64, c_void_p]),
}

EP_MAX_RANKS = 8
EP_HANDLE_BYTES = 64


class EpDesc(ctypes.Structure):
    """b200moe_ep_desc (include/b200moe.h)."""
    _fields_ = [
        ("peer", c_void_p * EP_MAX_RANKS),
        ("world_size", c_int),
        ("rank", c_int),
        ("slots_per_rank", c_int),
        ("row_bytes", c_int),
        ("cap_rows", c_int64),
        ("comb_rows", c_int64),
        ("counters", c_void_p),
        ("status", c_void_p),
        ("timeout_ns", ctypes.c_uint64),
    ]


class B200MoEError(RuntimeError):
    """A C-ABI call returned an error code."""


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise B200MoEError(
                    f"{_LIB_PATH} is not built; run `python -m easyinfra_b200.build` "
                    "(no CPU fallback exists for this path)")
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


# Optional callable(name, "start" | "end") invoked around every entry-point call (on the
# caller's thread, so it can record CUDA events on the launching stream); bench.py
# uses it for its per-op breakdown.
CALL_HOOK = {"fn": None}


def call(name: str, *args) -> None:
    """Invoke an entry point; raise B200MoEError with the library's message on failure."""
    lib = load()
    hook = CALL_HOOK["fn"]
    if hook is not None:
        hook(name, "start")
    rc = getattr(lib, name)(*args)
    if hook is not None:
        hook(name, "end")
    if rc != 0:
        msg = lib.b200moe_last_error().decode(errors="replace")
        raise B200MoEError(f"{name} failed ({rc}): {msg}")
