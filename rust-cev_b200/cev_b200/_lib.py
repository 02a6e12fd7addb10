"""ctypes binding of the C ABI in ``include/cevk.h`` (``libcevk.so``).

The library is built in-tree by ``rust-cev_b200/build.py``.  Loading fails
loudly if it is missing: there is no CPU fallback anywhere in the product.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcevk.so")

OK, E_SHAPE, E_RANGE, E_CUDA, E_TIMEOUT, E_UNSUPPORTED = 0, -1, -2, -3, -5, -6
BF16, F32 = 1, 2

P, I32, I64, F, D, SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_double, C.c_size_t


class Segment(C.Structure):
    """``cevk_segment``."""
    _fields_ = [("q_start", I32), ("q_len", I32), ("prefix_off", I32), ("prefix_len", I32),
                ("self_off", I32), ("tile_start", I32), ("flags", I32)]


SEG_BIDIRECTIONAL = 1  # CEVK_SEG_BIDIRECTIONAL


# name -> (restype, argtypes), exactly the declarations of include/cevk.h
SIGNATURES = {
    "cevk_last_error": (C.c_char_p, []),
    "cevk_version": (C.c_int, []),
    "cevk_device_status": (C.c_int, []),
    "cevk_selftest_wait_timeout": (C.c_int, [I64, P]),
    "cevk_attn_schedule": (C.c_int, [P, I32, I32, I32, I32, I32, I32, I32, P]),
    "cevk_attn_packed_prefill": (C.c_int, [P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32, P, I32, I32, F, I32, P]),
    "cevk_attn_split_plan": (C.c_int, [P, I32, I32, I32, I32, I32, I32, P, P]),
    "cevk_ipc_alloc": (C.c_int, [I64, P]),
    "cevk_ipc_free": (C.c_int, [P]),
    "cevk_ipc_handle": (C.c_int, [P, P]),
    "cevk_ipc_open": (C.c_int, [P, P]),
    "cevk_ipc_close": (C.c_int, [P]),
    "cevk_attn_packed_prefill_gather": (C.c_int, [P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32, I32, P, I32, I32,
                                                  F, I32, P, I64, P]),
    "cevk_gather_signal": (C.c_int, [P, I32, I32, I32, P]),
    "cevk_gather_wait": (C.c_int, [P, I32, I32, I64, P]),
    "cevk_gather_signal_dev": (C.c_int, [P, I32, I32, P, P]),
    "cevk_gather_wait_dev": (C.c_int, [P, I32, P, I64, P]),
    "cevk_rows_to_peers": (C.c_int, [P, P, I32, I64, P]),
    "cevk_gather_sync_dev": (C.c_int, [P, I32, I32, P, P, I64, P]),
    "cevk_rows_gather_dev": (C.c_int, [P, P, I32, I64, P, I32, I32, P, P, I64, P, P]),
    "cevk_attn_split_workspace_size": (I64, [I32, I32, I32, I32]),
    "cevk_attn_packed_prefill_split": (C.c_int, [P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32, P, I32, I32, F, I32,
                                                 P, I64, I32, P]),
    "cevk_qk_norm_rope": (C.c_int, [P, I32, I32, I32, I32, P, P, F, I32, P, D, I32, P, P, P, I32, P, I32, I32, I32, I32, I32, P]),
    "cevk_rms_norm": (C.c_int, [P, P, P, P, P, I32, I32, F, I32, I32, P]),
    "cevk_swiglu": (C.c_int, [P, P, I32, I32, I32, P]),
    "cevk_debias": (C.c_int, [P, P, I32, P, P, P, I32, P, P, I32, P]),
    "cevk_embed": (C.c_int, [P, P, P, I32, I32, I32, I32, P]),
    "cevk_sigmoid_gate": (C.c_int, [P, P, I32, I32, P, I32, I32, I32, I32, P]),
    "cevk_readout": (C.c_int, [P, P, I32, P, F, I32, P, I32, P, P, I32, I32, P]),
    "cevk_gdn_conv": (C.c_int, [P, I32, P, P, I64, P, P, I32, I32, I32, I32, I32, P]),
    "cevk_gdn_workspace_size": (SZ, [I32, I32, I32, I32, I32]),
    "cevk_gdn_chunk_prefill": (C.c_int, [P, I32, P, I32, P, I32, P, P, P, F, P, I64, P, P, I32, I32, I32, I32, I32, I32, P, SZ, I32, P]),
    "cevk_gdn_chunk_prefill_noalloc": (C.c_int, [P, I32, P, I32, P, I32, P, P, P, F, P, I64, P, P, I32, I32, I32, I32, I32, I32, I32, P]),
    "cevk_short_conv": (C.c_int, [P, P, P, P, I64, P, P, I32, I32, I32, I32, I32, P]),
}

_lib = None


class CevkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"cevk error {code}: {msg}")
        self.code = code


def lib() -> C.CDLL:
    """The loaded library with argument types set (loaded once)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python rust-cev_b200/build.py`")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise CevkError(rc, lib().cevk_last_error().decode())
