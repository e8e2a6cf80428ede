"""ctypes binding of liblxb.so (the C ABI in include/lxb.h). There is no fallback: if the
library is missing or fails to load, every entry point raises."""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from . import build as _build

P = ctypes.c_void_p
I = ctypes.c_int

_lib = None


class LxbError(RuntimeError):
    pass


# device status bits (include/lxb.h): the errors; LXB_S_HELPER (4) is informational
S_TOKEN, S_STAGE, S_HELPER, S_SYNC = 1, 2, 4, 8
S_ERRORS = S_TOKEN | S_STAGE


class Caps(ctypes.Structure):
    _fields_ = [("device", I), ("cc_major", I), ("cc_minor", I), ("sm_count", I),
                ("max_smem_optin", I), ("cluster_launch", I), ("max_clusters", I)]


class Typing(ctypes.Structure):
    """lxb_typing (include/lxb.h)."""
    _fields_ = [("keys", P), ("n_keys", P), ("max_keys", ctypes.c_int32),
                ("key0_base", ctypes.c_int32), ("key_base", ctypes.c_int32),
                ("rx_slots", ctypes.c_int32), ("tclass", P), ("n_class", ctypes.c_int32),
                ("tstate", P)]


class Err(ctypes.Structure):
    _fields_ = [("status", ctypes.c_uint32), ("first_stream", ctypes.c_int32),
                ("first_step", ctypes.c_int32)]


SIGNATURES = {
    "lxb_abi_version": (I, []),
    "lxb_query": (I, [I, P]),
    "lxb_plan_create": (I, [P, ctypes.c_size_t, I, P]),
    "lxb_decode": (I, [P, P, P, I, P, P, I, P, I, I, P, P, P]),
    "lxb_scratch_bytes": (ctypes.c_size_t, [P, I]),
    "lxb_decode_noalloc": (I, [P, P, P, I, P, I, P, I, I, P, P, P]),
    "lxb_status": (I, [P, P]),
    "lxb_plan_set_profile": (I, [P, P]),
    "lxb_plan_set_head_helpers": (I, [P, I]),
    "lxb_plan_set_typing": (I, [P, P]),
    "lxb_profile_sections": (I, []),
    "lxb_cluster_sync_cycles": (I, [I, I, P]),
    "lxb_plan_staging": (I, [P, P, P, P]),
    "lxb_status_clear": (I, [P]),
    "lxb_plan_bytes": (ctypes.c_size_t, [P]),
    "lxb_plan_max_clusters": (I, [P]),
    "lxb_plan_destroy": (None, [P]),
    "lxb_error_string": (ctypes.c_char_p, [I]),
    "lxb_prefill_check_image": (I, [P, ctypes.c_size_t]),
    "lxb_prefill_plan_create": (I, [P, ctypes.c_size_t, P]),
    "lxb_prefill_scratch_bytes": (ctypes.c_size_t, [P, I]),
    "lxb_prefill": (I, [P, P, P, P, I, P, P, P, P]),
    "lxb_prefill_layers": (I, [P, P, P, P, I, P, P]),
    "lxb_prefill_head": (I, [P, P, I, P, P, P]),
    "lxb_prefill_status": (I, [P, P]),
    "lxb_prefill_status_clear": (I, [P]),
    "lxb_prefill_plan_destroy": (None, [P]),
    "lxb_prefill_set_timing": (I, [P, I]),
    "lxb_prefill_timing": (I, [P, P, P, I]),
    "lxb_prefill_stage_name": (ctypes.c_char_p, [I]),
    "lxb_text_plan_create": (I, [P, I, P, I, P, I, P, P, I, ctypes.c_float, I, P]),
    "lxb_text_scratch_bytes": (ctypes.c_size_t, [P]),
    "lxb_text_decode": (I, [P, P, I, I, I, P, P, P, ctypes.c_size_t, P]),
    "lxb_text_status": (I, [P, P]),
    "lxb_text_status_clear": (I, [P]),
    "lxb_text_grid": (I, [P]),
    "lxb_text_set_profile": (I, [P, P]),
    "lxb_text_plan_destroy": (None, [P]),
}


def lib():
    """The loaded library (`python -m linuxformer_b200.build` builds it; a missing one raises)."""
    global _lib
    if _lib is None:
        # LXB_LIBRARY: another build of liblxb.so to load instead (A/B timing of two builds)
        path = Path(os.environ["LXB_LIBRARY"]) if os.environ.get("LXB_LIBRARY") else _build.LIB
        if not path.exists():
            raise LxbError(f"{path} is not built: run `python -m linuxformer_b200.build`")
        L = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        if L.lxb_abi_version() != 1:
            raise LxbError("liblxb.so has another ABI version than this binding")
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc:
        msg = lib().lxb_error_string(rc).decode()
        raise LxbError(f"{what}: error {rc} ({msg})")
