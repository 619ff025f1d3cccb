"""ctypes binding of libexl3b200.so (C ABI declared in include/exl3b200.h).

The library is built in-tree (``exl3xpu-mixedk_b200/csrc/build.py``).  There
is no fallback: if it is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libexl3b200.so")

RC_NAMES = {
    0: "OK", 1: "NO_DEVICE", 2: "ALLOC", 3: "BAD_DEVICE", 4: "DEVICE_ERROR",
    5: "TOO_MANY_BYTES", 6: "BAD_NSEQ", 7: "BAD_REQUEST", 8: "BAD_K",
    9: "NOT_SPD", 10: "NONFINITE", 11: "WORKSPACE",
}
CODE_IDS = {"exl3_mul1": 0, "exl3_3inst": 1, "exl3_mcg": 2}

_lib = None
_lock = threading.Lock()

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
F = ctypes.c_float
D = ctypes.c_double
I64 = ctypes.c_int64

# name -> (restype, argtypes); every function declared in include/exl3b200.h
SIGNATURES = {
    "exl3b_last_error": (ctypes.c_char_p, []),
    "exl3b_abi_version": (I, []),
    "exl3b_code_lut": (I, [I, P]),
    "exl3b_launch_count": (ctypes.c_longlong, []),
    "exl3b_profile_begin": (None, []),
    "exl3b_profile_end": (I, [I, P, P, P]),
    "exl3b_device_init": (I, [I]),
    "exl3b_set_wait_limit_ms": (I, [D]),
    "exl3b_viterbi_workspace_bytes": (SZ, [I, I]),
    "exl3b_viterbi": (I, [P, I, I, I, I, P, I, P, P, SZ, P]),
    "exl3b_tailbite_workspace_bytes": (SZ, [I, I]),
    "exl3b_tailbite": (I, [P, I, I, I, I, I, P, P, SZ, P]),
    "exl3b_tailbite_noalloc": (I, [P, I, I, I, I, I, P, P]),
    "xtq_vit_init": (I, []),
    "xtq_vit_run": (I, [P, I, ctypes.c_char_p, I, I, P]),
    "exl3b_incoherence_fwd": (I, [P, I, I, I, P, P, P, P, P]),
    "exl3b_incoherence_inv": (I, [P, I, I, P, P, P, P, P]),
    "exl3b_rotate_hessian": (I, [P, I, P, P, P]),
    "exl3b_channel_scale_workspace_bytes": (SZ, [I, I]),
    "exl3b_channel_scale_fwd": (I, [P, I, I, I, P, P, P, P, P, P, P, P, SZ, P]),
    "exl3b_channel_scale_store": (I, [P, P, P, P, P, I, I, P, P, P]),
    "exl3b_damp_hessian": (I, [P, I, F, P, P]),
    "exl3b_convert_f32_f64": (I, [P, P, SZ, P]),
    "exl3b_damp_hessian_f64": (I, [P, I, D, P]),
    "exl3b_transpose_scale": (I, [I, P, I, I, P, P, P, P, P, P]),
    "exl3b_rms_scale": (I, [P, I, D, F, P, P, P]),
    "exl3b_div_scalar": (I, [P, P, P, SZ, P]),
    "exl3b_block_ldl_workspace_bytes": (SZ, [I, I]),
    "exl3b_block_ldl": (I, [P, I, I, P, P, P, SZ, P]),
    "exl3b_u_to_gram_workspace_bytes": (SZ, [I]),
    "exl3b_u_to_gram": (I, [P, I, P, P, SZ, P]),
    "exl3b_ldlq_workspace_bytes": (SZ, [I, I, I, I]),
    "exl3b_ldlq_sweep": (I, [P, P, I, I, I, P, P, P, I, I, I, I, P, P, P, I, I,
                             P, SZ, P]),
    "exl3b_feedback_gemm_workspace_bytes": (SZ, [I, I, I]),
    "exl3b_feedback_gemm": (I, [I, I, I, P, I, P, I, P, I, P, SZ, P]),
    "exl3b_verify_trellis": (I, [P, I, I, I, I, P, I, P, I, P, P]),
    "exl3b_hadamard_axis": (I, [P, I, I, I, P, P]),
    "exl3b_pack_states": (I, [P, I, I, P, P]),
    "exl3b_unpack_states": (I, [P, I, I, P, P]),
    "exl3b_decode_trellis": (I, [P, I, I, I, I, P, P]),
}


class Exl3bError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} failed: rc={rc} ({RC_NAMES.get(rc, '?')}): {msg}")
        self.rc = rc


def lib():
    """The loaded library (raises if it is absent: no CPU fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python exl3xpu-mixedk_b200/csrc/build.py`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    return lib().exl3b_last_error().decode(errors="replace")


def check(fn: str, rc: int) -> None:
    if rc != 0:
        raise Exl3bError(fn, rc, last_error())


def call(name: str, *args) -> int:
    """Call an rc-returning entry point; raise Exl3bError on failure."""
    rc = getattr(lib(), name)(*args)
    check(name, rc)
    return rc
