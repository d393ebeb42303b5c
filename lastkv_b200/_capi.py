"""ctypes binding of ``liblastkv_b200.so`` (the C ABI in include/lastkv_b200.h).

There is no fallback: if the library is missing or fails to load, every op
raises.  ``declared_symbols()`` parses the public header so tests can check
that the library exports exactly what the header declares.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

from .contract import RMarinBackendContractError

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "liblastkv_b200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "lastkv_b200.h")

_lib = None
_lock = threading.Lock()

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float
SZ = ctypes.c_size_t

_SIGNATURES = {
    "lkv_status_string": (ctypes.c_char_p, [I32]),
    "lkv_abi_version": (I32, []),
    "lkv_check_device": (I32, [I32]),
    "lkv_read_error_word": (I32, [P, P, P]),
    "lkv_clear_error_word": (I32, [P, P]),
    "lkv_decode_workspace_bytes": (SZ, [I32, I32, I32, I32]),
    "lkv_decode_paged": (I32, [P, I64, P, P, I64, P, I64, P, P, I64, P, P, P, P,
                               I32, I32, I32, I32, I32, F32, P, SZ, I32, P]),
    "lkv_decode_plan": (I32, [I32, I32, I32, I32, I32, SZ, I32, P, P]),
    "lkv_decode_paged_noalloc": (I32, [P, I64, P, P, I64, P, I64, P, P, I64, P, P,
                                       I32, I32, I32, I32, I32, F32, P, P]),
    "lkv_merge_partials": (I32, [P, P, I32, I64, I32, I32, I64, I64, P, P, P, P]),
    "lkv_rope_norm_append": (I32, [P, I64, P, I64, P, I64, P, P, I64, I64, P, P, F32, P, P, I64,
                                   P, P, P, I64, P, P, P, I64, I32, I32, I32, I32, I32, P, P]),
    "lkv_rope_norm_append_commit": (I32, [P, I64, P, I64, P, I64, P, P, I64, I64, P, P, F32, P, P, I64,
                                          P, P, P, I64, P, P, P, I64, I32, I32, I32, I32, I32,
                                          P, P, I64, P, P, I64, P, I32, I32, I32, P, I32, P, P]),
    "lkv_gather_blend": (I32, [P, P, I64, P, P, P, P, P, I32, I32, I32, P, P]),
    "lkv_blend_chunk": (I32, [P, P, I64, P, P, I64, P, I32, I32, I32, I32, I32, P, P]),
    "lkv_blend_chunk_f32": (I32, [P, P, I64, P, P, I64, P, I32, I32, I32, I32, I32, P, P]),
    "lkv_attention_paged_f32": (I32, [P, I64, P, P, I64, P, I64, P, P, P, I64, P, P,
                                      I32, I32, I32, I32, I32, I32, I32, F32, P, P]),
    "lkv_build_layer_block_tables": (I32, [P, I64, P, P, I32, I32, I32, P, P]),
    "lkv_rmsnorm": (I32, [P, I64, P, I64, P, I64, P, P, I64, I32, I32, F32, P]),
    "lkv_silu_mul": (I32, [P, I64, P, I64, I64, I32, P]),
    "lkv_argmax_rows": (I32, [P, I64, I32, I32, P, P]),
    "lkv_decode_gemm_plan": (I32, [I64, I64, I32, P, P, P]),
    "lkv_cp_combine_sizes": (I32, [I64, I32, I32, P, P]),
    "lkv_cp_combine": (I32, [P, P, I32, I32, P, I64, I32, I32, P, P, I64, P, P]),
    "lkv_decode_cp_state_words": (I32, [I32, I32, P]),
    "lkv_decode_paged_cp": (I32, [P, I64, P, P, I64, P, I64, P, P, I64, P, I32, I32, I32, I32, I32, F32, P, SZ,
                                  P, I32, I32, P, P, I32, P]),
    "lkv_decode_gemm": (I32, [P, I64, P, I64, P, I64, I32, I64, I64, I32, P, P, P]),
    "lkv_prefill_paged": (I32, [P, I64, P, P, I64, P, I64, P, P, P, I64, P, P,
                                I32, I32, I32, I32, I32, I32, I32, I32, F32, P, P]),
    "lkv_prefill_paged_split": (I32, [P, I64, P, P, I64, P, I64, P, P, P, I64, P, P,
                                      I32, I32, I32, I32, I32, I32, I32, F32, I32, P, P, P, P]),
    "lkv_prefill_split_plan": (I32, [I32, I32, I32, I32, I32, I32, I32, P]),
}


def declared_symbols() -> list[str]:
    """Names of every ``lkv_*`` function declared in the public header."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lkv_[a-z0-9_]+)\s*\(", text)))


def load(path: str = LIB_PATH):
    """Load the library (once) and bind every declared signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RMarinBackendContractError(
                f"liblastkv_b200.so not built at {path}; run `python -m lastkv_b200.build` "
                "(there is no CPU or library fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            if not hasattr(lib, name):
                continue
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else load()


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().lkv_status_string(status).decode()
        raise RMarinBackendContractError(f"{what} failed: {msg} (status {status})")
