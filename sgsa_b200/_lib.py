"""ctypes binding of libsgsa_b200.so (the C ABI declared in include/sgsa_b200.h).

There is no fallback: if the library is missing or the device is not an
sm_100 part, every op raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# SGSA_CHECK=1 selects the bounds-checked debug build (same C ABI; see sgsa_check_status)
CHECK_BUILD = os.environ.get("SGSA_CHECK", "0") == "1"
LIB_PATH = os.path.join(_HERE, "_lib", "libsgsa_b200_check.so" if CHECK_BUILD else "libsgsa_b200.so")

SGSA_OK = 0
DTYPE_F32, DTYPE_BF16 = 0, 1
FLAG_HAS_SPARSE, FLAG_HAS_INIT, FLAG_STORE_FINAL, FLAG_OUT_F32 = 1, 2, 4, 8
FLAG_TRANSITION, FLAG_REUSE_PREP = 16, 32

_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/sgsa_b200.h
SIGNATURES = {
    "sgsa_status_string": (ctypes.c_char_p, [_i]),
    "sgsa_last_error": (ctypes.c_char_p, []),
    "sgsa_version": (_i, []),
    "sgsa_kernel_launches": (ctypes.c_ulonglong, []),
    "sgsa_watchdog_status": (_i, [_vp]),
    "sgsa_watchdog_selftest": (_i, [ctypes.c_uint, _vp]),
    "sgsa_check_status": (_i, [_vp, _i]),
    "sgsa_chunk_fwd_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "sgsa_chunk_fwd": (_i, [_vp] * 11 + [_i] * 7 + [_vp, _sz, _vp]),
    "sgsa_chunk_fwd_noalloc": (_i, [_vp] * 11 + [_i] * 7 + [_vp]),
    "sgsa_indexer_topk": (_i, [_vp, _vp, _vp] + [_i] * 6 + [_vp]),
    "sgsa_indexer_topk_scores": (_i, [_vp] * 4 + [_i] * 5 + [_vp]),
    "sgsa_indexer_stats": (_i, [_vp, _i]),
    "sgsa_topk_select": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "sgsa_sparse_attn_mix": (_i, [_vp] * 7 + [_i] * 6 + [ctypes.c_float, _i, _i, _vp]),
    "sgsa_indexer_thresholds": (_i, [_vp] * 5 + [_i] * 6 + [_vp]),
    "sgsa_sparse_attn_thresholds": (_i, [_vp] * 7 + [_i] + [_vp] * 3 + [_i] * 6 +
                                    [ctypes.c_float, _i, _i, _vp, _vp]),
    "sgsa_sparse_attn_index_scores": (_i, [_vp] * 8 + [_i] * 3 + [_vp]),
    "sgsa_sparse_retrieve": (_i, [_vp] * 6 + [_i] * 6 + [ctypes.c_float, _i, _vp]),
    "sgsa_rmsnorm": (_i, [_vp] * 3 + [ctypes.c_longlong, _i, ctypes.c_float, _i, _vp]),
    "sgsa_swiglu": (_i, [_vp] * 2 + [ctypes.c_longlong, _i, _i, _vp]),
    "sgsa_rope_qkv": (_i, [_vp] * 5 + [_i] * 6 + [_vp]),
    "sgsa_layer_proj": (_i, [_vp, _i] + [_vp] * 8 + [ctypes.c_longlong] + [_i] * 4 + [_vp]),
    "sgsa_embed": (_i, [_vp] * 3 + [ctypes.c_longlong, _i, _i, _i, _vp]),
    "sgsa_gate_mix": (_i, [_vp] * 4 + [ctypes.c_longlong, _i, _i, _i, _vp]),
    "sgsa_recurrent_fwd": (_i, [_vp] * 11 + [_i] * 6 + [_vp]),
    "sgsa_decode_append": (_i, [_vp] * 6 + [_i] * 7 + [_vp]),
    "sgsa_decode_topk": (_i, [_vp] * 3 + [_i] * 7 + [_vp]),
    "sgsa_decode_attn_mix": (_i, [_vp] * 7 + [_i] * 5 + [ctypes.c_float, _i, _i, _vp]),
    "sgsa_layer_fwd_workspace_size": (_sz, [_i] * 8),
    "sgsa_layer_fwd": (_i, [_vp] * 12 + [_i] * 9 + [_vp, _sz, _vp]),
}

_lib = None


class SGSAError(RuntimeError):
    pass


def load():
    """Load the library once (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m sgsa_b200.build"
                + (" --check" if CHECK_BUILD else "") + "` (there is no CPU or Python fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


# SGSA_WATCHDOG_CHECK=1: after every op, synchronise its stream and raise if a
# bounded wait inside a tensor-core kernel gave up (its results are then invalid).
# Off by default: the check costs a stream synchronisation per op.
WATCHDOG_CHECK = os.environ.get("SGSA_WATCHDOG_CHECK", "0") == "1"


def check_watchdog(stream: int, what: str) -> None:
    """Raise SGSAError if the device watchdog recorded a wait that gave up."""
    w = load().sgsa_watchdog_status(stream)
    if w != 0:
        raise SGSAError(f"{what}: device watchdog 0x{w & 0xffffffff:x} (a bounded wait inside a "
                        "kernel gave up; its outputs are invalid)")


def check(status: int, what: str, tensor=None) -> None:
    """Raise on a non-OK status (ValueError for argument errors, SGSAError for device
    errors); with SGSA_WATCHDOG_CHECK=1 also check the watchdog of `tensor`'s stream."""
    if status == SGSA_OK:
        if WATCHDOG_CHECK and tensor is not None:
            import torch
            check_watchdog(torch.cuda.current_stream(tensor.device).cuda_stream, what)
        return
    lib = load()
    msg = lib.sgsa_status_string(status).decode()
    extra = lib.sgsa_last_error().decode()
    text = f"{what}: {msg}" + (f" ({extra})" if extra else "")
    if status in (-1, -2, -3, -4, -6):
        raise ValueError(text)
    raise SGSAError(text)
