"""ctypes binding of libprism_b200.so (declared in include/prism_b200.h).

The library is built in-tree by ``prism_test_b200.build``. There is no fallback:
if the shared library is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

PRISM_OK = 0
PRISM_E_INVALID = -1
PRISM_E_UNSUPPORTED = -2
PRISM_E_WORKSPACE = -3
PRISM_E_CUDA = -4
PRISM_E_DEVICE_STATUS = -5

DTYPE_BF16 = 0
DTYPE_FP16 = 1
KERNEL_SCORE = 0
KERNEL_SELECT = 1
KERNEL_MERGE = 2
MODE_EXACT = 0
MODE_BLOCKMAX = 1
MODE_EXACT_STREAM = 2
SPAN_CENTERED = 0
SPAN_FLOOR = 1
KERNEL_WEIGHT = 3
KERNEL_SCALE = 4
KERNEL_THRESHOLD = 5
KERNEL_ATTN = 6
KERNEL_UNROTATE = 7
RECALL_QK = 0
RECALL_QKV = 1
RECALL_QKV2 = 2
IPC_HANDLE_BYTES = 64
PEER_HEADER_BYTES = 512
PEER_MAX_RANKS = 16

# Every function the header declares: name -> (restype, argtypes)
_c_i64 = ctypes.c_int64
_c_i32 = ctypes.c_int32
_vp = ctypes.c_void_p
SIGNATURES = {
    "prism_einsum_topk": (ctypes.c_int, [
        _vp, _vp, _vp, ctypes.c_int,
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64), _c_i64,
        _c_i64, _c_i32, _c_i32, _c_i64,
        _vp, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_einsum_topk_weighted": (ctypes.c_int, [
        _vp, _vp, _vp, _vp, ctypes.c_int,
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64),
        _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i64,
        _vp, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_einsum_topk_weighted_workspace_size": (ctypes.c_size_t, [
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32,
    ]),
    "prism_einsum_topk_rope_workspace_size": (ctypes.c_size_t, [
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32,
    ]),
    "prism_einsum_topk_workspace_size": (ctypes.c_size_t, [
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32,
    ]),
    "prism_sparse_attention": (ctypes.c_int, [
        _vp, _vp, _vp, _vp, _c_i64, _vp, _vp, _c_i32, ctypes.c_float, ctypes.c_int,
        _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64),
        _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_sparse_attention_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "prism_topk_merge": (ctypes.c_int, [
        _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i32, _vp, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_topk_merge_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "prism_topk_merge_runs": (ctypes.c_int, [
        _vp, _c_i32, _c_i64, _c_i64, _c_i32, _vp, _vp, _vp,
    ]),
    "prism_topk_merge_noalloc": (ctypes.c_int, [
        _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i32, _vp, _vp, _vp,
    ]),
    "prism_post_select": (ctypes.c_int, [
        _vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _vp, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_post_select_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i32]),
    "prism_peer_buffer_bytes": (ctypes.c_size_t, [_c_i64, _c_i32]),
    "prism_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "prism_peer_open": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "prism_peer_close": (ctypes.c_int, [_vp]),
    "prism_peer_free": (ctypes.c_int, [_vp]),
    "prism_peer_publish": (ctypes.c_int, [ctypes.POINTER(_vp), _c_i32, _c_i32, _vp]),
    "prism_peer_wait_acks": (ctypes.c_int, [ctypes.POINTER(_vp), _c_i32, _c_i32, _c_i64, _vp]),
    "prism_peer_merge": (ctypes.c_int, [
        ctypes.POINTER(_vp), _c_i32, _c_i32, _c_i64, _c_i32, _c_i32, _c_i64, _vp, _vp, _vp,
    ]),
    "prism_peer_read_timings": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint64), _c_i32, _vp]),
    "prism_sharded_topk": (ctypes.c_int, [
        _vp, _vp, _vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64), _c_i64, _c_i32,
        ctypes.POINTER(_vp), _c_i32, _c_i32, _c_i32, _c_i64, _vp, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
    "prism_read_status": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), _vp]),
    "prism_profile_start": (ctypes.c_int, [_c_i32]),
    "prism_profile_stop": (ctypes.c_int, []),
    "prism_profile_read": (ctypes.c_int, [_c_i32, ctypes.POINTER(_c_i64), ctypes.POINTER(ctypes.c_double)]),
    "prism_launch_count": (_c_i64, []),
    "prism_last_error": (ctypes.c_char_p, []),
    "prism_abi_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


class PrismLibraryError(RuntimeError):
    """The native library is missing, or a call into it failed."""


def lib_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise PrismLibraryError(
                f"{LIB_PATH.name} is not built; run `python -m prism_test_b200.build`"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.prism_abi_version() != 1:
            raise PrismLibraryError("libprism_b200.so ABI version mismatch")
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().prism_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Turn a PRISM_E_* code into a Python exception.

    Argument errors become AssertionError, as the reference launcher's
    ``assert`` statements raise (eval_harness/kernels/einsum_topk.py:182-195);
    everything else becomes PrismLibraryError (a RuntimeError).
    """
    if rc == PRISM_OK:
        return
    msg = f"{what}: {last_error()} (code {rc})"
    if rc in (PRISM_E_INVALID, PRISM_E_UNSUPPORTED):
        raise AssertionError(msg)
    raise PrismLibraryError(msg)


def i64_array(vals):
    arr = (_c_i64 * len(vals))(*[int(v) for v in vals])
    return arr
