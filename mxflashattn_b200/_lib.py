"""ctypes binding of libmxfa_b200.so (the C ABI declared in include/mxfa_b200.h).

This replaces the reference's pybind modules (``csrc_native/m1_binding.cpp``,
``csrc/mxmac/attention_forward.cpp``): the library takes raw device pointers
and sizes, and this module converts torch tensors to those.  Loading fails
loudly -- there is no silent CPU path behind it.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmxfa_b200.so")

MXFA_OK = 0
MXFA_ERR_UNSUPPORTED = -1
MXFA_ERR_INVALID = -2
MXFA_ERR_CUDA = -3

FLAG_PAGE_OUT_OF_RANGE = 0x1
FLAG_TABLE_TOO_NARROW = 0x2
FLAG_WAIT_TIMEOUT = 0x4
FLAG_DENSE_OVERFLOW = 0x8
FLAG_BAD_ORDER = 0x10

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "mxfa_abi_version": (_i, []),
    "mxfa_last_error": (ctypes.c_char_p, []),
    "mxfa_is_available": (_i, []),
    "mxfa_read_error_flags": (_i, [ctypes.POINTER(ctypes.c_uint)]),
    "mxfa_paged_decode_split_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "mxfa_split_workspace_bytes": (_sz, [_i, _i, _i]),
    "mxfa_kvcache_plan": (_i, [_i, _i, _i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "mxfa_kvcache_attention_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _f, _vp]),
    "mxfa_split_counter_bytes": (_sz, [_i, _i, _i, _i]),
    "mxfa_kvcache_attention_counted_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _f, _vp]),
    "mxfa_kvcache_attention_fp8_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _f, _f, _f, _vp]),
    "mxfa_kvcache_length_order_launch": (_i, [_vp, _i, _vp, _vp]),
    "mxfa_kvcache_attention_ordered_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _i, _f, _i, _f, _f, _vp]),
    "mxfa_kvcache_append_attention_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _i, _i, _f, _vp]),
    "mxfa_cp_buffer_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "mxfa_peer_alloc": (_i, [_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "mxfa_peer_free": (_i, [_vp]),
    "mxfa_peer_export": (_i, [_vp, _vp]),
    "mxfa_peer_import": (_i, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "mxfa_peer_close": (_i, [_vp]),
    "mxfa_cp_decode_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _f, _vp]),
    "mxfa_cp_merge_launch": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "mxfa_cp_last_merged_in_place": (_i, []),
    "mxfa_cp_attention_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _i, _i, _f, _vp]),
    "mxfa_kvcache_attention_noalloc_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
    "mxfa_kvcache_attention_packed_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
    "mxfa_split_combine_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "mxfa_lse_merge_launch": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "mxfa_kv_append_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "mxfa_seqlens_add_launch": (_i, [_vp, _i, _i, _i, _vp]),
    "mxfa_varlen_fwd_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
    "mxfa_varlen_fwd_exact_launch": (
        _i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
}

_lock = threading.Lock()
_lib = None


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing, unloadable, or returned an error status."""


def load(path: str | None = None):
    """Load (once) and return the ctypes library with typed signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = path or LIB_PATH
        if not os.path.exists(target):
            raise NativeLibraryError(
                f"{target} is not built; run `python -m mxflashattn_b200.build` (nvcc, sm_100a)")
        try:
            lib = ctypes.CDLL(target)
        except OSError as exc:
            raise NativeLibraryError(f"cannot load {target}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    return load().mxfa_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != MXFA_OK:
        kind = {MXFA_ERR_UNSUPPORTED: "unsupported configuration", MXFA_ERR_INVALID: "invalid argument",
                MXFA_ERR_CUDA: "CUDA error"}.get(rc, f"status {rc}")
        raise NativeLibraryError(f"{what}: {kind}: {last_error()}")


def read_error_flags() -> int:
    """Device error flags since the last read (synchronises; diagnostics only)."""
    flags = ctypes.c_uint(0)
    check(load().mxfa_read_error_flags(ctypes.byref(flags)), "mxfa_read_error_flags")
    return int(flags.value)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
