"""ctypes binding of libpaged_decode_b200.so (include/paged_decode_b200.h).

There is no fallback: if the library is missing or fails to load, every op
raises. Build it with ``python <package>/build.py`` (``__graft_entry__.build()``
does this too).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_ptr = ctypes.c_void_p
_c_size = ctypes.c_size_t

# (name, restype, argtypes) for every entry point of the C header.
SIGNATURES = {
    "pdb_last_error": (ctypes.c_char_p, []),
    "pdb_version": (ctypes.c_char_p, []),
    "pdb_paged_attention_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int]),
    "pdb_paged_attention": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                     _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                     _c_i64, _c_i64, _c_int, _c_ptr, _c_size, _c_ptr]),
    "pdb_paged_attention_impl": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                          _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                          _c_i64, _c_i64, _c_int, _c_ptr, _c_size, _c_ptr, _c_int]),
    "pdb_paged_attention_noalloc": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                             _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                             _c_i64, _c_i64, _c_i64, _c_int, _c_ptr]),
    "pdb_rope_kv_write": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                   _c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_i64,
                                   _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                   _c_i64, _c_int, _c_ptr, _c_size, _c_ptr]),
    "pdb_rope_kv_write_workspace_size": (_c_size, [_c_i64, _c_i64, _c_int]),
    "pdb_decode_attention": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                      _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                      _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_ptr,
                                      _c_size, _c_ptr]),
    "pdb_decode_attention_ex": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                         _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_ptr,
                                         _c_size, _c_ptr, ctypes.c_uint]),
    "pdb_decode_attention_supported": (_c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                                _c_int]),
    "pdb_prefill_attention": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64,
                                       _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                       _c_int, _c_ptr]),
    "pdb_prefill_attention_impl": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                            _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                            _c_i64, _c_i64, _c_int, _c_ptr, _c_int]),
    "pdb_rope_kv_write_decode": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                          _c_ptr, _c_i64, _c_ptr, _c_int, _c_ptr, _c_i64,
                                          _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int,
                                          _c_ptr]),
    "pdb_read_device_errors": (_c_int, [ctypes.POINTER(ctypes.c_uint32), _c_int]),
    "pdb_debug_partition": (_c_i64, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr]),
    "pdb_debug_dyn_partition": (_c_i64, [_c_i64, _c_i64, _c_ptr, _c_i64]),
    "pdb_fast_grid_size": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64, _c_int]),
}

DTYPE_FLOAT32 = 0
DTYPE_FLOAT16 = 1
IMPL_AUTO, IMPL_FAST, IMPL_GENERIC, IMPL_SIMT, IMPL_MMA, IMPL_TMA_STATIC = 0, 1, 2, 3, 4, 5
PREFILL_AUTO, PREFILL_TCGEN05, PREFILL_MMA = 0, 1, 2
DECODE_STABLE_METADATA = 0x1
DECODE_STABLE_POOLS = 0x2
STATUS_NAMES = {0: "ok", 1: "invalid argument", 2: "workspace", 3: "cuda"}

_lock = threading.Lock()
_lib = None


def lib_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (no CPU or torch fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run the package's build.py (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().pdb_last_error().decode()


def check(status: int, what: str) -> None:
    """Raise RuntimeError (the reference's TORCH_CHECK type) on a failed call."""
    if status != 0:
        raise RuntimeError(f"{last_error()}")
