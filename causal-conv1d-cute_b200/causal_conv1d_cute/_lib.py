"""Load libcc1d.so, the sm_100a kernel library, and describe its C ABI to ctypes.

The library sits next to this file (build it with ``python build.py`` in the parent directory).
There is no fallback: if it is missing or does not load, every entry point raises.
"""

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("CC1D_LIBRARY", Path(__file__).with_name("libcc1d.so")))

BF16, F16, F32 = 0, 1, 2
DTYPE_CODES = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}

DEV_BAD_SLOT, DEV_BAD_QSL, DEV_BAD_INTER_SLOT = 1, 2, 4

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32

# Argument lists, in the order of include/cc1d.h.
SIGNATURES = {
    "cc1d_fwd": [_p, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64,
                 _i64, _i64, _i64, _i32, _i32, _i32, _p],
    "cc1d_fwd_states": [_p, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64,
                        _p, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                        _i64, _i64, _i64, _i32, _i32, _i32, _p],
    "cc1d_update": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64,
                    _p, _i64, _p, _i64, _i64, _i64, _p, _i32, _p, _i64, _i64, _i64, _i64, _i64,
                    _p, _i64, _i64, _i32, _i32, _i32, _i32, _p, _p],
    "cc1d_update_ring": [_p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _i64,
                         _p, _i64, _i64, _p, _p, _i32, _i64, _i64, _i32, _i32, _i32, _p, _p],
    "cc1d_to_ring": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i32, _i32, _p],
    "cc1d_from_ring": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i32, _i32, _p],
    "cc1d_varlen": [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _p, _i64, _i64,
                    _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i64, _i32, _i32, _i32, _p, _p],
    "cc1d_update_unpack": [_p, _i64, _p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _i32,
                           _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _p],
    "cc1d_copy": [_p, _p, _i64, _p],
}

EXPORTS = ("cc1d_abi_version", "cc1d_status_string", "cc1d_last_error", *SIGNATURES)

_lib = None
_load_error = None


class LibraryError(RuntimeError):
    """libcc1d.so is missing, failed to load, or a call returned an error status."""


def load():
    """Return the loaded library, loading it on first use; raise LibraryError if unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise LibraryError(_load_error)
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:
        _load_error = (
            f"causal_conv1d_cute: cannot load the CUDA kernel library {LIB_PATH} ({e}); "
            "build it with `python build.py` (there is no CPU fallback)"
        )
        raise LibraryError(_load_error) from None
    lib.cc1d_abi_version.restype = ctypes.c_int32
    lib.cc1d_abi_version.argtypes = []
    lib.cc1d_status_string.restype = ctypes.c_char_p
    lib.cc1d_status_string.argtypes = [ctypes.c_int32]
    lib.cc1d_last_error.restype = ctypes.c_char_p
    lib.cc1d_last_error.argtypes = []
    for name, args in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = ctypes.c_int32
        f.argtypes = args
    if lib.cc1d_abi_version() != 1:
        _load_error = f"{LIB_PATH} has ABI {lib.cc1d_abi_version()}, expected 1"
        raise LibraryError(_load_error)
    _lib = lib
    return lib


def check(status):
    """Raise LibraryError for a non-zero status returned by an entry point."""
    if status != 0:
        lib = load()
        what = lib.cc1d_status_string(status).decode()
        detail = lib.cc1d_last_error().decode()
        raise LibraryError(f"causal_conv1d_cute kernel call failed: {what}: {detail}")


def dtype_code(dtype):
    code = DTYPE_CODES.get(dtype)
    if code is None:
        raise NotImplementedError(f"dtype {dtype} is not bf16, fp16 or fp32")
    return code
