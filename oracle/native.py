"""Build and load the C port of the oracle (oracle/cc1d_oracle.c) - TEST INFRASTRUCTURE ONLY.

It is the multithreaded CPU baseline that bench.py times (cpu_baseline and the --impl reference
arm) and a second checker in the tests. The shared object goes to oracle/_build/ (git-ignored);
build() compiles it with the system gcc and OpenMP.
"""

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "cc1d_oracle.c"
LIB = HERE / "_build" / "libcc1d_oracle.so"

_lib = None


def build(force=False):
    LIB.parent.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        # Portable x86-64 code: the object is built once and may run on another host.
        cmd = ["gcc", "-O3", "-fopenmp", "-fPIC", "-shared", str(SRC), "-o", str(LIB), "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        lib.oracle_threads.restype = i32
        lib.oracle_set_threads.argtypes = [i32]
        lib.oracle_fwd_cl_bf16.argtypes = [p, p, p, p, i64, i64, i64, i32, i32]
        lib.oracle_varlen_bf16.argtypes = [p, p, p, p, p, i64, i64, i32, p, p, p, i32, i32]
        lib.oracle_update_bf16.argtypes = [p, p, p, p, p, p, i64, i64, i32, i32, i32]
        _lib = lib
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def threads():
    return load().oracle_threads()


def set_threads(n):
    load().oracle_set_threads(int(n))


def fwd_cl_bf16(x, w, bias, silu):
    """x (B, L, D) uint16 bf16 bits, w (D, W), bias (D,) or None -> out (B, L, D) uint16."""
    B, L, D = x.shape
    out = np.empty_like(x)
    load().oracle_fwd_cl_bf16(_p(x), _p(w), _p(bias), _p(out), B, L, D, w.shape[1], int(silu))
    return out


def varlen_bf16(x, w, bias, qsl, cidx, hinit, states, pad, silu):
    """x (T, D) uint16 token-major; states (slots, D, W-1) uint16 updated in place."""
    out = np.zeros_like(x)
    load().oracle_varlen_bf16(_p(x), _p(w), _p(bias), _p(out), _p(qsl), len(qsl) - 1, x.shape[1],
                              w.shape[1], _p(cidx), _p(hinit), _p(states), int(pad), int(silu))
    return out


def update_bf16(x, state, w, bias, idx, pad, silu):
    out = np.zeros_like(x)
    load().oracle_update_bf16(_p(x), _p(state), _p(w), _p(bias), _p(out), _p(idx), x.shape[0],
                              x.shape[1], w.shape[1], int(pad), int(silu))
    return out
