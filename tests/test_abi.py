"""The C ABI library loads without a GPU, exports every function include/cc1d.h declares, and the
ctypes argument lists match the header. Calls here stop at host-side validation or at a zero
size, so nothing is launched."""

import ctypes
import re
from pathlib import Path

import pytest

from causal_conv1d_cute import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "cc1d.h"


def _declarations():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(cc1d_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(2).split(",") if p.strip() and p.strip() != "void"]
        decls[m.group(1)] = params
    return decls


def _ctype_of(param):
    p = param.replace("const", "").strip()
    if "*" in p:
        return ctypes.c_void_p
    if p.startswith("int64_t"):
        return ctypes.c_int64
    if p.startswith("int32_t") or p.startswith("cc1d_status_t"):
        return ctypes.c_int32
    raise AssertionError(param)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    decls = _declarations()
    assert set(decls) == set(_lib.EXPORTS)
    for name in decls:
        assert hasattr(lib, name), name
    assert lib.cc1d_abi_version() == 1


@pytest.mark.parametrize("name", sorted(_lib.SIGNATURES))
def test_ctypes_signature_matches_header(name):
    decls = _declarations()
    assert [_ctype_of(p) for p in decls[name]] == _lib.SIGNATURES[name]


def test_status_strings():
    lib = _lib.load()
    for code in range(6):
        assert lib.cc1d_status_string(code)
    assert lib.cc1d_status_string(0) == b"ok"


def test_host_validation_rejects_before_launch():
    lib = _lib.load()
    # bad dtype
    st = lib.cc1d_fwd(None, 0, 0, 0, None, 0, 0, None, 0, None, 0, 0, 0, 1, 16, 16, 4, 7, 0, None)
    assert st == 2 and b"dtype" in lib.cc1d_last_error()
    # bad width
    st = lib.cc1d_fwd(None, 0, 0, 0, None, 0, 0, None, 0, None, 0, 0, 0, 1, 16, 16, 9, 0, 0, None)
    assert st == 3
    # negative size
    st = lib.cc1d_fwd(None, 0, 0, 0, None, 0, 0, None, 0, None, 0, 0, 0, -1, 16, 16, 4, 0, 0, None)
    assert st == 1
    # null pointers with work to do
    st = lib.cc1d_fwd(None, 0, 0, 0, None, 0, 0, None, 0, None, 0, 0, 0, 1, 16, 16, 4, 0, 0, None)
    assert st == 1
    # empty work is a successful no-op
    st = lib.cc1d_fwd(None, 0, 0, 0, None, 0, 0, None, 0, None, 0, 0, 0, 0, 16, 16, 4, 0, 0, None)
    assert st == 0
    # state shorter than width - 1
    args = [None, 0, 0, 0, None, 0, 0, 0, 2, 4, None, 0, 0, None, 0, None, 0, 0, 0, None, -1,
            None, 0, 0, 0, 0, 0, None, 1, 16, 1, 4, 0, 0, None, None]
    assert lib.cc1d_update(*args) == 1
    # varlen token count beyond int32
    vargs = [None, 0, 0, None, 0, 0, None, 0, None, 0, 0, None, 1, 2**31, None, None, None,
             0, 0, 0, 0, -1, 16, 4, 0, 0, None, None]
    assert lib.cc1d_varlen(*vargs) == 1
    # fused decode: dim not a multiple of the vector width
    uargs = [1, 0, 1, 0, 1, 0, 1, None, 1, 1, 1, 1, 1, -1, 1, 12, 16, 4, 4, 0, 0, 1, None]
    assert lib.cc1d_update_unpack(*uargs) == 4
    # prefill with states: sequence ids exclude states
    fargs = [1, 0, 0, 0, 1, 0, 0, None, 0, 1, 0, 0, 0, 1, 0, 0, 1, 0, 0, 0, None, 0, 0, 0,
             1, 16, 16, 4, 0, 0, None]
    assert lib.cc1d_fwd_states(*fargs) == 1 and b"exclude" in lib.cc1d_last_error()
    # ring conversion: state and ring overlap
    rargs = [4096, 48, 3, 1, 4096, 48, 16, 1, 8, 1, 16, 4, 0, None]
    assert lib.cc1d_to_ring(*rargs) == 1 and b"overlap" in lib.cc1d_last_error()
    # ring conversion: width outside 2..8
    rargs[11] = 9
    assert lib.cc1d_from_ring(*rargs) == 3
