"""Pin the CPU oracle to the reference: every golden vector, produced by running the reference
package's own public API on the CPU (tests/golden/make_golden.py), must be reproduced by
oracle/restate.py. States, ring rows and per-step windows are copies and must match bit for bit;
outputs within one rounding of the storage dtype (the oracle sums in float64, the reference in
float32)."""

import numpy as np
import pytest

import oracle
from golden import load, names

# Outputs: the oracle and the reference round different float sums, which may land on the two
# sides of a rounding boundary of the storage dtype.
OUT_TOL = {"bf16": 2.0**-7, "f16": 2.0**-10, "f32": 2.0**-20}


def _close(got, ref, dtype, mask=None):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    if mask is not None:
        got, ref = got[mask], ref[mask]
    tol = OUT_TOL[dtype]
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    assert err.max(initial=0.0) <= tol, err.max()
    if dtype != "f32":
        # Nearly all 16-bit elements must round identically.
        assert np.mean(got == ref) >= 0.98


def _bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("name", names("fn_"))
def test_fn_golden(name):
    meta, a = load(name)
    dt = a.dtypes["x"]
    out = oracle.fwd(a["x"], a["w"], a.get("b"), meta["act"] == "silu", dt)
    _close(out, a["out"], dt)


@pytest.mark.parametrize("name", names("varlen_"))
def test_varlen_golden(name):
    meta, a = load(name)
    states = a["st0"] if meta["states"] else None
    out, st = oracle.varlen(a["x"], a["w"], a.get("b"), a["qsl"], a.get("cidx") if states is not None else None,
                            a.get("hinit") if states is not None else None, states, True, meta["pad"], "bf16")
    mask = a["mask"].astype(bool)
    _close(out, a["out"], "bf16", mask)
    if states is not None:
        _bits_equal(st, a["st"])


@pytest.mark.parametrize("name", names("update_"))
def test_update_golden(name):
    meta, a = load(name)
    dt = a.dtypes["x"]
    x = a["x"]
    if meta["L"] > 1 or meta["inter"] is not None:
        x = x.reshape(x.shape[0], x.shape[1], -1) if x.ndim == 3 else x[..., None]
    inter = None
    if meta["inter"] == "dense":
        inter = a["inter0"]
    elif meta["inter"] == "dedup":
        S, D, PW = a["inter0"].shape
        L = meta["L"]
        K = PW - L + 1
        dense0 = np.empty((S, L, D, K), np.float32)
        for t in range(L):
            dense0[:, t] = a["inter0"][:, :, t : t + K]
        inter = dense0
    out, st, it = oracle.update(x, a["st0"], a["w"], a.get("b"), meta["act"] == "silu",
                                a.get("idx"), meta["pad"], inter, a.get("iidx"), dt)
    mask = a["mask"].astype(bool)
    _close(out[mask], a["out"][mask], dt)
    _bits_equal(st, a["st"])
    if meta["inter"] == "dense":
        _bits_equal(it, a["inter"])
    elif meta["inter"] == "dedup":
        S, D, PW = a["inter"].shape
        L = meta["L"]
        K = PW - L + 1
        for t in range(L):
            _bits_equal(it[:, t], a["inter"][:, :, t : t + K])


@pytest.mark.parametrize("name", [n for n in names("ring_") if n != "ring_convert"])
def test_ring_golden(name):
    meta, a = load(name)
    dt = a.dtypes["ring0"]
    ring = a["ring0"]
    mask = a["mask"].astype(bool)
    for s in range(meta["steps"]):
        out, ring = oracle.update_ring(a[f"x{s}"], ring, a["w"], a.get("b"), True,
                                       a[f"lens{s}"], a.get("idx"), meta["pad"], dt)
        _close(out[mask], a[f"out{s}"][mask], dt)
        _bits_equal(ring, a[f"ring_after{s}"])


def test_ring_convert_golden():
    _, a = load("ring_convert")
    _bits_equal(oracle.to_ring(a["state"], a["seen"]), a["ring"])
    _bits_equal(oracle.from_ring(a["ring"], a["seen"]), a["back"])


def test_round_to_matches_numpy_f16_and_bf16_ties():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-8, 65504.0, 3.0e38], np.float32)
    assert np.array_equal(oracle.round_to(x, "f16"), x.astype(np.float16).astype(np.float32))
    # bf16 keeps 8 significant bits: 1 + 2^-8 is a tie and rounds to even (1.0); 1 + 3 * 2^-8
    # is a tie between 1 + 2^-7 and 1 + 2^-6 and rounds to the even 1 + 2^-6.
    r = oracle.round_to(x[:3], "bf16")
    assert r.tolist() == [1.0, 1.0, 1.015625]


@pytest.mark.parametrize("name", names("unpack_"))
def test_unpack_golden(name):
    """The fused decode+unpack vectors come from the reference's GPU kernel (ConvUpdateUnpack,
    unpack.py:33-222; tests/golden/make_golden_unpack.py), its only implementation."""
    meta, a = load(name)
    dt = a.dtypes["qkvz"]
    out, z, b, ga, st = oracle.update_unpack(a["qkvz"], a["ba"], a["state0"], a["w"], a.get("bias"),
                                             a["idx"], meta["heads"], meta["act"] is not None,
                                             meta["pad"], dt)
    _close(out, a["out"], dt)
    _bits_equal(z, a["z"])
    _bits_equal(b, a["b"])
    _bits_equal(ga, a["a"])
    _bits_equal(st, a["state"])
