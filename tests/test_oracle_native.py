"""The C port of the oracle (the CPU baseline bench.py times) agrees with the numpy oracle:
states bit-exact, outputs within one bf16 rounding."""

import numpy as np

import oracle
from oracle import native


def _bf16_bits(a):
    return (oracle.round_to(a, "bf16").view(np.uint32) >> 16).astype(np.uint16)


def _f(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def test_fwd_channel_last():
    rng = np.random.default_rng(0)
    B, L, D, W = 2, 70, 48, 4
    x = _bf16_bits(rng.standard_normal((B, L, D)).astype(np.float32))
    w = _bf16_bits(rng.uniform(-0.5, 0.5, (D, W)).astype(np.float32))
    b = _bf16_bits((rng.standard_normal(D) * 0.1).astype(np.float32))
    out = native.fwd_cl_bf16(x, w, b, True)
    ref = oracle.fwd(_f(x).transpose(0, 2, 1), _f(w), _f(b), True, "bf16").transpose(0, 2, 1)
    np.testing.assert_allclose(_f(out), ref, rtol=2**-7, atol=2**-7)


def test_varlen_and_update():
    rng = np.random.default_rng(1)
    D, W, K = 32, 4, 3
    lens = [5, 1, 2, 0, 30]
    qsl = np.array([0] + list(np.cumsum(lens)), np.int32)
    T = int(qsl[-1])
    x = _bf16_bits(rng.standard_normal((T, D)).astype(np.float32))
    w = _bf16_bits(rng.uniform(-0.5, 0.5, (D, W)).astype(np.float32))
    st = _bf16_bits(rng.standard_normal((8, D, K)).astype(np.float32))
    cidx = np.array([3, 0, -1, 5, 1], np.int32)
    hinit = np.array([1, 0, 1, 1, 1], np.uint8)
    st_c = st.copy()
    out = native.varlen_bf16(x, w, None, qsl, cidx, hinit, st_c, -1, True)
    r_out, r_st = oracle.varlen(_f(x).T, _f(w), None, qsl, cidx, hinit, _f(st), True, -1, "bf16")
    mask = ~np.isnan(r_out)
    np.testing.assert_allclose(_f(out).T[mask], r_out[mask], rtol=2**-7, atol=2**-7)
    assert np.array_equal(_f(st_c), r_st)

    xs = _bf16_bits(rng.standard_normal((4, D)).astype(np.float32))
    idx = np.array([7, 2, -1, 4], np.int32)
    st_u = st.copy()
    o = native.update_bf16(xs, st_u, w, None, idx, -1, False)
    r_o, r_s, _ = oracle.update(_f(xs), _f(st), _f(w), None, False, idx, -1, None, None, "bf16")
    live = idx >= 0
    np.testing.assert_allclose(_f(o)[live], r_o[live], rtol=2**-7, atol=2**-7)
    assert np.array_equal(_f(st_u), r_s)
