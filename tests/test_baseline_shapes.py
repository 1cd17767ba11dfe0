"""Parity at the exact BASELINE configurations the performance claims rest on.

Each test calls the public API with the shapes, value distributions and options of one BASELINE
config and checks the result three ways:
- against the oracle (the numpy restatement of the reference's fallback, pinned to the reference's
  golden vectors) on whole batch rows, or on a channel subset where the full tensor would take the
  float64 oracle minutes;
- against the fp32 PyTorch reference (causal_conv1d_cute.testing) on every element;
- cache writes (conv states, ring rows, per-step windows) bit for bit over the whole cache,
  including the slots the call must leave untouched.
Outputs: atol = rtol = 1e-2 (bf16). Where a scalar kernel exists for the same call (reached by a
view whose rows are not 16-byte aligned), the whole result must equal it bit for bit.
"""

import numpy as np
import pytest
import torch

import oracle
from _util import assert_bits, assert_close, to_np
import causal_conv1d_cute as C
from causal_conv1d_cute import testing as T

bf = torch.bfloat16
TOL = 1e-2
D = 8192


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def _w(W, g):
    return (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(bf)


def _bias(g):
    return (torch.randn(D, device="cuda", generator=g) * 0.1).to(bf)


def _misaligned(shape, src):
    """A tensor of `shape` holding src's values whose storage starts one element past a 16-byte
    line, which sends every call to the scalar kernels."""
    buf = torch.empty(src.numel() + 1, device=src.device, dtype=src.dtype)
    v = buf[1:].view(shape)
    v.copy_(src.reshape(shape))
    return v


# ---------------------------------------------------------------------------------------------
# Config 2: prefill bf16, x (8, 4096, 8192) token-major passed as its (8, 8192, 4096) view.
# ---------------------------------------------------------------------------------------------


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["channel_last", "channel_first"])
def test_config2_prefill(layout):
    B, L, W = 8, 4096, 4
    g = _gen(2)
    if layout == "channel_last":
        x = torch.randn(B, L, D, device="cuda", generator=g).to(bf).transpose(1, 2)
    else:
        x = torch.randn(B, D, L, device="cuda", generator=g).to(bf)
    w, b = _w(W, g), _bias(g)
    out = (torch.empty(B, L, D, device="cuda", dtype=bf).transpose(1, 2) if layout == "channel_last"
           else torch.empty(B, D, L, device="cuda", dtype=bf))
    y = C.causal_conv1d_fn(x, w, b, "silu", out=out)
    assert y.data_ptr() == out.data_ptr()
    for i in range(B):
        assert T.within(y[i], T.ref_fwd(x[i:i + 1], w, b, True)[0], TOL), f"batch row {i}"
    for i in (0, B - 1):
        ref = oracle.fwd(to_np(x[i:i + 1]), to_np(w), to_np(b), True, "bf16")
        assert_close(y[i:i + 1], ref, bf)
    if layout == "channel_last":
        xs = _misaligned((B, L, D), x.transpose(1, 2)).transpose(1, 2)
    else:
        xs = _misaligned((B, D, L), x)
    ys = C.causal_conv1d_fn(xs, w, b, "silu")
    assert torch.equal(y, ys)


# ---------------------------------------------------------------------------------------------
# Config 3: single-token indexed decode, B = 256 against a 1024-slot cache; and its ring form.
# ---------------------------------------------------------------------------------------------


def _config3(g):
    x = torch.randn(256, D, device="cuda", generator=g).to(bf)
    cache = torch.randn(1024, D, 3, device="cuda", generator=g).to(bf)
    idx = torch.randperm(1024, device="cuda", generator=g)[:256].to(torch.int32)
    return x, cache, idx


@pytest.mark.gpu
@pytest.mark.parametrize("checks", [True, False])
def test_config3_indexed_decode(checks):
    """Both decode variants (with and without the device status word) at the config-3 shape."""
    g = _gen(3)
    x, cache0, idx = _config3(g)
    w, b = _w(4, g), _bias(g)
    cache = cache0.clone()
    C.set_device_checks(checks)
    try:
        y = C.causal_conv1d_update(x, cache, w, b, "silu", idx)
    finally:
        C.set_device_checks(True)
    r_out, r_st, _ = oracle.update(to_np(x), to_np(cache0), to_np(w), to_np(b), True, to_np(idx),
                                   -1, None, None, "bf16")
    assert_close(y, r_out, bf)
    assert_bits(cache, r_st)
    t_out, t_st, _ = T.ref_update(x, cache0, w, b, True, idx)
    assert T.within(y, t_out, TOL)
    assert torch.equal(cache, t_st)
    # The scalar kernel (rows not 16-byte aligned) gives the same bits.
    cs = _misaligned(cache0.shape, cache0)
    ys = C.causal_conv1d_update(_misaligned(x.shape, x), cs, w, b, "silu", idx)
    assert torch.equal(y, ys)
    assert torch.equal(cache, cs)


@pytest.mark.gpu
def test_config3_ring_decode():
    g = _gen(31)
    x = torch.randn(256, D, device="cuda", generator=g).to(bf)
    ring0 = torch.randn(256, 3, D, device="cuda", generator=g).to(bf)
    seen = torch.randint(1, 8193, (256,), device="cuda", generator=g, dtype=torch.int32)
    w, b = _w(4, g), _bias(g)
    ring = ring0.clone()
    y = C.causal_conv1d_update_ring(x, ring, w, b, "silu", seen)
    r_out, r_ring = oracle.update_ring(to_np(x), to_np(ring0), to_np(w), to_np(b), True,
                                       to_np(seen), None, -1, "bf16")
    assert_close(y, r_out, bf)
    assert_bits(ring, r_ring)
    t_out, t_ring = T.ref_update_ring(x, ring0, w, b, True, seen)
    assert T.within(y, t_out, TOL)
    assert torch.equal(ring, t_ring)
    # The ordered-state decode of the same history gives the same outputs bit for bit.
    st = C.from_ring(ring0, seen)
    y2 = C.causal_conv1d_update(x, st, w, b, "silu")
    assert torch.equal(y, y2)
    assert torch.equal(C.to_ring(st, seen + 1), ring)
    rs = _misaligned(ring0.shape, ring0)
    ys = C.causal_conv1d_update_ring(_misaligned(x.shape, x), rs, w, b, "silu", seen)
    assert torch.equal(y, ys)
    assert torch.equal(ring, rs)


# ---------------------------------------------------------------------------------------------
# Config 4: 4-step speculative verify, B = 64, dense per-step windows, permuted indices.
# ---------------------------------------------------------------------------------------------


@pytest.mark.gpu
def test_config4_spec_decode():
    B, S = 64, 4
    g = _gen(4)
    x = torch.randn(B, S, D, device="cuda", generator=g).to(bf).transpose(1, 2)
    st0 = torch.randn(B, D, 3, device="cuda", generator=g).to(bf)
    perm = torch.randperm(B, device="cuda", generator=g).to(torch.int32)
    w, b = _w(4, g), _bias(g)
    inter0 = torch.randn(B, S, D, 3, device="cuda", generator=g).to(bf)
    st, inter = st0.clone(), inter0.clone()
    y = C.causal_conv1d_update(x, st, w, b, "silu", perm, -1, inter, perm)
    assert y.shape == x.shape and y.stride() == x.stride()
    r_out, r_st, r_it = oracle.update(to_np(x), to_np(st0), to_np(w), to_np(b), True, to_np(perm),
                                      -1, to_np(inter0), to_np(perm), "bf16")
    assert_close(y, r_out, bf)
    assert_bits(st, r_st)
    assert_bits(inter, r_it)
    t_out, t_st, t_it = T.ref_update(x, st0, w, b, True, perm, -1, inter0, perm)
    assert T.within(y, t_out, TOL)
    assert torch.equal(st, t_st) and torch.equal(inter, t_it)


# ---------------------------------------------------------------------------------------------
# Config 5: packed prefill of 32 lognormal(7, 1) sequences at D = 8192, in-place state cache.
# ---------------------------------------------------------------------------------------------


def _config5(W, seed=0):
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(rng.lognormal(7, 1, 32)), 1, 8192).astype(np.int64)
    T_ = int(lens.sum())
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device="cuda", dtype=torch.int32)
    cidx = torch.from_numpy(rng.choice(512, 32, replace=False).astype(np.int32)).cuda()
    hinit = torch.from_numpy(rng.random(32) < 0.5).cuda()
    g = _gen(50 + W)
    x = torch.randn(T_, D, device="cuda", generator=g).to(bf)
    w = _w(W, g)
    states = torch.randn(512, D, W - 1, device="cuda", generator=g).to(bf)
    return qsl, cidx, hinit, x, w, states


@pytest.mark.gpu
@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_config5_varlen(W):
    qsl, cidx, hinit, xt, w, st0 = _config5(W)
    results = {}
    for layout in ("token_major", "channel_first"):
        x = xt.t() if layout == "token_major" else xt.t().contiguous()
        st = st0.clone()
        y = C.causal_conv1d_varlen_fn(x, w, None, qsl, cidx, hinit, st, "silu")
        results[layout] = (y, st)
    y, st = results["token_major"]
    yc, stc = results["channel_first"]
    t_out, t_st = T.ref_varlen(xt.t(), w, None, qsl, cidx, hinit, st0, True)
    for got, got_st in ((y, st), (yc, stc)):
        assert T.within(got, t_out, TOL)
        assert torch.equal(got_st, t_st)
    # Oracle: every sequence and token, every 8th channel (and the whole state cache through it).
    sub = torch.arange(0, D, 8, device="cuda")
    r_out, r_st = oracle.varlen(to_np(xt.t()[sub]), to_np(w[sub]), None, to_np(qsl), to_np(cidx),
                                to_np(hinit), to_np(st0[:, sub]), True, -1, "bf16")
    assert_close(y[sub], r_out, bf)
    assert_close(yc[sub], r_out, bf)
    assert_bits(st[:, sub], r_st)
    # Scalar path over token rows that are not 16-byte aligned: the same bits.
    sts = st0.clone()
    ys = C.causal_conv1d_varlen_fn(_misaligned(xt.shape, xt).t(), w, None, qsl, cidx, hinit, sts,
                                   "silu")
    assert torch.equal(y, ys) and torch.equal(st, sts)
