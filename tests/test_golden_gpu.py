"""The CUDA path reproduces the reference's own outputs (the golden vectors in tests/golden,
produced by the reference package): conv states, ring rows and per-step windows bit for bit,
outputs within the stated tolerance."""

import numpy as np
import pytest
import torch

from _util import TORCH, assert_bits, assert_close, from_np
from golden import load, names
import causal_conv1d_cute as C

PAD = -1


def _t(a, key):
    v = a.get(key)
    if v is None:
        return None
    tag = a.dtypes[key]
    if tag in TORCH:
        return from_np(v, TORCH[tag])
    return torch.from_numpy(np.ascontiguousarray(v)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("fn_"))
def test_fn(name):
    meta, a = load(name)
    x = _t(a, "x")
    if meta["layout"] == "btd":
        x = x.transpose(1, 2).contiguous().transpose(1, 2)
    y = C.causal_conv1d_fn(x, _t(a, "w"), _t(a, "b"), meta["act"])
    assert_close(y, a["out"], x.dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("varlen_"))
def test_varlen(name):
    meta, a = load(name)
    x = _t(a, "x").t().contiguous().t()  # token-major view, as the reference was called
    st = _t(a, "st0") if meta["states"] else None
    y = C.causal_conv1d_varlen_fn(x, _t(a, "w"), _t(a, "b"), _t(a, "qsl"),
                                  _t(a, "cidx") if st is not None else None,
                                  _t(a, "hinit") if st is not None else None, st, meta["act"], PAD)
    mask = a["mask"].astype(bool)
    assert_close(y, a["out"], torch.bfloat16, mask)
    if st is not None:
        assert_bits(st, a["st"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("update_"))
def test_update(name):
    meta, a = load(name)
    x = _t(a, "x")
    L = meta["L"]
    if L > 1 or meta["inter"] is not None:
        x = x.reshape(x.shape[0], x.shape[1], -1)
        x = x.transpose(1, 2).contiguous().transpose(1, 2)
    st = _t(a, "st0")
    inter = phys = None
    if meta["inter"] == "dense":
        inter = phys = _t(a, "inter0")
    elif meta["inter"] == "dedup":
        phys = _t(a, "inter0")
        S, D, PW = phys.shape
        K = PW - L + 1
        inter = phys.as_strided((S, L, D, K), (D * PW, 1, PW, 1))
    y = C.causal_conv1d_update(x, st, _t(a, "w"), _t(a, "b"), meta["act"], _t(a, "idx"), PAD, inter,
                               _t(a, "iidx") if inter is not None else None)
    mask = a["mask"].astype(bool)
    assert_close(y.cpu().float().numpy()[mask], a["out"][mask], x.dtype)
    assert_bits(st, a["st"])
    if phys is not None:
        assert_bits(phys, a["inter"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", [n for n in names("ring_") if n != "ring_convert"])
def test_ring(name):
    meta, a = load(name)
    ring = _t(a, "ring0")
    mask = a["mask"].astype(bool)
    for s in range(meta["steps"]):
        x = _t(a, f"x{s}")
        y = C.causal_conv1d_update_ring(x, ring, _t(a, "w"), _t(a, "b"), meta["act"], _t(a, f"lens{s}"),
                                        _t(a, "idx"), PAD)
        assert_close(y.cpu().float().numpy()[mask], a[f"out{s}"][mask], x.dtype)
        assert_bits(ring, a[f"ring_after{s}"])


@pytest.mark.gpu
def test_ring_convert():
    _, a = load("ring_convert")
    r = C.to_ring(_t(a, "state"), _t(a, "seen"))
    assert_bits(r, a["ring"])
    assert_bits(C.from_ring(r, _t(a, "seen")), a["back"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("unpack_"))
def test_update_unpack(name):
    """Fused decode+unpack against the reference's own GPU kernel's outputs."""
    from causal_conv1d_cute import unpack

    meta, a = load(name)
    q = _t(a, "qkvz")
    B, cols = q.shape
    wide = torch.zeros(B, cols + meta["row_extra"], device="cuda", dtype=q.dtype)
    wide[:, :cols] = q
    qkvz = wide[:, :cols]
    st = _t(a, "state0")
    out, z, b, ga = unpack.causal_conv1d_update_unpack(qkvz, _t(a, "ba"), st, _t(a, "w"),
                                                       _t(a, "bias"), _t(a, "idx"), meta["heads"],
                                                       meta["act"], meta["pad"])
    assert_close(out, a["out"], q.dtype)
    assert_bits(z, a["z"])
    assert_bits(b, a["b"])
    assert_bits(ga, a["a"])
    assert_bits(st, a["state"])
