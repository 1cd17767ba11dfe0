"""Every entry point can be captured in a CUDA graph and replayed: no host synchronisation, no
forbidden call during capture, identical results to eager execution."""

import pytest
import torch

import causal_conv1d_cute as C
from causal_conv1d_cute import unpack


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


@pytest.mark.gpu
def test_prefill_and_varlen_in_a_graph():
    torch.manual_seed(0)
    x = torch.randn(2, 300, 512, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    w = torch.randn(512, 4, device="cuda", dtype=torch.bfloat16)
    g, y = _capture(lambda: C.causal_conv1d_fn(x, w, None, "silu"))
    g.replay()
    assert torch.equal(y, C.causal_conv1d_fn(x, w, None, "silu"))

    qsl = torch.tensor([0, 7, 100, 300], device="cuda", dtype=torch.int32)
    xv = x[0]
    st0 = torch.randn(4, 512, 3, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    h = torch.tensor([True, False, True], device="cuda")
    g, y = _capture(lambda: C.causal_conv1d_varlen_fn(xv, w, None, qsl, None, h, st, "silu"))
    st.copy_(st0)
    g.replay()
    st_e = st0.clone()
    ye = C.causal_conv1d_varlen_fn(xv, w, None, qsl, None, h, st_e, "silu")
    assert torch.equal(y, ye) and torch.equal(st, st_e)


@pytest.mark.gpu
@pytest.mark.parametrize("W", [4, 8])
def test_channel_first_varlen_in_a_graph(W):
    """Channel-first varlen is two launches, the second a programmatic dependent of the first; the
    captured pair, replayed twice, must equal two eager calls (outputs and cache)."""
    torch.manual_seed(W)
    D, T = 512, 1000
    xv = torch.randn(D, T, device="cuda", dtype=torch.bfloat16)  # contiguous (dim, tokens)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    qsl = torch.tensor([0, 3, 150, 151, 600, 1000], device="cuda", dtype=torch.int32)
    cidx = torch.tensor([5, 0, 2, 6, 1], device="cuda", dtype=torch.int32)
    h = torch.tensor([True, False, True, True, False], device="cuda")
    st0 = torch.randn(8, D, W - 1, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    g, y = _capture(lambda: C.causal_conv1d_varlen_fn(xv, w, b, qsl, cidx, h, st, "silu"))
    st.copy_(st0)
    g.replay()
    y1 = y.clone()
    g.replay()
    st_e = st0.clone()
    ye1 = C.causal_conv1d_varlen_fn(xv, w, b, qsl, cidx, h, st_e, "silu")
    ye2 = C.causal_conv1d_varlen_fn(xv, w, b, qsl, cidx, h, st_e, "silu")
    torch.cuda.synchronize()
    assert torch.equal(y1, ye1) and torch.equal(y, ye2) and torch.equal(st, st_e)


@pytest.mark.gpu
def test_decode_paths_in_a_graph():
    torch.manual_seed(1)
    B, D = 16, 1024
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, 4, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    st0 = torch.randn(40, D, 3, device="cuda", dtype=torch.bfloat16)
    idx = torch.randperm(40, device="cuda")[:B].to(torch.int32)
    st = st0.clone()
    g, y = _capture(lambda: C.causal_conv1d_update(x, st, w, b, "silu", idx))
    st.copy_(st0)
    g.replay()
    st_e = st0.clone()
    assert torch.equal(y, C.causal_conv1d_update(x, st_e, w, b, "silu", idx))
    assert torch.equal(st, st_e)

    ring0 = torch.randn(B, 3, D, device="cuda", dtype=torch.bfloat16)
    seen = torch.randint(0, 50, (B,), device="cuda", dtype=torch.int32)
    ring = ring0.clone()
    g, y = _capture(lambda: C.causal_conv1d_update_ring(x, ring, w, b, "silu", seen))
    ring.copy_(ring0)
    g.replay()
    ring_e = ring0.clone()
    assert torch.equal(y, C.causal_conv1d_update_ring(x, ring_e, w, b, "silu", seen))
    assert torch.equal(ring, ring_e)

    qkvz = torch.randn(B, D + 256, device="cuda", dtype=torch.bfloat16)
    ba = torch.randn(B, 16, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    g, outs = _capture(lambda: unpack.causal_conv1d_update_unpack(qkvz, ba, st, w, b, idx, 8, "silu", -1))
    st.copy_(st0)
    g.replay()
    st_e = st0.clone()
    ref = unpack.causal_conv1d_update_unpack(qkvz, ba, st_e, w, b, idx, 8, "silu", -1)
    for a, e in zip(outs, ref):
        assert torch.equal(a, e)
    assert torch.equal(st, st_e)
