"""Packed variable-length prefill (causal_conv1d_varlen_fn) on the GPU. Mirrors the reference's
tests/test_varlen.py and adds the edge cases the single-launch ownership scheme has to get right:
sequences shorter than W - 1, empty sequences, sequences that start in the last tokens of a strip,
padding rows, layouts, widths 2..8, and no state cache."""

import random

import numpy as np
import pytest
import torch

import oracle
from _util import assert_bits, assert_close, to_np
from causal_conv1d_cute import causal_conv1d_varlen_fn, device_status

PAD = -1


def _batch(seed, widths=(2, 3, 4, 7, 8), dims=(64, 1024, 1536)):
    random.seed(seed)
    torch.manual_seed(seed)
    D, W = random.choice(dims), random.choice(widths)
    K, act, has_bias = W - 1, random.choice([None, "silu"]), random.random() < 0.5
    nseq = random.choice([1, 2, 5, 9, 33])
    lens = [random.choice([0, 1, 2, 3, K, K + 1, 17, 62, 63, 64, 65, 333, 1000]) for _ in range(nseq)]
    if sum(lens) == 0:
        lens[0] = 5
    slots = nseq + 3
    qsl = torch.tensor([0] + list(np.cumsum(lens)), device="cuda", dtype=torch.int32)
    cidx = torch.tensor(random.sample(range(slots), nseq), device="cuda", dtype=torch.int32)
    pads = [random.random() < 0.15 for _ in range(nseq)]
    cidx[torch.tensor(pads, device="cuda")] = PAD
    hinit = torch.tensor([random.random() < 0.5 for _ in range(nseq)], device="cuda")
    T = int(qsl[-1])
    x = torch.randn(D, T, device="cuda", dtype=torch.bfloat16)
    w = torch.rand(D, W, device="cuda", dtype=torch.bfloat16) - 0.5
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16) if has_bias else None
    st0 = torch.randn(slots, D, K, device="cuda", dtype=torch.bfloat16)
    return D, W, K, act, nseq, qsl, cidx, pads, hinit, x, w, b, st0


def _check(y, st, x, w, b, act, qsl, cidx, hinit, st0, with_states=True):
    r_out, r_st = oracle.varlen(to_np(x), to_np(w), to_np(b), to_np(qsl),
                                to_np(cidx) if with_states else None,
                                to_np(hinit) if with_states else None,
                                to_np(st0) if with_states else None, act is not None, PAD, "bf16")
    mask = ~np.isnan(r_out)
    assert_close(to_np(y), np.nan_to_num(r_out), torch.bfloat16, mask)
    if with_states:
        assert_bits(st, r_st)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["token_major", "channel_first"])
@pytest.mark.parametrize("seed", range(24))
def test_varlen_outputs_and_states(seed, layout):
    D, W, K, act, nseq, qsl, cidx, pads, hinit, x, w, b, st0 = _batch(seed)
    if layout == "token_major":
        x = x.t().contiguous().t()
    st = st0.clone()
    y = causal_conv1d_varlen_fn(x, w, b, qsl, cidx, hinit, st, act, PAD)
    torch.cuda.synchronize()
    _check(y, st, x, w, b, act, qsl, cidx, hinit, st0)


@pytest.mark.gpu
@pytest.mark.parametrize("W", [2, 3, 4, 5, 6, 7, 8])
def test_every_width_and_short_sequences(W):
    """Lengths around W - 1 and the 64-token strip boundary, every width."""
    torch.manual_seed(W)
    K = W - 1
    lens = [1, K, K + 1, 2, 60, 3, 1, 64, 0, 65, 128, 5, 59]
    D = 256
    qsl = torch.tensor([0] + list(np.cumsum(lens)), device="cuda", dtype=torch.int32)
    nseq = len(lens)
    cidx = torch.randperm(nseq + 2, device="cuda")[:nseq].to(torch.int32)
    hinit = torch.rand(nseq, device="cuda") < 0.5
    T = int(qsl[-1])
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16).t()
    w = torch.rand(D, W, device="cuda", dtype=torch.bfloat16) - 0.5
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16) * 0.1
    st0 = torch.randn(nseq + 2, D, K, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    y = causal_conv1d_varlen_fn(x, w, b, qsl, cidx, hinit, st, "silu", PAD)
    _check(y, st, x, w, b, "silu", qsl, cidx, hinit, st0)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_other_dtypes(dtype):
    torch.manual_seed(1)
    D, W, K = 128, 4, 3
    lens = [7, 1, 100, 2]
    qsl = torch.tensor([0] + list(np.cumsum(lens)), device="cuda", dtype=torch.int32)
    cidx = torch.tensor([3, 0, 1, 5], device="cuda", dtype=torch.int32)
    hinit = torch.tensor([1, 1, 0, 1], device="cuda", dtype=torch.uint8)
    x = torch.randn(sum(lens), D, device="cuda", dtype=dtype).t()
    w = torch.randn(D, W, device="cuda", dtype=dtype)
    st0 = torch.randn(6, D, K, device="cuda", dtype=dtype)
    st = st0.clone()
    y = causal_conv1d_varlen_fn(x, w, None, qsl, cidx, hinit, st, "silu", PAD)
    from _util import TAG
    r_out, r_st = oracle.varlen(to_np(x), to_np(w), None, to_np(qsl), to_np(cidx), to_np(hinit),
                                to_np(st0), True, PAD, TAG[dtype])
    assert_close(y, r_out, dtype)
    assert_bits(st, r_st)


@pytest.mark.gpu
def test_without_state_cache():
    D, W, K, act, nseq, qsl, cidx, pads, hinit, x, w, b, st0 = _batch(3)
    y = causal_conv1d_varlen_fn(x, w, b, qsl, None, None, None, act, PAD)
    _check(y, None, x, w, b, act, qsl, None, None, None, with_states=False)


@pytest.mark.gpu
def test_padding_rows_and_leading_gap_are_left_alone():
    """Tokens outside every sequence are not written; nothing before qsl[0] or after qsl[-1]
    is read into a sequence."""
    torch.manual_seed(0)
    D, W = 64, 4
    T = 120
    qsl = torch.tensor([10, 30, 31, 90], device="cuda", dtype=torch.int32)
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16).t()
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st0 = torch.randn(3, D, W - 1, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    hinit = torch.tensor([True, False, True], device="cuda")
    y = causal_conv1d_varlen_fn(x, w, None, qsl, None, hinit, st, "silu", PAD)
    _check(y, st, x, w, None, "silu", qsl, torch.arange(3, device="cuda", dtype=torch.int32),
           hinit, st0)


@pytest.mark.gpu
def test_bad_sequence_bounds_are_clamped_and_reported(request):
    request.node._expect_status = True
    D, W = 64, 4
    x = torch.randn(50, D, device="cuda", dtype=torch.bfloat16).t()
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st = torch.randn(2, D, W - 1, device="cuda", dtype=torch.bfloat16)
    qsl = torch.tensor([0, 20, 500], device="cuda", dtype=torch.int32)
    device_status()
    causal_conv1d_varlen_fn(x, w, None, qsl, None, None, st, None, PAD)
    assert device_status() & 2


@pytest.mark.gpu
@pytest.mark.parametrize("cols_extra", [0, 16, 6144, 8])
def test_token_major_views_of_wider_rows(cols_extra):
    D, W, K, act, nseq, qsl, cidx, pads, hinit, x, w, b, st0 = _batch(7, dims=(1024,))
    T = x.shape[1]
    wide = torch.zeros(T, D + cols_extra, device="cuda", dtype=torch.bfloat16)
    wide[:, :D] = x.t()
    xv = wide[:, :D].t()
    st = st0.clone()
    y = causal_conv1d_varlen_fn(xv, w, b, qsl, cidx, hinit, st, act, PAD)
    _check(y, st, x, w, b, act, qsl, cidx, hinit, st0)


def _chunk_edge_lengths(T, chunk, K):
    """Sequence lengths whose starts sit on, just before and just after warp-chunk edges of a
    channel-first row (so heads cross chunk ends), plus an empty and a one-token sequence."""
    starts = {0}
    for edge in range(chunk, T, chunk):
        for d in (-K, -K + 1, -1, 0, 1, K - 1):
            if 0 < edge + d < T:
                starts.add(edge + d)
    starts = sorted(starts)
    lens = [b - a for a, b in zip(starts, starts[1:] + [T])]
    lens.insert(3, 0)
    lens.insert(6, 1)
    lens[-1] -= 1
    return lens


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("W", [2, 4, 7, 8])
def test_channel_first_matches_token_major(W, dtype):
    """Contiguous (D, T) streams (stream pass + boundary launch) against token-major rows (one
    launch): sequence starts on and around the stream kernel's warp-chunk edges, rows whose end
    falls inside a chunk, an empty and a one-token sequence, a padding slot and sequences with and
    without initial state. The outputs must equal each other bit for bit (the same arithmetic in
    the same order) and the oracle's within tolerance; states bit-exact."""
    torch.manual_seed(W)
    K = W - 1
    ept = 32 if dtype != torch.float32 and W != 7 else 16
    D, T = 96, 3 * 32 * ept + 37
    lens = _chunk_edge_lengths(T, 32 * ept, K)
    nseq = len(lens)
    qsl = torch.tensor([0] + list(np.cumsum(lens)), device="cuda", dtype=torch.int32)
    slots = nseq + 3
    cidx = torch.randperm(slots, device="cuda")[:nseq].to(torch.int32)
    cidx[2] = PAD
    hinit = torch.rand(nseq, device="cuda") < 0.5
    hinit[0] = True
    x = torch.randn(D, T, device="cuda", dtype=dtype)
    w = torch.rand(D, W, device="cuda", dtype=dtype) - 0.5
    b = torch.randn(D, device="cuda", dtype=dtype) * 0.1
    st0 = torch.randn(slots, D, K, device="cuda", dtype=dtype)
    st_cf, st_tm = st0.clone(), st0.clone()
    y_cf = causal_conv1d_varlen_fn(x, w, b, qsl, cidx, hinit, st_cf, "silu", PAD)
    y_tm = causal_conv1d_varlen_fn(x.t().contiguous().t(), w, b, qsl, cidx, hinit, st_tm, "silu",
                                   PAD)
    torch.cuda.synchronize()
    assert torch.equal(st_cf, st_tm)
    live = int(qsl[-1])
    assert torch.equal(y_cf[:, :live], y_tm[:, :live])
    from _util import TAG

    r_out, r_st = oracle.varlen(to_np(x), to_np(w), to_np(b), to_np(qsl), to_np(cidx),
                                to_np(hinit), to_np(st0), True, PAD, TAG[dtype])
    mask = ~np.isnan(r_out)
    assert_close(to_np(y_cf), np.nan_to_num(r_out), dtype, mask)
    assert_bits(st_cf, r_st)


@pytest.mark.gpu
def test_channel_first_bad_bounds_are_clamped_and_reported(request):
    request.node._expect_status = True
    D, W, T = 64, 4, 3000
    x = torch.randn(D, T, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st = torch.randn(3, D, W - 1, device="cuda", dtype=torch.bfloat16)
    qsl = torch.tensor([0, 1500, 1200, 90000], device="cuda", dtype=torch.int32)
    device_status()
    causal_conv1d_varlen_fn(x, w, None, qsl, None, None, st, None, PAD)
    assert device_status() & 2
