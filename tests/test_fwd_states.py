"""Prefill with the Dao-AILab extras (causal_conv1d_fwd_states and the dao_compat shim that serves
it) on the GPU against the oracle: outputs within the dtype tolerance, final states bit for bit."""

import numpy as np
import pytest
import torch

import oracle
from _util import TAG, assert_bits, assert_close, to_np
from causal_conv1d_cute import causal_conv1d_fwd_states, dao_compat

LENGTHS = [1, 2, 3, 7, 129, 300]


def _inputs(B, D, L, W, dtype, layout, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if layout == "btd":
        x = torch.randn(B, L, D, device="cuda", generator=g).to(dtype).transpose(1, 2)
    else:
        x = torch.randn(B, D, L, device="cuda", generator=g).to(dtype)
    w = (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(dtype)
    b = (torch.randn(D, device="cuda", generator=g) * 0.1).to(dtype)
    init = torch.randn(B, W - 1, D, device="cuda", generator=g).to(dtype).transpose(1, 2)
    return x, w, b, init


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["btd", "bdl"])
@pytest.mark.parametrize("W", [2, 3, 4, 5, 6, 7, 8])
def test_initial_and_final_states(W, layout):
    for i, L in enumerate(LENGTHS):
        x, w, b, init = _inputs(3, 256, L, W, torch.bfloat16, layout, W * 10 + i)
        out, fin = causal_conv1d_fwd_states(x, w, b, None, init, True, None, "silu")
        torch.cuda.synchronize()
        r_out, r_fin = oracle.fwd_states(to_np(x), to_np(w), to_np(b), None, to_np(init), True, "bf16")
        assert_close(out, r_out, torch.bfloat16)
        assert_bits(fin, r_fin)
        assert out.stride() == x.stride() or layout == "bdl"
        assert fin.shape == (3, 256, W - 1) and fin.stride(1) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_other_dtypes_and_no_initial_state(dtype):
    x, w, b, _ = _inputs(2, 128, 77, 4, dtype, "btd", 3)
    out, fin = causal_conv1d_fwd_states(x, w, None, None, None, True, None, None)
    torch.cuda.synchronize()
    r_out, r_fin = oracle.fwd_states(to_np(x), to_np(w), None, None, None, False, TAG[dtype])
    assert_close(out, r_out, dtype)
    assert_bits(fin, r_fin)


@pytest.mark.gpu
def test_final_states_out_is_written_in_place_with_its_strides():
    x, w, b, init = _inputs(2, 512, 5, 6, torch.bfloat16, "btd", 4)
    fin = torch.full((2, 512, 5), 7.0, device="cuda", dtype=torch.bfloat16)  # contiguous (B, D, K)
    out, got = causal_conv1d_fwd_states(x, w, b, None, init, True, fin, "silu")
    torch.cuda.synchronize()
    assert got is fin
    _, r_fin = oracle.fwd_states(to_np(x), to_np(w), to_np(b), None, to_np(init), True, "bf16")
    assert_bits(fin, r_fin)


@pytest.mark.gpu
def test_empty_sequence_returns_the_initial_state_tail():
    x, w, b, init = _inputs(2, 64, 0, 4, torch.bfloat16, "btd", 5)
    out, fin = causal_conv1d_fwd_states(x, w, b, None, init, True, None, None)
    torch.cuda.synchronize()
    assert out.shape == (2, 64, 0)
    assert torch.equal(fin, init)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["btd", "bdl"])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_sequence_ids(W, layout):
    # L = 301: the second row's ids start 4 bytes past a 16-byte line, so the staged kernel loads
    # them one by one there and four to a 16-byte load in the first row.
    for L in (300, 301):
        B, D = 2, 256
        x, w, b, _ = _inputs(B, D, L, W, torch.bfloat16, layout, 40 + W)
        rng = np.random.default_rng(W)
        cuts = [np.sort(rng.choice(np.arange(1, L), 6, replace=False)) for _ in range(B)]
        seq = np.stack([np.searchsorted(c, np.arange(L), side="right") for c in cuts]).astype(np.int32)
        seq[1, 200:205] = 0  # an id that recurs after other ids
        out = causal_conv1d_fwd_states(x, w, b, torch.from_numpy(seq).cuda(), None, False, None,
                                       "silu")
        torch.cuda.synchronize()
        r_out, _ = oracle.fwd_states(to_np(x), to_np(w), to_np(b), seq, None, True, "bf16")
        assert_close(out, r_out, torch.bfloat16)


@pytest.mark.gpu
def test_rejections():
    x, w, b, init = _inputs(2, 64, 10, 4, torch.bfloat16, "btd", 6)
    seq = torch.zeros(2, 10, device="cuda", dtype=torch.int32)
    with pytest.raises(ValueError):
        causal_conv1d_fwd_states(x, w, b, seq, init, False, None, None)
    with pytest.raises(ValueError):
        causal_conv1d_fwd_states(x, w, b, seq, None, True, None, None)
    with pytest.raises(ValueError):
        causal_conv1d_fwd_states(x, w, b, None, init, True, init, None)
    with pytest.raises(ValueError):
        causal_conv1d_fwd_states(x, w, b, torch.zeros(2, 9, device="cuda"), None, False, None, None)


@pytest.mark.gpu
def test_dao_shim_serves_state_calls():
    x, w, b, init = _inputs(2, 256, 33, 4, torch.bfloat16, "btd", 7)

    def upstream(*a, **k):
        raise AssertionError("served calls must not reach upstream")

    before = dao_compat.stats["fn_fast"]
    out, fin = dao_compat.around_fn(upstream, x, w, b, initial_states=init, return_final_states=True,
                                    activation="silu")
    seq = torch.zeros(2, 33, device="cuda", dtype=torch.int32)
    out2 = dao_compat.around_fn(upstream, x, w, b, seq_idx=seq, activation="silu")
    torch.cuda.synchronize()
    assert dao_compat.stats["fn_fast"] == before + 2
    r_out, r_fin = oracle.fwd_states(to_np(x), to_np(w), to_np(b), None, to_np(init), True, "bf16")
    assert_close(out, r_out, torch.bfloat16)
    assert_bits(fin, r_fin)
    r_out2, _ = oracle.fwd_states(to_np(x), to_np(w), to_np(b), None, None, True, "bf16")
    assert_close(out2, r_out2, torch.bfloat16)
