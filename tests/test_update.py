"""Single-token decode (causal_conv1d_update, CausalConv1d.update) on the GPU. Mirrors the
reference's tests/test_update.py: outputs against the oracle and the accuracy classifier, states
bit-exact."""

import pytest
import torch

import oracle
from _util import TAG, assert_bits, assert_close, to_np
from causal_conv1d_cute import CausalConv1d, causal_conv1d_update, device_status
from causal_conv1d_cute import testing as T
from causal_conv1d_cute.api import padded_width


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 3, 64, 131])
@pytest.mark.parametrize("act", [None, "silu"])
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("W", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("D", [64, 1536])
def test_standard_state(D, W, bias, act, B):
    case = T.Case("t", "update", D, W, B, 1, bias, act)
    t = T.make_inputs(case)
    ref_out, ref_state = T.reference(case, t)
    state = t["state"].clone()
    out = causal_conv1d_update(t["x"], state, t["w"], t["b"], act)
    torch.cuda.synchronize()
    assert T.check(case, t, out, ref_out)[0] == "ok"
    assert_bits(state, ref_state)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_against_oracle(dtype, W):
    torch.manual_seed(W)
    B, D = 9, 256
    x = torch.randn(B, D, device="cuda", dtype=dtype)
    w = torch.rand(D, W, device="cuda", dtype=dtype) - 0.5
    b = torch.randn(D, device="cuda", dtype=dtype) * 0.1
    st0 = torch.randn(B + 3, D, W - 1, device="cuda", dtype=dtype)
    idx = torch.randperm(B + 3, device="cuda")[:B].to(torch.int32)
    st = st0.clone()
    out = causal_conv1d_update(x, st, w, b, "silu", idx)
    r_out, r_st, _ = oracle.update(to_np(x), to_np(st0), to_np(w), to_np(b), True, to_np(idx), -1,
                                   None, None, TAG[dtype])
    assert_close(out, r_out, dtype)
    assert_bits(st, r_st)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 8, 131, 256])
@pytest.mark.parametrize(
    "D,W,bias,act", [(1536, 7, True, None), (2048, 3, False, None), (2048, 4, False, "silu"),
                     (256, 2, True, "silu")]
)
def test_padded_state(D, W, bias, act, B):
    """Power-of-two padded state (batch, dim, P): history in the last W-1 entries, whole row
    shifts (reference tests/test_update.py:24-39, update.py:235-316)."""
    case = T.Case("t", "update", D, W, B, 1, bias, act)
    t = T.make_inputs(case)
    ref_out, ref_state = T.reference(case, t)
    layer = CausalConv1d(t["w"], t["b"], act)
    P = layer.wpad.shape[1]
    assert P == padded_width(W)
    hist = torch.randn(B, D, P - (W - 1), device="cuda", dtype=case.dtype)
    state = torch.cat([hist, t["state"]], dim=-1).contiguous()
    before = state.clone()
    out = layer.update(t["x"], state)
    torch.cuda.synchronize()
    assert T.check(case, t, out, ref_out)[0] == "ok"
    assert_bits(state[..., P - (W - 1):], ref_state)
    assert_bits(state[..., : P - 1], before[..., 1:])


@pytest.mark.gpu
@pytest.mark.parametrize("S", [4, 6, 9])
def test_state_longer_than_history(S):
    """Any state length >= W - 1 through the functional API (the reference's fallback case)."""
    torch.manual_seed(S)
    B, D, W = 5, 96, 4
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st0 = torch.randn(B + 2, D, S, device="cuda", dtype=torch.bfloat16)
    idx = torch.tensor([6, 0, 3, -1, 2], device="cuda", dtype=torch.int32)
    st = st0.clone()
    out = causal_conv1d_update(x, st, w, None, "silu", idx)
    r_out, r_st, _ = oracle.update(to_np(x), to_np(st0), to_np(w), None, True, to_np(idx), -1,
                                   None, None, "bf16")
    live = to_np(idx) >= 0
    assert_close(to_np(out)[live], r_out[live], torch.bfloat16)
    assert_bits(st, r_st)


@pytest.mark.gpu
def test_indices_and_padding():
    D, W, B, slots = (1536, 4, 8, 13)
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    idx = torch.randperm(slots, device="cuda")[:B].to(torch.int32)
    idx[2] = -1
    st0 = torch.randn(slots, D, W - 1, device="cuda", dtype=torch.bfloat16)
    st = st0.clone()
    out = causal_conv1d_update(x, st, w, None, "silu", conv_state_indices=idx)
    torch.cuda.synchronize()
    exp = st0.clone()
    for b in range(B):
        if int(idx[b]) >= 0:
            exp[int(idx[b])] = torch.cat([st0[int(idx[b])][:, 1:], x[b].unsqueeze(-1)], dim=1)
    assert_bits(st, exp)
    live = idx >= 0
    full = torch.cat([st0[idx.clamp_min(0).long()].float(), x.float().unsqueeze(-1)], -1)
    ref = torch.nn.functional.silu((full * w.float()).sum(-1))
    assert (out[live].float() - ref[live]).abs().max() < 0.07


@pytest.mark.gpu
def test_in_place_update_is_deterministic():
    """Every (row, channel group) is owned by one thread: repeated runs agree bit for bit
    (reference tests/test_update.py:63-74 pins the same race)."""
    D, W, B = (1536, 7, 1)
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st = torch.randn(B, D, 8, device="cuda", dtype=torch.bfloat16)
    ref = torch.cat([st[..., 1:], x.unsqueeze(-1)], -1)
    layer = CausalConv1d(w, None, None)
    for _ in range(100):
        s2 = st.clone()
        layer.update(x, s2)
        assert torch.equal(s2, ref)


@pytest.mark.gpu
def test_slot_outside_cache_is_skipped_and_reported(request):
    """A slot index beyond the cache is neither read nor written; the status word reports it."""
    request.node._expect_status = True
    D, W, B, slots = (256, 4, 4, 6)
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    st0 = torch.randn(slots, D, W - 1, device="cuda", dtype=torch.bfloat16)
    idx = torch.tensor([0, 1000, 2, -7], device="cuda", dtype=torch.int32)
    st = st0.clone()
    device_status()
    causal_conv1d_update(x, st, w, None, None, conv_state_indices=idx)
    assert device_status() == 1
    assert torch.equal(st[[1, 3, 4, 5]], st0[[1, 3, 4, 5]])
    assert torch.equal(st[0], torch.cat([st0[0][:, 1:], x[0].unsqueeze(-1)], 1))


@pytest.mark.gpu
@pytest.mark.parametrize("W,padded", [(4, False), (2, False), (8, True)])
def test_unchecked_decode_matches_checked(W, padded):
    """With the status word off the decode runs a variant without the slot report; it must give
    the same outputs and states bit for bit, skip the pad slot and slots outside the cache alike."""
    from causal_conv1d_cute import set_device_checks

    D, B, slots = 2048, 64, 80
    g = torch.Generator(device="cuda").manual_seed(W)
    x = torch.randn(B, D, device="cuda", dtype=torch.bfloat16, generator=g)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16, generator=g)
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16, generator=g)
    S = 8 if padded else W - 1
    st0 = torch.randn(slots, D, S, device="cuda", dtype=torch.bfloat16, generator=g)
    idx = torch.randperm(slots, device="cuda", generator=g)[:B].to(torch.int32)
    idx[5] = -1
    st_on, st_off = st0.clone(), st0.clone()
    out_on = causal_conv1d_update(x, st_on, w, b, "silu", conv_state_indices=idx)
    set_device_checks(False)
    try:
        out_off = causal_conv1d_update(x, st_off, w, b, "silu", conv_state_indices=idx)
    finally:
        set_device_checks(True)
    torch.cuda.synchronize()
    live = idx >= 0
    assert torch.equal(out_on[live], out_off[live])
    assert torch.equal(st_on, st_off)
    assert torch.equal(st_off[~torch.isin(torch.arange(slots, device="cuda"), idx)],
                       st0[~torch.isin(torch.arange(slots, device="cuda"), idx)])
