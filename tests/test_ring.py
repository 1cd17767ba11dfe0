"""Ring-state decode (causal_conv1d_update_ring) and layout conversion on the GPU. Mirrors the
reference's tests/test_ring.py with the oracle as the expected values."""

import random

import numpy as np
import pytest
import torch

import oracle
from _util import TAG, assert_bits, assert_close, to_np
from causal_conv1d_cute import causal_conv1d_update, causal_conv1d_update_ring, from_ring, to_ring

PAD = -1


def test_layout_conversion_has_no_cpu_path():
    from causal_conv1d_cute import Unsupported

    with pytest.raises(Unsupported):
        to_ring(torch.randn(7, 32, 3), torch.zeros(7, dtype=torch.int32))
    with pytest.raises(ValueError):
        to_ring(torch.randn(7, 32), torch.zeros(7, dtype=torch.int32))


@pytest.mark.gpu
def test_round_trip_between_layouts():
    torch.manual_seed(0)
    st = torch.randn(7, 32, 3, device="cuda")
    n = torch.randint(0, 50, (7,), device="cuda", dtype=torch.int32)
    ring = to_ring(st, n)
    assert ring.shape == (7, 3, 32) and torch.equal(from_ring(ring, n), st)
    assert np.array_equal(ring.cpu().numpy(), oracle.to_ring(st.cpu().numpy(), n.cpu().numpy()))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("K", [1, 2, 3, 7])
@pytest.mark.parametrize("layout", ["contiguous", "strided"])
def test_conversion_kernels_match_oracle(K, dtype, layout):
    """Vector kernel (contiguous, 16-byte aligned) and element kernel (strided views, odd dim),
    negative and large sequence lengths, int64 lengths."""
    torch.manual_seed(K)
    S, D = 33, 1024 if layout == "contiguous" else 100
    st = torch.randn(S, D, K, device="cuda").to(dtype)
    if layout == "strided":
        st = torch.randn(S, K, D + 3, device="cuda").to(dtype)[:, :, 1:D + 1].transpose(1, 2)
    n = torch.randint(-1000, 10**6, (S,), device="cuda", dtype=torch.int64)
    ring = to_ring(st, n)
    exp = oracle.to_ring(to_np(st), n.cpu().numpy())
    assert_bits(ring, exp)
    back_src = ring if layout == "contiguous" else ring.transpose(1, 2).contiguous().transpose(1, 2)
    back = from_ring(back_src, n)
    assert_bits(back, to_np(st))
    assert back.is_contiguous()


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(40))
def test_ring_decode_matches_oracle(seed):
    random.seed(seed)
    torch.manual_seed(seed)
    D = random.choice([64, 1024, 2048, 10240, 8192, 100])
    W = random.choice([2, 3, 4, 4, 4, 5, 8])
    B = random.choice([1, 2, 5, 48, 130, 131])  # 2 rows per thread below 128, 4 from 128
    dtype = random.choice([torch.bfloat16, torch.bfloat16, torch.float16, torch.float32])
    act = random.choice([None, "silu"])
    indexed = random.random() < 0.5
    K = W - 1
    slots = B + 4 if indexed else B
    w = torch.randn(D, W, device="cuda", dtype=dtype)
    b = torch.randn(D, device="cuda", dtype=dtype) if random.random() < 0.5 else None
    ordered = torch.randn(slots, D, K, device="cuda", dtype=dtype)
    seen = torch.randint(0, 97, (slots,), device="cuda", dtype=torch.int32)
    ring = to_ring(ordered, seen).contiguous()
    idx = None
    rows = torch.arange(B, device="cuda")
    if indexed:
        idx = torch.tensor(random.sample(range(slots), B), device="cuda", dtype=torch.int32)
        rows = idx.long()
    pads = [indexed and B > 1 and random.random() < 0.25 for _ in range(B)]
    if indexed and any(pads):
        idx[torch.tensor(pads, device="cuda")] = PAD
    live = np.array([not p for p in pads])
    for _ in range(5):
        x = torch.randn(B, D, device="cuda", dtype=dtype)
        lens = seen[rows.clamp_min(0)] if indexed else seen
        ring_before = to_np(ring)
        y = causal_conv1d_update_ring(x, ring, w, b, act, lens, idx, PAD)
        torch.cuda.synchronize()
        r_out, r_ring = oracle.update_ring(to_np(x), ring_before, to_np(w), to_np(b), act is not None,
                                           to_np(lens), to_np(idx), PAD, TAG[dtype])
        assert_close(to_np(y)[live], r_out[live], dtype)
        assert_bits(ring, r_ring)
        if not indexed:
            # The ordered-state decode sums in the same order: identical outputs.
            ordered_state = from_ring(torch.from_numpy(ring_before).cuda().to(dtype), lens)
            assert torch.equal(causal_conv1d_update(x, ordered_state, w, b, act), y)
        live_rows = rows[torch.tensor(live, device="cuda")]
        seen[live_rows] += 1


@pytest.mark.gpu
def test_ring_with_channel_count_not_multiple_of_16():
    torch.manual_seed(0)
    D, W = (100, 4)
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    ordered = torch.randn(3, D, W - 1, device="cuda", dtype=torch.bfloat16)
    seen = torch.tensor([4, 5, 9], device="cuda", dtype=torch.int32)
    ring = to_ring(ordered, seen).contiguous()
    x = torch.randn(3, D, device="cuda", dtype=torch.bfloat16)
    y = causal_conv1d_update_ring(x, ring, w, None, "silu", seen)
    r_out, r_st, _ = oracle.update(to_np(x), to_np(ordered), to_np(w), None, True, None, PAD, None,
                                   None, "bf16")
    assert_close(y, r_out, torch.bfloat16)
    assert_bits(from_ring(ring, seen + 1), r_st)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [5, 130])
@pytest.mark.parametrize("form", ["plain", "silu", "bias", "silu+bias", "strided"])
def test_ring_decode_flag_forms(B, form):
    """Each compile-time form of the 16-bit ring kernel (SiLU and a contiguous bias on or off) and
    the run-time form that strided weights and a strided bias take, against the oracle."""
    torch.manual_seed(B)
    D, W = 1024, 4
    dtype = torch.bfloat16
    act = "silu" if "silu" in form or form == "strided" else None
    if form == "strided":
        w = torch.randn(D, W + 3, device="cuda", dtype=dtype)[:, 1:W + 1]
        b = torch.randn(D, 2, device="cuda", dtype=dtype)[:, 1]
    else:
        w = torch.randn(D, W, device="cuda", dtype=dtype)
        b = torch.randn(D, device="cuda", dtype=dtype) if "bias" in form else None
    ordered = torch.randn(B, D, W - 1, device="cuda", dtype=dtype)
    seen = torch.randint(0, 50, (B,), device="cuda", dtype=torch.int32)
    ring = to_ring(ordered, seen).contiguous()
    x = torch.randn(B, D, device="cuda", dtype=dtype)
    ring_before = to_np(ring)
    y = causal_conv1d_update_ring(x, ring, w, b, act, seen)
    r_out, r_ring = oracle.update_ring(to_np(x), ring_before, to_np(w), to_np(b), act is not None,
                                       to_np(seen), None, PAD, TAG[dtype])
    assert_close(y, r_out, dtype)
    assert_bits(ring, r_ring)
