"""Fused Gated DeltaNet decode (unpack.causal_conv1d_update_unpack and the sglang hook) on the GPU
against the oracle: conv outputs within tolerance, state and the Z/B/A copies bit-exact."""

import numpy as np
import pytest
import torch

import oracle
from _util import TAG, assert_bits, assert_close, to_np
from causal_conv1d_cute import sglang_compat, unpack

PAD = -1


def _inputs(B, D, zdim, heads, W, dtype, gdtype, slots, row_extra=0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkvz = torch.randn(B, D + zdim + row_extra, device="cuda", dtype=dtype, generator=g)[:, : D + zdim]
    ba = torch.randn(B, 2 * heads, device="cuda", dtype=gdtype, generator=g)
    w = torch.randn(D, W, device="cuda", dtype=dtype, generator=g) * 0.5
    bias = torch.randn(D, device="cuda", dtype=dtype, generator=g) * 0.1
    st0 = torch.randn(slots, D, W - 1, device="cuda", dtype=dtype, generator=g)
    return qkvz, ba, w, bias, st0


@pytest.mark.gpu
@pytest.mark.parametrize(
    "B,D,zdim,heads,W,dtype,gdtype,row_extra",
    [
        (4, 256, 128, 8, 4, torch.bfloat16, torch.bfloat16, 0),
        (33, 1024, 512, 16, 4, torch.bfloat16, torch.float32, 16),
        (3, 64, 64, 4, 3, torch.float16, torch.float16, 8),
        (7, 128, 32, 6, 2, torch.float32, torch.bfloat16, 0),
        # 128 rows and more take the wider CTAs; an odd count leaves a half row pair.
        (131, 512, 256, 16, 4, torch.bfloat16, torch.bfloat16, 0),
        (129, 256, 64, 8, 8, torch.float16, torch.float32, 8),
        (130, 96, 32, 40, 6, torch.bfloat16, torch.float32, 0),
    ],
)
def test_unpack_against_oracle(B, D, zdim, heads, W, dtype, gdtype, row_extra):
    slots = B + 3
    qkvz, ba, w, bias, st0 = _inputs(B, D, zdim, heads, W, dtype, gdtype, slots, row_extra)
    idx = torch.randperm(slots, device="cuda")[:B].to(torch.int32)
    idx[0] = PAD
    if B > 2:
        idx[2] = slots + 5  # outside the cache: treated like padding
    assert unpack.unpack_reason(qkvz, ba, st0, w, bias, heads) is None
    st = st0.clone()
    out, z, b, a = unpack.causal_conv1d_update_unpack(qkvz, ba, st, w, bias, idx, heads, "silu", PAD)
    r_out, r_z, r_b, r_a, r_st = oracle.update_unpack(to_np(qkvz), to_np(ba), to_np(st0), to_np(w),
                                                      to_np(bias), to_np(idx), heads, True, PAD,
                                                      TAG[dtype])
    assert_close(out, r_out, dtype)
    invalid = [i for i in range(B) if not 0 <= int(idx[i]) < slots]
    for i in invalid:
        assert_bits(out[i], qkvz[i, :D])
    assert_bits(z, r_z)
    assert_bits(b, r_b)
    assert_bits(a, r_a)
    assert_bits(st, r_st)


@pytest.mark.gpu
def test_sglang_unpack_hook_serves_and_shapes():
    B, D, heads, hv = 5, 512, 8, 32
    zdim = heads * hv
    qkvz, ba, w, bias, st0 = _inputs(B, D, zdim, heads, 4, torch.bfloat16, torch.bfloat16, 9)
    idx = torch.tensor([3, 1, -1, 0, 8], device="cuda", dtype=torch.int32)
    called = []

    def original(*a, **k):
        called.append(1)

    st = st0.clone()
    out, z, b, a = sglang_compat.around_unpack(original, qkvz, ba, st, w, bias, idx, qkv_dim=D,
                                               v_dim=zdim, num_v_heads=heads, head_v_dim=hv,
                                               activation="silu")
    assert not called
    assert z.shape == (B, heads, hv) and b.shape == (B, heads) and a.shape == (B, heads)
    r = oracle.update_unpack(to_np(qkvz), to_np(ba), to_np(st0), to_np(w), to_np(bias), to_np(idx),
                             heads, True, PAD, "bf16")
    assert_close(out, r[0], torch.bfloat16)
    assert_bits(st, r[4])
    assert np.array_equal(to_np(z).reshape(B, -1), r[1])
