"""Prefill (causal_conv1d_fn) on the GPU against the oracle and the fp32 accuracy classifier.
Mirrors the reference's tests/test_prefill.py and adds the layouts this library serves in place."""

import pytest
import torch

import oracle
from _util import TAG, assert_close, to_np
from causal_conv1d_cute import CausalConv1d, causal_conv1d_fn
from causal_conv1d_cute import testing as T

SHAPES = [(1, 16), (1, 17), (3, 33), (2, 1000), (1, 2047), (2, 512)]


def _run(case, seed=0):
    t = T.make_inputs(case, seed)
    out = causal_conv1d_fn(t["x"], t["w"], t["b"], case.act)
    torch.cuda.synchronize()
    ref = oracle.fwd(to_np(t["x"]), to_np(t["w"]), to_np(t["b"]), case.act is not None, TAG[case.dtype])
    assert_close(out, ref, case.dtype)
    return T.check(case, t, out, T.reference(case, t)), out, t


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["bdl", "btd"])
@pytest.mark.parametrize("act", [None, "silu"])
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("W", [2, 3, 4, 5, 6, 7, 8])
def test_all_widths(W, bias, act, layout):
    for B, L in SHAPES:
        (status, _, bwd), out, t = _run(T.Case("t", "fwd", 64, W, B, L, bias, act, layout))
        assert status == "ok", (B, L, status, bwd)
        assert out.shape == t["x"].shape
        if layout == "btd":
            assert out.transpose(1, 2).is_contiguous()


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["bdl", "btd"])
@pytest.mark.parametrize(
    "D,W,bias,act", [(1536, 7, True, None), (2048, 3, False, None), (2048, 4, False, "silu")]
)
def test_real_shapes(D, W, bias, act, layout):
    for B, L in SHAPES:
        (status, _, bwd), _, _ = _run(T.Case("t", "fwd", D, W, B, L, bias, act, layout))
        assert status == "ok", (B, L, status, bwd)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("layout", ["bdl", "btd"])
def test_other_dtypes(dtype, layout):
    (status, _, bwd), _, _ = _run(T.Case("t", "fwd", 1536, 7, 2, 512, True, "silu", layout, dtype))
    assert status == "ok", (status, bwd)


@pytest.mark.gpu
@pytest.mark.parametrize("extra", [16, 6144, 8, 1])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_channel_last_rows_of_wider_buffer(extra, W):
    """x = leading D columns of (B, L, D + extra) storage: read in place, equal to a copy.
    extra = 1 gives rows that are not 16-byte aligned (scalar path)."""
    torch.manual_seed(extra + W)
    B, L, D = 2, 333, 256
    wide = torch.randn(B, L, D + extra, device="cuda", dtype=torch.bfloat16)
    x = wide[:, :, :D].transpose(1, 2)
    w = torch.rand(D, W, device="cuda", dtype=torch.bfloat16) - 0.5
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16) * 0.1
    keep = wide.clone()
    y = causal_conv1d_fn(x, w, b, "silu")
    r = causal_conv1d_fn(x.contiguous(), w, b, "silu")
    torch.cuda.synchronize()
    assert torch.equal(wide, keep)
    assert torch.equal(y, r)


@pytest.mark.gpu
@pytest.mark.parametrize("D,W", [(100, 4), (24, 2), (40, 8), (1, 3)])
@pytest.mark.parametrize("layout", ["bdl", "btd"])
def test_channel_counts_the_reference_sent_to_pytorch(D, W, layout):
    torch.manual_seed(D)
    x = torch.randn(2, 40, D, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    if layout == "bdl":
        x = x.contiguous()
    w = torch.randn(D, W, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(D, device="cuda", dtype=torch.bfloat16)
    y = causal_conv1d_fn(x, w, b, "silu")
    ref = oracle.fwd(to_np(x), to_np(w), to_np(b), True, "bf16")
    assert_close(y, ref, torch.bfloat16)


@pytest.mark.gpu
def test_strided_and_unaligned_inputs():
    torch.manual_seed(0)
    base = torch.randn(2, 64, 97, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(64, 4, device="cuda", dtype=torch.bfloat16)
    for x in (base[:, :, ::2], base[:, :, 1:], base[:, :, 1:].transpose(1, 2).contiguous().transpose(1, 2)):
        y = causal_conv1d_fn(x, w, None, None)
        ref = oracle.fwd(to_np(x), to_np(w), None, False, "bf16")
        assert_close(y, ref, torch.bfloat16)
    # Non-contiguous weights and a strided bias are read through their strides.
    wt = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16).t()
    bb = torch.randn(128, device="cuda", dtype=torch.bfloat16)[::2]
    x = base[:, :, :64]
    y = causal_conv1d_fn(x, wt, bb, "silu")
    assert_close(y, oracle.fwd(to_np(x), to_np(wt), to_np(bb), True, "bf16"), torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("S", [2, 3, 4, 5, 8])
def test_short_sequences_stay_in_bounds(S):
    """Sequences shorter than the strip and than W - 1 (reference test_prefill.py:44-53)."""
    case = T.Case("t", "fwd", 1536, 7, 3, S, True, None, "btd")
    (status, _, _), _, _ = _run(case)
    assert status == "ok"


@pytest.mark.gpu
def test_out_argument_and_in_place_refused():
    case = T.Case("t", "fwd", 64, 4, 1, 64, False, None, "bdl")
    t = T.make_inputs(case)
    with pytest.raises(ValueError):
        CausalConv1d(t["w"], None, None).fwd(t["x"], out=t["x"])
    out = torch.empty_like(t["x"])
    y = causal_conv1d_fn(t["x"], t["w"], None, None, out=out)
    assert y is out
    assert T.check(case, t, out, T.reference(case, t))[0] == "ok"


@pytest.mark.gpu
def test_repeat_is_deterministic():
    case = T.Case("t", "fwd", 8192, 4, 2, 1000, True, "silu", "btd")
    t = T.make_inputs(case)
    first = causal_conv1d_fn(t["x"], t["w"], t["b"], "silu")
    for _ in range(5):
        assert torch.equal(causal_conv1d_fn(t["x"], t["w"], t["b"], "silu"), first)
