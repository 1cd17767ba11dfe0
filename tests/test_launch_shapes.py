"""Shapes that reach each launch form of the token-row walks.

For 16-bit types up to W = 5 the channel-last prefill and the token-major varlen kernels run as
staged 16-token strips (one per CTA, landed in shared memory); the cases below include partial last
strips, partial channel blocks and, for varlen, sequence starts at every offset inside a strip,
sequences shorter than W - 1 and heads that run past a strip end. Wider filters and fp32 take the
register walks, either as fixed strips over several waves or as one wave of balanced shares, chosen
on the host from the width, the sequence lengths and the GPU's resident-CTA count (the fp32 runs of
the prefill cases reach those for W <= 5). These cases sit on both sides of that choice, with shares
that cross batch and sequence boundaries and a partial last channel block, and check that the
result is bit-identical to the scalar path (the same arithmetic in the same order, reached by
viewing rows of a wider buffer that are not 16-byte aligned), and, for a small case, to the oracle.
From W = 5 the 16-bit walks give each thread 4 channels (8-byte vectors); the W = 5..8 cases, with
channel counts that leave a partial last CTA of 64 or 128 threads, cover that form.
"""

import numpy as np
import pytest
import torch

import oracle
from _util import assert_bits, assert_close, to_np
from causal_conv1d_cute import causal_conv1d_fn, causal_conv1d_varlen_fn

PAD = -1

# (B, L, D, W): W = 2 strips over many CTAs; short sequences (one strip each, enough CTAs);
# balanced shares crossing batch boundaries; shares with a partial channel block; long shares;
# half-width walks (W >= 5) with partial 128- and 64-thread channel blocks.
FWD_SHAPES = [
    (8, 1000, 8192, 2),
    (64, 100, 4096, 4),
    (5, 37, 512, 4),
    (3, 1000, 2304, 8),
    (2, 5000, 1024, 3),
    (1, 17, 64, 6),
    (2, 700, 1000, 5),
    (3, 333, 776, 7),
]


def _unaligned_view(t, D):
    """(B, L, D) tensor -> a view with the same values whose rows are 2 bytes past 16-byte lines."""
    B, L, _ = t.shape
    wide = torch.empty(B, L, D + 1, device=t.device, dtype=t.dtype)
    v = wide[:, :, 1:]
    v.copy_(t)
    return v


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,L,D,W", FWD_SHAPES)
def test_prefill_launch_forms_match_scalar_path(B, L, D, W, dtype):
    g = torch.Generator(device="cuda").manual_seed(B * 7919 + L * 31 + W)
    x = torch.randn(B, L, D, device="cuda", generator=g).to(dtype)
    w = (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(dtype)
    b = (torch.randn(D, device="cuda", generator=g) * 0.1).to(dtype)
    y = causal_conv1d_fn(x.transpose(1, 2), w, b, "silu")
    ys = causal_conv1d_fn(_unaligned_view(x, D).transpose(1, 2), w, b, "silu")
    torch.cuda.synchronize()
    assert torch.equal(y, ys)
    if B * L * D <= 1 << 20:
        name = "bf16" if dtype == torch.bfloat16 else "f32"
        ref = oracle.fwd(to_np(x.transpose(1, 2)), to_np(w), to_np(b), True, name)
        assert_close(y, ref, dtype)


# (lengths, D, W): many short sequences (strips at W = 2), lognormal lengths with balanced shares
# at W = 3 and 8, and sequences shorter than W - 1 inside a share.
def _lengths(seed, n, mean):
    rng = np.random.default_rng(seed)
    return [int(v) for v in np.clip(np.round(rng.lognormal(mean, 1.0, n)), 1, 6000)]


VARLEN_CASES = [
    (_lengths(1, 400, 4.0), 2048, 2),
    (_lengths(2, 32, 7.0), 512, 3),
    (_lengths(3, 32, 7.0), 768, 8),
    ([1, 2, 3, 0, 9, 1, 700, 2, 5], 1024, 8),
    (_lengths(4, 20, 6.0), 1000, 5),
    (_lengths(5, 12, 6.5), 776, 6),
    # staged strips: starts at every offset of a 16-token strip, sequences shorter than W - 1,
    # heads past a strip end, a partial last strip (T = 79) and a partial channel block (D = 520)
    ([1, 2, 3, 13, 15, 16, 17, 1, 31, 2, 3, 45, 14, 18, 7, 4, 5, 6, 8, 9, 10, 11, 12], 512, 4),
    ([5, 11, 16, 1, 1, 1, 40, 3, 29, 2, 14, 0, 17], 520, 5),
    ([15, 17, 33, 14], 256, 3),
    (_lengths(6, 60, 2.5), 1024, 2),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(VARLEN_CASES)))
def test_varlen_launch_forms_match_scalar_path(case):
    lens, D, W = VARLEN_CASES[case]
    K, nseq = W - 1, len(lens)
    g = torch.Generator(device="cuda").manual_seed(case)
    qsl = torch.tensor([0] + list(np.cumsum(lens)), device="cuda", dtype=torch.int32)
    T = int(qsl[-1])
    slots = nseq + 2
    cidx = torch.randperm(slots, device="cuda", generator=g)[:nseq].to(torch.int32)
    cidx[::7] = PAD
    hinit = torch.rand(nseq, device="cuda", generator=g) < 0.5
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(torch.bfloat16)
    st0 = torch.randn(slots, D, K, device="cuda", dtype=torch.bfloat16, generator=g)
    st = st0.clone()
    y = causal_conv1d_varlen_fn(x.t(), w, None, qsl, cidx, hinit, st, "silu")
    sts = st0.clone()
    xs = _unaligned_view(x.unsqueeze(0), D)[0]
    ys = causal_conv1d_varlen_fn(xs.t(), w, None, qsl, cidx, hinit, sts, "silu")
    torch.cuda.synchronize()
    assert torch.equal(y, ys)
    assert torch.equal(st, sts)
    if T * D <= 1 << 21:
        r_out, r_st = oracle.varlen(to_np(x.t()), to_np(w), None, to_np(qsl), to_np(cidx),
                                    to_np(hinit), to_np(st0), True, PAD, "bf16")
        mask = ~np.isnan(r_out)
        assert_close(to_np(y), np.nan_to_num(r_out), torch.bfloat16, mask)
        assert_bits(st, r_st)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_channel_first_prefill_16_byte_aligned_stream(dtype):
    """Contiguous (B, D, L) storage starting 16 bytes past a 32-byte line takes the 16-byte access
    variant of the flat-stream kernel; it must equal the 32-byte variant bit for bit."""
    B, D, L, W = 2, 96, 1000, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(B, D, L, device="cuda", generator=g).to(dtype)
    w = (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(dtype)
    off = 16 // x.element_size()
    buf = torch.empty(B * D * L + off, device="cuda", dtype=dtype)
    xs = buf[off:].view(B, D, L)
    xs.copy_(x)
    assert xs.data_ptr() % 32 == 16
    y = causal_conv1d_fn(x, w, None, "silu")
    ys = causal_conv1d_fn(xs, w, None, "silu")
    torch.cuda.synchronize()
    assert torch.equal(y, ys)


@pytest.mark.gpu
@pytest.mark.parametrize("W", [3, 4, 6, 8])
def test_strided_weights_take_the_register_walk(W):
    """The staged kernels read the contiguous (dim, W) weights and a contiguous bias; strided views
    of them go to the register walks, which must give the same bits (prefill, prefill with
    states, token-major varlen)."""
    from causal_conv1d_cute import causal_conv1d_fwd_states

    B, L, D, K = 2, 300, 1024, W - 1
    g = torch.Generator(device="cuda").manual_seed(W)
    x = torch.randn(B, L, D, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.rand(D, W, device="cuda", generator=g) - 0.5).to(torch.bfloat16)
    b = (torch.randn(D, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    wide_w = torch.zeros(D, W + 1, device="cuda", dtype=torch.bfloat16)
    wide_w[:, :W] = w
    wide_b = torch.zeros(D, 2, device="cuda", dtype=torch.bfloat16)
    wide_b[:, 0] = b
    ws, bs = wide_w[:, :W], wide_b[:, 0]
    assert not ws.is_contiguous() and not bs.is_contiguous()
    xv = x.transpose(1, 2)
    assert torch.equal(causal_conv1d_fn(xv, w, b, "silu"), causal_conv1d_fn(xv, ws, bs, "silu"))
    init = torch.randn(B, K, D, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
    y1, f1 = causal_conv1d_fwd_states(xv, w, b, None, init, True, None, "silu")
    y2, f2 = causal_conv1d_fwd_states(xv, ws, bs, None, init, True, None, "silu")
    assert torch.equal(y1, y2) and torch.equal(f1, f2)
    qsl = torch.tensor([0, 5, 133, 290, 600], device="cuda", dtype=torch.int32)
    xt = x.reshape(B * L, D)
    st0 = torch.randn(6, D, K, device="cuda", generator=g).to(torch.bfloat16)
    cidx = torch.tensor([4, 0, 2, 5], device="cuda", dtype=torch.int32)
    hinit = torch.tensor([True, False, True, True], device="cuda")
    s1, s2 = st0.clone(), st0.clone()
    v1 = causal_conv1d_varlen_fn(xt.t(), w, b, qsl, cidx, hinit, s1, "silu")
    v2 = causal_conv1d_varlen_fn(xt.t(), ws, bs, qsl, cidx, hinit, s2, "silu")
    torch.cuda.synchronize()
    assert torch.equal(v1, v2) and torch.equal(s1, s2)
