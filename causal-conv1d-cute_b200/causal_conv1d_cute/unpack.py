"""Fused Gated DeltaNet decode step (drop-in for the reference's causal_conv1d_cute/unpack.py).

Gated DeltaNet layers project the hidden state into a [Q | K | V | Z] row and a [B | A] row. One
decode step needs a conv-state update over the leading Q, K, V columns plus contiguous copies of
Z, B and A for later kernels. causal_conv1d_update_unpack does all of it in one launch
(cc1d_update_unpack), reading the conv input, the filter weights and the bias in place.
"""

import torch

from . import _ops

_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def _aligned(t):
    return t.data_ptr() % 16 == 0


def unpack_reason(qkvz, ba, conv_state, weight, bias, heads):
    """Why a fused decode call cannot be served, or None (unpack.py:289-325).

    Args:
        qkvz: (batch, dim + zdim) projection rows; the conv reads the leading dim columns.
        ba: (batch, 2 * heads) projection rows.
        conv_state: (slots, dim, width - 1) cache.
        weight: (dim, width) filter weights.
        bias: optional (dim,) bias.
        heads: width of B and of A.
    """
    D, W = weight.shape
    zdim = qkvz.shape[1] - D
    if torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (qkvz, ba, weight, bias)
    ):
        return "gradients are required"
    if not (qkvz.is_cuda and ba.is_cuda and conv_state.is_cuda and weight.is_cuda):
        return "tensors are not on a CUDA device"
    if qkvz.dtype not in _DTYPES or ba.dtype not in _DTYPES or weight.dtype != qkvz.dtype:
        return f"dtypes {qkvz.dtype}, {ba.dtype}, {weight.dtype}"
    vec = 16 // qkvz.element_size()
    if not 2 <= W <= 8 or D % vec or zdim <= 0 or zdim % vec:
        return f"conv of {D} channels and width {W} with {zdim} further columns"
    if qkvz.stride(1) != 1 or ba.stride(1) != 1 or (qkvz.stride(0) * qkvz.element_size()) % 16:
        return f"projection strides {qkvz.stride()}, {ba.stride()}"
    if ba.shape[1] != 2 * heads or ba.shape[0] != qkvz.shape[0]:
        return f"{heads} heads with [B|A] rows of shape {tuple(ba.shape)}"
    if conv_state.dtype != qkvz.dtype or tuple(conv_state.shape[1:]) != (D, W - 1):
        return f"conv state {tuple(conv_state.shape)} {conv_state.dtype}"
    if not conv_state.is_contiguous() or not weight.is_contiguous():
        return "conv state or weight is not contiguous"
    if bias is not None and (bias.dtype != weight.dtype or bias.stride(0) != 1):
        return "bias dtype or stride"
    tensors = [qkvz, conv_state, weight] + ([] if bias is None else [bias])
    if not all(_aligned(t) for t in tensors) or ba.data_ptr() % ba.element_size():
        return "tensors are not aligned to 16 bytes"
    if qkvz.shape[0] > 65535:
        return "more than 65535 rows"
    return None


def causal_conv1d_update_unpack(
    qkvz, ba, conv_state, weight, bias, conv_state_indices, heads, activation, pad, vec=None, bs=None
):
    """Advance an indexed conv state by one token and unpack Z, B and A (unpack.py:328-374).

    Args:
        qkvz: (batch, dim + zdim) rows; the conv reads the leading dim columns in place.
        ba: (batch, 2 * heads) rows.
        conv_state: (slots, dim, width - 1) cache, updated in place.
        weight: (dim, width) contiguous filter weights, read in place.
        bias: optional (dim,) bias.
        conv_state_indices: int32 (batch,) slot of each row; rows whose slot is pad or outside
            the cache keep their state and get their conv input copied to the output.
        heads: width of B and of A.
        activation: "silu" or None.
        pad: pad slot id.
        vec, bs: accepted for signature compatibility (the library picks the launch shape).

    Returns:
        (out (batch, dim), z (batch, zdim), b (batch, heads), a (batch, heads)).
    """
    B = qkvz.shape[0]
    D = weight.shape[0]
    zdim = qkvz.shape[1] - D
    dev = qkvz.device
    out = torch.empty((B, D), dtype=qkvz.dtype, device=dev)
    z = torch.empty((B, zdim), dtype=qkvz.dtype, device=dev)
    b = torch.empty((B, heads), dtype=ba.dtype, device=dev)
    a = torch.empty_like(b)
    idx = conv_state_indices
    if idx.device != dev:
        idx = idx.to(dev)
    if idx.dtype != torch.int32:
        idx = idx.to(torch.int32)
    return _ops.update_unpack(qkvz, ba, conv_state, weight, bias, out, z, b, a, idx, heads,
                              activation is not None, pad)


def unpack_config(dim, batch, stride):
    """Launch shape of the reference's fused kernel (unpack.py:377-401), kept for callers that
    pass it through; this library chooses its own launch shape and ignores the value."""
    vec = 16
    while stride % vec:
        vec //= 2
    return (vec, 32)
