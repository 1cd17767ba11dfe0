"""Functional interface for depthwise causal conv1d on B200 (sm_100a) CUDA kernels.

Drop-in for the reference's causal_conv1d_cute.functional (functional.py:315-930): the same four
entry points with the same signatures, argument meaning, output shapes and strides, in-place cache
updates and ValueError cases, plus the support predicates (supported, varlen_reason,
update_reason) and the private helpers that the sglang and Dao-AILab shims call (_varlen,
_update, _int32).

One deliberate difference, required of this implementation: there is no PyTorch fallback. A call
the kernels cannot serve (a CPU tensor, a tensor that requires grad, a dtype other than
bf16/fp16/fp32, a kernel width outside 2..8) raises Unsupported instead of running slowly on
PyTorch operators. The kernels address arbitrary strides, so layouts and channel counts that the
reference sent to its fallback (dim not a multiple of 16, strided or unaligned views, conv states
longer than width - 1, short packed batches) run on the GPU here.
"""

import torch

from . import _ops
from .api import CausalConv1d

PAD_SLOT_ID = -1
MAX_STEPS = 16
_layers = {}
_MAX_LAYERS = 1024
_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


class Unsupported(NotImplementedError):
    """The call needs something the CUDA kernels do not provide (there is no CPU fallback)."""


def _unsupported(why):
    raise Unsupported(f"causal_conv1d_cute: {why}; the B200 kernels have no CPU fallback")


def _act(activation):
    """Normalize the activation argument (functional.py:21-37): "silu" or None."""
    if activation in ("silu", "swish") or activation is True:
        return "silu"
    if activation in (None, False):
        return None
    raise ValueError(f'activation must be None, "silu" or "swish", got {activation!r}')


def _layer(weight, bias, activation):
    """Return the cached CausalConv1d for (weight, bias, activation) (functional.py:40-62).

    Keyed on data pointer, shape, dtype and version counter, since callers pass a fresh view of
    the parameter on every call; an entry pins its tensors so the pointer cannot be reused.
    """
    key = (
        weight.data_ptr(),
        tuple(weight.shape),
        weight.dtype,
        weight._version,
        None if bias is None else (bias.data_ptr(), bias._version),
        activation,
    )
    hit = _layers.get(key)
    if hit is None:
        if len(_layers) >= _MAX_LAYERS:
            _layers.pop(next(iter(_layers)))
        hit = _layers[key] = (weight, bias, CausalConv1d(weight, bias, activation))
    return hit[2]


def _check(x, weight, bias, channel_dim):
    """Reject shapes inconsistent with a depthwise causal conv (functional.py:65-84)."""
    if weight.dim() != 2 or weight.shape[1] < 2:
        raise ValueError(f"weight must have shape (dim, width >= 2), got {tuple(weight.shape)}")
    D = weight.shape[0]
    if x.dim() <= channel_dim or x.shape[channel_dim] != D:
        raise ValueError(f"input shape {tuple(x.shape)} does not have {D} channels")
    if bias is not None and tuple(bias.shape) != (D,):
        raise ValueError(f"bias must have shape ({D},), got {tuple(bias.shape)}")


def _reason(x, weight, bias=None):
    """Return why the kernels cannot serve these tensors, or None (functional.py:87-115)."""
    D, W = weight.shape
    if torch.is_grad_enabled() and (
        x.requires_grad or weight.requires_grad or (bias is not None and bias.requires_grad)
    ):
        return "gradients are required and the kernels have no backward pass"
    if not x.is_cuda:
        return "input is not a CUDA tensor"
    if x.dtype not in _DTYPES:
        return f"dtype {x.dtype} is not bf16, fp16 or fp32"
    if weight.dtype != x.dtype or weight.device != x.device:
        return "weight must share the input dtype and device"
    if bias is not None and (bias.dtype != x.dtype or bias.device != x.device):
        return "bias must share the input dtype and device"
    if not 2 <= W <= 8:
        return f"kernel width {W} is outside 2..8"
    return None


def supported(x, weight, bias=None):
    """Whether the kernels serve x with these weights (functional.py:118-132)."""
    return _reason(x, weight, bias) is None


def _state_reason(conv_state, D, W, dtype, device=None, exact=True):
    """Why a conv-state cache cannot be served, or None (functional.py:135-153).

    exact: the state length must be width - 1; otherwise any length >= width - 1 is accepted
    (decode shifts the whole row, as the reference's fallback does).
    """
    K = W - 1
    if conv_state.dim() != 3 or conv_state.shape[1] != D:
        return f"conv state shape {tuple(conv_state.shape)} is not (slots, {D}, {K})"
    if conv_state.shape[2] < K or (exact and conv_state.shape[2] != K):
        return f"conv state shape {tuple(conv_state.shape)} is not (slots, {D}, {K})"
    if conv_state.dtype != dtype:
        return "conv state dtype differs from the input dtype"
    if device is not None and conv_state.device != device:
        return "conv state is on another device"
    return None


def _state_ok(conv_state, D, W, dtype):
    return _state_reason(conv_state, D, W, dtype) is None


def varlen_reason(x, weight, bias, query_start_loc, conv_states):
    """Why a packed (variable-length) call cannot be served, or None (functional.py:190-213)."""
    D, W = weight.shape
    if x.dim() != 2 or x.shape[0] != D:
        return f"input shape {tuple(x.shape)} is not ({D}, total_seqlen)"
    if query_start_loc is None or query_start_loc.dtype != torch.int32:
        return "query_start_loc must be an int32 tensor"
    why = _reason(x, weight, bias)
    if why is None and conv_states is not None:
        why = _state_reason(conv_states, D, W, x.dtype, x.device)
    return why


def varlen_supported(x, weight, bias, query_start_loc, conv_states):
    return varlen_reason(x, weight, bias, query_start_loc, conv_states) is None


def update_reason(x, conv_state, weight, bias, intermediate_conv_window=None):
    """Why a decode call cannot be served, or None (functional.py:234-271)."""
    D, W = weight.shape
    why = _reason(x, weight, bias) or _state_reason(
        conv_state, D, W, x.dtype, x.device, exact=False
    )
    if why is not None:
        return why
    if x.dim() == 2:
        if x.shape[1] != D:
            return f"input shape {tuple(x.shape)} is not (batch, {D})"
        if intermediate_conv_window is not None:
            return "per-token states need a (batch, dim, steps) input"
        return None
    if x.dim() != 3 or x.shape[1] != D:
        return f"input shape {tuple(x.shape)} is not (batch, {D}, steps)"
    L = x.shape[2]
    if not 1 <= L <= MAX_STEPS:
        return f"{L} steps is outside 1..{MAX_STEPS}"
    inter = intermediate_conv_window
    if inter is not None:
        if inter.device != x.device:
            return "per-token state cache is on another device"
        if _inter_layout(inter, D, W, L, x.dtype) is None:
            return f"per-token state shape {tuple(inter.shape)} strides {inter.stride()} unsupported"
    return None


def update_supported(x, conv_state, weight, bias):
    return update_reason(x, conv_state, weight, bias) is None


def _inter_layout(inter, D, W, L, dtype):
    """Classify a per-token state cache (functional.py:289-312): "dense", "dedup" or None.

    "dedup" is the overlapping view in which the state after token t starts t elements into a
    per-channel row of steps + width - 2 elements. Alignment is not required here: unaligned
    caches take the kernels' scalar path.
    """
    if inter.dim() != 4 or tuple(inter.shape[1:]) != (L, D, W - 1) or inter.dtype != dtype:
        return None
    PW = L + W - 2
    if inter.stride() == (D * PW, 1, PW, 1):
        return "dedup"
    if inter.is_contiguous():
        return "dense"
    return None


def _device(t, device):
    return t if t.device == device else t.to(device)


def _int32(index, device, nseq=1):
    """Slot indices as int32 on device; None stays None (the kernels then use slot i)."""
    if index is None:
        return None
    index = _device(index, device)
    return index if index.dtype == torch.int32 else index.to(torch.int32)


def _flags(flags, device, nseq=1):
    """Per-sequence initial-state flags as uint8 on device; None stays None (no initial state)."""
    if flags is None:
        return None
    flags = _device(flags, device)
    return flags.view(torch.uint8) if flags.dtype == torch.bool else flags.to(torch.uint8)


def causal_conv1d_fn(x, weight, bias=None, activation=None, out=None):
    """Causal 1D convolution over batched sequences (functional.py:315-347).

    Args:
        x: (batch, dim, seqlen), any strides; a (batch, dim, seqlen) view of (batch, seqlen, dim)
            storage (channel-last, token rows possibly wider than dim) is read in place.
        weight: (dim, width) filter weights, width 2..8.
        bias: optional (dim,) bias.
        activation: None, "silu" or "swish".
        out: optional (batch, dim, seqlen) output; must not share storage with x.

    Returns:
        (batch, dim, seqlen) output; for channel-last x it views (batch, seqlen, dim) storage.

    Raises:
        ValueError: inconsistent shapes, or out shares storage with x.
        Unsupported: the kernels cannot serve the call (see module docstring).
    """
    _check(x, weight, bias, 1)
    if x.dim() != 3:
        raise ValueError(f"input must have shape (batch, dim, seqlen), got {tuple(x.shape)}")
    act = _act(activation)
    why = _reason(x, weight, bias)
    if why is not None:
        _unsupported(why)
    return _layer(weight, bias, act).fwd(x, out=out)


def causal_conv1d_fwd_states(
    x,
    weight,
    bias=None,
    seq_idx=None,
    initial_states=None,
    return_final_states=False,
    final_states_out=None,
    activation=None,
):
    """Prefill with the Dao-AILab causal_conv1d_fn extras, which the reference's dao_compat shim
    passes upstream (dao_compat.py:28-78); upstream signature and results.

    Args:
        x: (batch, dim, seqlen), any strides.
        weight: (dim, width), width 2..8; bias: optional (dim,).
        seq_idx: optional int (batch, seqlen) sequence ids: a tap reaches back only to tokens of
            the same id (packed sequences inside one row). Excludes the two state arguments.
        initial_states: optional (batch, dim, width - 1): the inputs before token 0 of each row.
        return_final_states: also return the last width - 1 inputs of [initial_states | x] per
            row, (batch, dim, width - 1).
        final_states_out: optional (batch, dim, width - 1) tensor to write the final states to;
            must not overlap initial_states.
        activation: None, "silu" or "swish".

    Returns:
        out, or (out, final_states) with return_final_states. out has x's layout (as
        causal_conv1d_fn); allocated final states view (batch, width - 1, dim) storage, as
        upstream.

    Raises:
        ValueError: inconsistent shapes or dtypes, seq_idx with states, overlapping states.
        Unsupported: the kernels cannot serve the call.
    """
    _check(x, weight, bias, 1)
    if x.dim() != 3:
        raise ValueError(f"input must have shape (batch, dim, seqlen), got {tuple(x.shape)}")
    act = _act(activation)
    why = _reason(x, weight, bias)
    if why is None and initial_states is not None and torch.is_grad_enabled() and initial_states.requires_grad:
        why = "gradients are required and the kernels have no backward pass"
    if why is not None:
        _unsupported(why)
    B, D, L = x.shape
    K = weight.shape[1] - 1
    if seq_idx is not None:
        if initial_states is not None or return_final_states:
            raise ValueError("seq_idx excludes initial_states and return_final_states")
        if tuple(seq_idx.shape) != (B, L):
            raise ValueError(f"seq_idx must have shape {(B, L)}, got {tuple(seq_idx.shape)}")
        seq_idx = _int32(_device(seq_idx, x.device), x.device)
    for name, st in (("initial_states", initial_states), ("final_states_out", final_states_out)):
        if st is not None and (tuple(st.shape) != (B, D, K) or st.dtype != x.dtype or st.device != x.device):
            raise ValueError(f"{name} must be a {x.dtype} tensor of shape {(B, D, K)} on {x.device}")
    final = None
    if return_final_states:
        final = final_states_out
        if final is None:
            final = torch.empty((B, K, D), dtype=x.dtype, device=x.device).transpose(1, 2)
        elif initial_states is not None and (
            final.untyped_storage().data_ptr() == initial_states.untyped_storage().data_ptr()
        ):
            raise ValueError("final_states_out must not share storage with initial_states")
    if x.stride(1) == 1 and D > 1:
        out = torch.empty((B, L, D), dtype=x.dtype, device=x.device).transpose(1, 2)
    else:
        out = torch.empty((B, D, L), dtype=x.dtype, device=x.device)
    _ops.fwd_states(x, weight, bias, act, out, seq_idx, initial_states, final)
    return (out, final) if return_final_states else out


def causal_conv1d_varlen_fn(
    x,
    weight,
    bias=None,
    query_start_loc=None,
    cache_indices=None,
    has_initial_state=None,
    conv_states=None,
    activation=None,
    pad_slot_id=PAD_SLOT_ID,
):
    """Causal 1D convolution over a packed variable-length batch (functional.py:350-418).

    One kernel launch for any number of sequences. A (dim, total_seqlen) view of token-major
    storage (including the leading dim columns of a wider buffer) is read in place and the
    output views contiguous (total_seqlen, dim) storage; other layouts give a (dim, total_seqlen)
    contiguous output.

    Args:
        x: (dim, total_seqlen) packed input.
        weight: (dim, width) filter weights.
        bias: optional (dim,) bias.
        query_start_loc: int32 (batch + 1,) cumulative sequence lengths.
        cache_indices: optional (batch,) conv-state slot of each sequence (default: slot i).
        has_initial_state: optional (batch,) bool/uint8: start from the cached state.
        conv_states: optional (slots, dim, width - 1) cache, updated in place with the last
            width - 1 inputs of [initial state | sequence].
        activation: None, "silu" or "swish".
        pad_slot_id: cache_indices value marking sequences to skip (their outputs are
            undefined and their slots untouched).

    Returns:
        (dim, total_seqlen) output.
    """
    _check(x, weight, bias, 0)
    if x.dim() != 2 or query_start_loc is None:
        raise ValueError("a packed batch needs x of shape (dim, total_seqlen) and query_start_loc")
    why = varlen_reason(x, weight, bias, query_start_loc, conv_states)
    if why is not None:
        _unsupported(why)
    return _varlen(
        x,
        weight,
        bias,
        query_start_loc,
        cache_indices,
        has_initial_state,
        conv_states,
        activation,
        pad_slot_id,
    )


def _varlen(
    x,
    weight,
    bias,
    query_start_loc,
    cache_indices,
    has_initial_state,
    conv_states,
    activation,
    pad_slot_id,
):
    """Run causal_conv1d_varlen_fn on arguments varlen_reason() accepted (functional.py:421)."""
    D, T = x.shape
    act = _act(activation)
    dev = x.device
    if x.stride(0) == 1 and D > 1:
        out = torch.empty((T, D), dtype=x.dtype, device=dev).t()
    else:
        out = torch.empty((D, T), dtype=x.dtype, device=dev)
    qsl = _device(query_start_loc, dev)
    cidx = _int32(cache_indices, dev) if conv_states is not None else None
    hinit = _flags(has_initial_state, dev) if conv_states is not None else None
    return _ops.varlen(x, weight, bias, act, out, qsl, cidx, hinit, conv_states, pad_slot_id)


def causal_conv1d_update(
    x,
    conv_state,
    weight,
    bias=None,
    activation=None,
    conv_state_indices=None,
    pad_slot_id=PAD_SLOT_ID,
    intermediate_conv_window=None,
    intermediate_state_indices=None,
):
    """Advance the conv state by one or more tokens and compute their outputs
    (functional.py:711-785).

    Args:
        x: (batch, dim) for one token, or (batch, dim, steps) with 1 <= steps <= 16 for the
            multi-token step that verifies speculative drafts; any strides.
        conv_state: (slots, dim, state_len >= width - 1) cache, updated in place; the last
            width - 1 entries are the history and the row shifts left by steps.
        weight: (dim, width) filter weights.
        bias: optional (dim,) bias.
        activation: None, "silu" or "swish".
        conv_state_indices: optional int32 (batch,) slot of each row (default: row b, slot b).
        pad_slot_id: slot value marking rows to skip (state untouched, output undefined).
        intermediate_conv_window: optional (slots, steps, dim, width - 1) cache receiving the
            state after every token: contiguous, or the overlapping "dedup" view.
        intermediate_state_indices: optional int32 (batch,) slots of that cache (default:
            conv_state_indices).

    Returns:
        Output with the shape of x ((batch, dim), or (batch, dim, steps) viewing
        (batch, steps, dim) storage).
    """
    _check(x, weight, bias, 1)
    D, W = weight.shape
    if conv_state.dim() != 3 or conv_state.shape[1] != D or conv_state.shape[2] < W - 1:
        raise ValueError(
            f"conv_state shape {tuple(conv_state.shape)} is not (slots, {D}, >= {W - 1})"
        )
    why = update_reason(x, conv_state, weight, bias, intermediate_conv_window)
    if why is not None:
        _unsupported(why)
    return _update(
        x,
        conv_state,
        weight,
        bias,
        activation,
        conv_state_indices,
        pad_slot_id,
        intermediate_conv_window,
        intermediate_state_indices,
    )


def _update(
    x,
    conv_state,
    weight,
    bias,
    activation,
    conv_state_indices,
    pad_slot_id,
    intermediate_conv_window,
    intermediate_state_indices,
):
    """Run causal_conv1d_update on arguments update_reason() accepted (functional.py:788-858)."""
    D, W = weight.shape
    act = _act(activation)
    B = x.shape[0]
    dev = x.device
    single = x.dim() == 2
    x3 = x.unsqueeze(-1) if single else x
    L = x3.shape[2]
    if single:
        out = torch.empty((B, D), dtype=x.dtype, device=dev)
        out3 = out.unsqueeze(-1)
    else:
        out3 = torch.empty((B, L, D), dtype=x.dtype, device=dev).transpose(1, 2)
        out = out3
    idx = _int32(conv_state_indices, dev)
    if idx is None and conv_state.shape[0] < B:
        raise ValueError(
            f"conv_state has {conv_state.shape[0]} slots for {B} rows and no conv_state_indices"
        )
    inter = intermediate_conv_window
    iidx = _int32(intermediate_state_indices, dev) if inter is not None else None
    _ops.update(x3, conv_state, weight, bias, act, out3, idx, pad_slot_id, inter, iidx)
    return out


def causal_conv1d_update_ring(
    x,
    ring_state,
    weight,
    bias=None,
    activation=None,
    cache_seqlens=None,
    conv_state_indices=None,
    pad_slot_id=PAD_SLOT_ID,
):
    """Advance a ring conv state by one token (functional.py:861-930).

    The ring state (slots, width - 1, dim) is not shifted: the step overwrites row
    cache_seqlens % (width - 1), which holds the oldest input, and leaves the others in place.

    Args:
        x: (batch, dim) input.
        ring_state: (slots, width - 1, dim) ring cache, updated in place.
        weight: (dim, width) filter weights.
        bias: optional (dim,) bias.
        activation: None, "silu" or "swish".
        cache_seqlens: integer (batch,) tokens each sequence absorbed before this step; the
            caller increments it afterwards.
        conv_state_indices: optional int32 (batch,) slot of each row.
        pad_slot_id: slot value marking rows to skip.

    Returns:
        (batch, dim) output.
    """
    _check(x, weight, bias, 1)
    D, W = weight.shape
    if x.dim() != 2 or ring_state.dim() != 3 or tuple(ring_state.shape[1:]) != (W - 1, D):
        raise ValueError(
            f"need x (batch, {D}) and ring_state (slots, {W - 1}, {D}), got {tuple(x.shape)} and"
            f" {tuple(ring_state.shape)}"
        )
    if cache_seqlens is None or cache_seqlens.shape != (x.shape[0],):
        raise ValueError("cache_seqlens must be an integer tensor of shape (batch,)")
    act = _act(activation)
    why = _reason(x, weight, bias)
    if why is None and (ring_state.dtype != x.dtype or ring_state.device != x.device):
        why = "the ring state must share the input dtype and device"
    if why is not None:
        _unsupported(why)
    return _layer(weight, bias, act).update_ring(
        x, ring_state, cache_seqlens, conv_state_indices, pad_slot_id
    )
