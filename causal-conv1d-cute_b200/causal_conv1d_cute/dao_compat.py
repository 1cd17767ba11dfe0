"""Serve calls written against the Dao-AILab causal_conv1d interface with these kernels
(reference dao_compat.py:1-144).

mamba_ssm, flash-linear-attention and the fast paths of Hugging Face transformers call
``causal_conv1d.causal_conv1d_fn`` and ``causal_conv1d.causal_conv1d_update``. install() wraps both
and rebinds them in every module that already imported them. The wrappers keep the upstream
signatures and pass a call on to the upstream function whenever it needs something these kernels
do not provide: gradients, a circular state through cache_seqlens, a multi-token update, or
tensors the kernels cannot serve. seq_idx, initial_states and return_final_states / final_states_out
are served by causal_conv1d_fwd_states (the reference passes them upstream). stats counts both
outcomes.
"""

import torch

from . import _patch
from . import functional as fn

TARGETS_FN = ("causal_conv1d.causal_conv1d_interface.causal_conv1d_fn",)
TARGETS_UPDATE = ("causal_conv1d.causal_conv1d_interface.causal_conv1d_update",)
stats = {"fn_fast": 0, "fn_fallback": 0, "update_fast": 0, "update_fallback": 0}


def _needs_grad(*tensors):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def around_fn(
    original_fn,
    x,
    weight,
    bias=None,
    seq_idx=None,
    initial_states=None,
    return_final_states=False,
    final_states_out=None,
    activation=None,
):
    """Serve causal_conv1d_fn or pass the call upstream (dao_compat.py:28-78).

    Calls with seq_idx, initial_states or final states are served here too (the reference passes
    them upstream), unless they combine seq_idx with states, which upstream rejects.
    """
    served = (
        activation in (None, "silu", "swish")
        and x.dim() == 3
        and not _needs_grad(x, weight, bias, initial_states)
        and fn.supported(x, weight, bias)
        and not (seq_idx is not None and (initial_states is not None or return_final_states))
    )
    if not served:
        stats["fn_fallback"] += 1
        return original_fn(
            x,
            weight,
            bias,
            seq_idx=seq_idx,
            initial_states=initial_states,
            return_final_states=return_final_states,
            final_states_out=final_states_out,
            activation=activation,
        )
    stats["fn_fast"] += 1
    if seq_idx is None and initial_states is None and not return_final_states:
        return fn.causal_conv1d_fn(x, weight, bias, activation)
    return fn.causal_conv1d_fwd_states(
        x, weight, bias, seq_idx, initial_states, return_final_states, final_states_out, activation
    )


def around_update(
    original_fn,
    x,
    conv_state,
    weight,
    bias=None,
    activation=None,
    cache_seqlens=None,
    conv_state_indices=None,
):
    """Serve a single-token causal_conv1d_update or pass it upstream (dao_compat.py:81-127)."""
    served = (
        cache_seqlens is None
        and activation in (None, "silu", "swish")
        and x.dim() == 2
        and not _needs_grad(x, weight, bias)
        and fn.update_reason(x, conv_state, weight, bias) is None
    )
    if not served:
        stats["update_fallback"] += 1
        return original_fn(
            x,
            conv_state,
            weight,
            bias,
            activation=activation,
            cache_seqlens=cache_seqlens,
            conv_state_indices=conv_state_indices,
        )
    stats["update_fast"] += 1
    return fn._update(
        x, conv_state, weight, bias, activation, conv_state_indices, fn.PAD_SLOT_ID, None, None
    )


def install():
    """Wrap the upstream functions in this process; import the model code first. Idempotent.

    Returns:
        The number of rebound module attributes.
    """
    count = sum(_patch.wrap(t, around_fn) for t in TARGETS_FN)
    return count + sum(_patch.wrap(t, around_update) for t in TARGETS_UPDATE)
