"""Serve sglang's causal conv1d calls with these kernels (reference sglang_compat.py:1-431).

sglang reaches its conv kernels through causal_conv1d_fn (packed prefill), causal_conv1d_update
(decode and the multi-token speculative verify) and, for Gated DeltaNet decode without
speculation, a fused kernel that also unpacks Z, B and A from the projection rows. Each is
wrapped: a call these kernels can serve runs here, any other call goes unchanged to the wrapped
function, so installing the wrappers never removes functionality.

Install inside a server through the sglang.srt.plugins entry point plugin() (active only with
CAUSAL_CONV1D_CUTE_SGLANG=1), or in one process with install() after importing sglang.
CAUSAL_CONV1D_CUTE_SGLANG_PATHS selects a subset of "fn,update,unpack";
CAUSAL_CONV1D_CUTE_SGLANG_DRY_RUN=1 installs the wrappers but passes every call on.
Prefill calls with fewer than MIN_PREFILL_TOKENS tokens are passed on. Every packed prefill is a
single kernel launch, whatever the number of sequences.
"""

import logging
import os
import pkgutil

import torch

from . import _patch
from . import functional as fn
from . import unpack

PAD_SLOT_ID = fn.PAD_SLOT_ID
ENV_ENABLE = "CAUSAL_CONV1D_CUTE_SGLANG"
ENV_PATHS = "CAUSAL_CONV1D_CUTE_SGLANG_PATHS"
ENV_DRY_RUN = "CAUSAL_CONV1D_CUTE_SGLANG_DRY_RUN"
MIN_PREFILL_TOKENS = 16
TARGETS_FN = ("sglang.srt.layers.attention.mamba.causal_conv1d.causal_conv1d_fn",)
TARGETS_UPDATE = (
    "sglang.srt.layers.attention.mamba.causal_conv1d.causal_conv1d_update",
    "sglang.kernels.ops.mamba.causal_conv1d_triton.causal_conv1d_update",
)
TARGETS_UNPACK = (
    "sglang.kernels.ops.attention.triton_gdn_fused_proj.fused_qkvzba_causal_conv1d_update_contiguous",
)
TARGET_LOAD = "sglang.srt.model_executor.model_runner.ModelRunner.load_model"
stats = {k: 0 for k in ("fn_fast", "fn_fallback", "update_fast", "update_fallback",
                        "unpack_fast", "unpack_fallback")}
logger = logging.getLogger(__name__)
_seen = set()
# Decode keyword arguments that these kernels do not implement (tree drafts, circular states).
_UNSERVED = (
    "cache_seqlens",
    "num_accept_tokens",
    "retrieve_next_token",
    "retrieve_next_sibling",
    "retrieve_parent_token",
)


def _note(op, why, x):
    """Count a call and log the first of each kind, with the reason when it was passed on."""
    stats[f"{op}_{'fast' if why is None else 'fallback'}"] += 1
    key = (op, why, x.dim(), x.dtype)
    if key in _seen or len(_seen) >= 64:
        return
    _seen.add(key)
    verdict = "served" if why is None else f"passed on ({why})"
    logger.info("causal_conv1d_%s %s: input %s strides %s %s", op, verdict, tuple(x.shape),
                x.stride(), x.dtype)


def _dry_run():
    return os.environ.get(ENV_DRY_RUN, "0") == "1"


def around_fn(
    original_fn,
    x,
    weight,
    bias=None,
    query_start_loc=None,
    cache_indices=None,
    has_initial_state=None,
    conv_states=None,
    activation="silu",
    pad_slot_id=PAD_SLOT_ID,
    **kwargs,
):
    """Serve a packed prefill call or pass it to the wrapped function (sglang_compat.py:91-156)."""
    if activation not in (None, "silu", "swish"):
        why = "activation"
    elif x.dim() == 2 and x.shape[1] < MIN_PREFILL_TOKENS:
        why = f"fewer than {MIN_PREFILL_TOKENS} tokens"
    else:
        why = fn.varlen_reason(x, weight, bias, query_start_loc, conv_states)
    if why is None and _dry_run():
        why = "dry run"
    _note("fn", why, x)
    if why is not None:
        return original_fn(
            x,
            weight,
            bias,
            query_start_loc=query_start_loc,
            cache_indices=cache_indices,
            has_initial_state=has_initial_state,
            conv_states=conv_states,
            activation=activation,
            pad_slot_id=pad_slot_id,
            **kwargs,
        )
    return fn._varlen(x, weight, bias, query_start_loc, cache_indices, has_initial_state,
                      conv_states, activation, pad_slot_id)


def around_update(
    original_fn,
    x,
    conv_state,
    weight,
    bias=None,
    activation=None,
    *args,
    conv_state_indices=None,
    intermediate_conv_window=None,
    intermediate_state_indices=None,
    pad_slot_id=PAD_SLOT_ID,
    **kwargs,
):
    """Serve a decode or speculative-verify call or pass it on (sglang_compat.py:159-242)."""
    if args:
        why = "positional arguments after activation"
    elif any(kwargs.get(k) is not None for k in _UNSERVED):
        why = "uses " + ", ".join(k for k in _UNSERVED if kwargs.get(k) is not None)
    elif isinstance(activation, str) and activation not in ("silu", "swish"):
        why = "activation"
    else:
        why = fn.update_reason(x, conv_state, weight, bias, intermediate_conv_window)
    if why is None and _dry_run():
        why = "dry run"
    _note("update", why, x)
    if why is not None:
        extra = {}
        if intermediate_conv_window is not None:
            extra = {
                "intermediate_conv_window": intermediate_conv_window,
                "intermediate_state_indices": intermediate_state_indices,
            }
        return original_fn(x, conv_state, weight, bias, activation, *args,
                           conv_state_indices=conv_state_indices, pad_slot_id=pad_slot_id,
                           **extra, **kwargs)
    return fn._update(x, conv_state, weight, bias, activation, conv_state_indices, pad_slot_id,
                      intermediate_conv_window, intermediate_state_indices)


def around_unpack(
    original_fn,
    mixed_qkvz,
    mixed_ba,
    conv_state,
    conv_weight,
    conv_bias,
    conv_state_indices,
    *,
    qkv_dim,
    v_dim,
    num_v_heads,
    head_v_dim,
    activation,
    pad_slot_id=PAD_SLOT_ID,
):
    """Serve the fused Gated DeltaNet decode or pass it on (sglang_compat.py:245-326).

    Returns:
        (conv out (batch, qkv_dim), Z (batch, num_v_heads, head_v_dim), B (batch, num_v_heads),
        A (batch, num_v_heads)).
    """
    if activation not in (None, "silu", "swish"):
        why = "activation"
    elif conv_weight.dim() != 2 or mixed_qkvz.dim() != 2 or mixed_ba.dim() != 2:
        why = "tensor ranks"
    elif mixed_qkvz.shape[1] != qkv_dim + v_dim or v_dim != num_v_heads * head_v_dim:
        why = "projection layout"
    elif conv_weight.shape[0] != qkv_dim or conv_state_indices.shape[0] != mixed_qkvz.shape[0]:
        why = "shapes"
    else:
        why = unpack.unpack_reason(mixed_qkvz, mixed_ba, conv_state, conv_weight, conv_bias,
                                   num_v_heads)
    if why is None and _dry_run():
        why = "dry run"
    _note("unpack", why, mixed_qkvz)
    if why is not None:
        return original_fn(
            mixed_qkvz,
            mixed_ba,
            conv_state,
            conv_weight,
            conv_bias,
            conv_state_indices,
            qkv_dim=qkv_dim,
            v_dim=v_dim,
            num_v_heads=num_v_heads,
            head_v_dim=head_v_dim,
            activation=activation,
            pad_slot_id=pad_slot_id,
        )
    batch = mixed_qkvz.shape[0]
    out, z, b, a = unpack.causal_conv1d_update_unpack(
        mixed_qkvz,
        mixed_ba,
        conv_state,
        conv_weight,
        conv_bias,
        fn._int32(conv_state_indices, mixed_qkvz.device),
        num_v_heads,
        None if activation is None else "silu",
        int(pad_slot_id),
    )
    return (out, z.view(batch, num_v_heads, head_v_dim), b, a)


def after_load_model(result, runner, *args, **kwargs):
    """AFTER hook on ModelRunner.load_model (sglang_compat.py:340-376).

    The reference packs the weights of layers its kernels cannot read in place here, before
    sglang sizes its memory pools. These kernels read every layer's (dim, width) weights and
    bias in place, so nothing is allocated; the hook only counts the conv layers it finds.
    """
    count = 0
    model = getattr(runner, "model", None)
    for module in (model.modules() if model is not None else ()):
        weights = getattr(module, "conv_weights", None)
        if isinstance(weights, torch.Tensor):
            weights = (weights,)
        if isinstance(weights, (tuple, list)):
            count += sum(isinstance(w, torch.Tensor) and w.dim() == 2 for w in weights)
    logger.info("causal-conv1d-cute: %d conv layers read their weights in place", count)
    return result


def _present(target):
    """Whether the function or method at a dotted path exists in the installed sglang."""
    try:
        pkgutil.resolve_name(target)
    except (ImportError, AttributeError, ValueError):
        return False
    return True


def _wrappers():
    """(target, wrapper) pairs selected by CAUSAL_CONV1D_CUTE_SGLANG_PATHS (default: all)."""
    paths = set(os.environ.get(ENV_PATHS, "fn,update,unpack").split(","))
    pairs = []
    if "fn" in paths:
        pairs += [(t, around_fn) for t in TARGETS_FN]
    if "update" in paths:
        pairs += [(t, around_update) for t in TARGETS_UPDATE]
    if "unpack" in paths:
        pairs += [(t, around_unpack) for t in TARGETS_UNPACK if _present(t)]
    return pairs


def plugin():
    """sglang.srt.plugins entry point: register the wrappers as AROUND hooks in every scheduler
    process when CAUSAL_CONV1D_CUTE_SGLANG=1 (sglang_compat.py:402-417)."""
    if os.environ.get(ENV_ENABLE, "0") != "1":
        return
    from sglang.srt.plugins.hook_registry import HookRegistry, HookType

    pairs = _wrappers()
    for target, hook in pairs:
        HookRegistry.register(target, hook, HookType.AROUND)
    if pairs and _present(TARGET_LOAD):
        HookRegistry.register(TARGET_LOAD, after_load_model, HookType.AFTER)
    logger.info("causal-conv1d-cute: wrapping %d sglang conv entry points", len(pairs))


def install():
    """Wrap the sglang entry points in this process (idempotent); returns the rebind count."""
    return sum(_patch.wrap(target, hook) for target, hook in _wrappers())
