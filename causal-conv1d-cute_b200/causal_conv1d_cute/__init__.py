"""Depthwise causal 1D convolution on B200 (sm_100a): drop-in for causal_conv1d_cute.

Public API (same names and signatures as the reference package):
  causal_conv1d_fn          prefill over dense batched sequences
  causal_conv1d_update      decode of one or more tokens against an indexed conv-state cache,
                            with optional per-step state recording for speculative decoding
  causal_conv1d_update_ring single-token decode on a ring conv state; to_ring / from_ring convert
  causal_conv1d_varlen_fn   packed variable-length prefill with an in-place conv-state cache
  supported                 whether the kernels serve a call

Beyond the reference:
  causal_conv1d_fwd_states  prefill with the Dao-AILab extras (seq_idx, initial_states, final
                            states), which dao_compat serves instead of passing them upstream
  CausalConv1d              layer object

Every entry point runs hand-written CUDA kernels from libcc1d.so (C ABI: include/cc1d.h). There is
no CPU fallback: calls the kernels cannot serve raise functional.Unsupported.
"""

__version__ = "0.1.0+b200"

from ._ops import device_status, set_device_checks
from .api import CausalConv1d
from .functional import (
    Unsupported,
    causal_conv1d_fn,
    causal_conv1d_fwd_states,
    causal_conv1d_update,
    causal_conv1d_update_ring,
    causal_conv1d_varlen_fn,
    supported,
)
from .ring import from_ring, to_ring

__all__ = [
    "CausalConv1d",
    "Unsupported",
    "causal_conv1d_fn",
    "causal_conv1d_fwd_states",
    "causal_conv1d_update",
    "causal_conv1d_update_ring",
    "causal_conv1d_varlen_fn",
    "device_status",
    "from_ring",
    "set_device_checks",
    "supported",
    "to_ring",
]
