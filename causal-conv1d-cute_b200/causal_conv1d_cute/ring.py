"""Ring conv-state layout (drop-in for the reference's causal_conv1d_cute/ring.py).

A ring state keeps the last width - 1 inputs of every channel in a (slots, width - 1, dim) tensor
whose rows are not ordered by age: row cache_seqlens % (width - 1) holds the oldest input, and in
general row (cache_seqlens + k) % (width - 1) holds entry k (oldest first) of the ordered
(slots, dim, width - 1) state that prefill writes. A decode step (causal_conv1d_update_ring)
overwrites only the oldest row. to_ring and from_ring convert between the two layouts
(ring.py:33-67) with one CUDA kernel each (cc1d_to_ring / cc1d_from_ring); the reference uses
torch gathers.
"""

import torch

from . import _ops
from .functional import _unsupported

_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def _check(t, seen, what):
    if t.dim() != 3:
        raise ValueError(f"{what} must be 3-D, got shape {tuple(t.shape)}")
    if seen.dim() != 1 or seen.shape[0] != t.shape[0]:
        raise ValueError(f"cache_seqlens must have shape ({t.shape[0]},), got {tuple(seen.shape)}")
    if not t.is_cuda:
        _unsupported(f"{what} is not a CUDA tensor")
    if t.dtype not in _DTYPES:
        _unsupported(f"dtype {t.dtype} is not bf16, fp16 or fp32")
    return seen.to(device=t.device, dtype=torch.int32)


def to_ring(conv_state, cache_seqlens):
    """Ordered (slots, dim, width - 1) state -> ring (slots, width - 1, dim) (ring.py:33-49).

    Args:
        conv_state: (slots, dim, width - 1), width 2..8, any strides.
        cache_seqlens: integer (slots,) tokens absorbed per slot.

    Returns:
        A new contiguous (slots, width - 1, dim) ring state.
    """
    seen = _check(conv_state, cache_seqlens, "conv_state")
    S, D, K = conv_state.shape
    if not 1 <= K <= 7:
        _unsupported(f"state length {K} is outside 1..7")
    ring = torch.empty((S, K, D), dtype=conv_state.dtype, device=conv_state.device)
    _ops.to_ring(conv_state, ring, seen)
    return ring


def from_ring(ring_state, cache_seqlens):
    """Ring (slots, width - 1, dim) state -> ordered (slots, dim, width - 1) (ring.py:52-67).

    Returns:
        A new contiguous (slots, dim, width - 1) ordered state.
    """
    seen = _check(ring_state, cache_seqlens, "ring_state")
    S, K, D = ring_state.shape
    if not 1 <= K <= 7:
        _unsupported(f"state length {K} is outside 1..7")
    state = torch.empty((S, D, K), dtype=ring_state.dtype, device=ring_state.device)
    _ops.from_ring(ring_state, state, seen)
    return state
