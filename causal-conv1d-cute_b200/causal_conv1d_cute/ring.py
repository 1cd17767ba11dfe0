"""Ring conv-state layout (drop-in for the reference's causal_conv1d_cute/ring.py).

A ring state keeps the last width - 1 inputs of every channel in a (slots, width - 1, dim) tensor
whose rows are not ordered by age: row cache_seqlens % (width - 1) holds the oldest input, and in
general row (cache_seqlens + k) % (width - 1) holds entry k (oldest first) of the ordered
(slots, dim, width - 1) state that prefill writes. A decode step (causal_conv1d_update_ring)
overwrites only the oldest row. to_ring and from_ring convert between the two layouts
(ring.py:33-67); both are index arithmetic on the slot axis, done with one advanced-indexing copy.
"""

import torch


def _rows(cache_seqlens, slots, K, device):
    """(slots, K) ring row of ordered entry k for every slot."""
    k = torch.arange(K, device=device)
    return (cache_seqlens.to(device=device, dtype=torch.long)[:, None] + k[None, :]) % K


def to_ring(conv_state, cache_seqlens):
    """Ordered (slots, dim, width - 1) state -> ring (slots, width - 1, dim) (ring.py:33-49)."""
    S, D, K = conv_state.shape
    rows = _rows(cache_seqlens, S, K, conv_state.device)
    ring = torch.empty((S, K, D), dtype=conv_state.dtype, device=conv_state.device)
    slot = torch.arange(S, device=conv_state.device)[:, None].expand(S, K)
    ring[slot, rows] = conv_state.transpose(1, 2)
    return ring


def from_ring(ring_state, cache_seqlens):
    """Ring (slots, width - 1, dim) state -> ordered (slots, dim, width - 1) (ring.py:52-67)."""
    S, K, D = ring_state.shape
    rows = _rows(cache_seqlens, S, K, ring_state.device)
    slot = torch.arange(S, device=ring_state.device)[:, None].expand(S, K)
    return ring_state[slot, rows].transpose(1, 2).contiguous()
