"""Layer object and dispatch (drop-in for the reference's causal_conv1d_cute/api.py).

The reference chooses a CuTe kernel configuration per call from tuned.json, keyed by
architecture, falling back to heuristics (api.py:19-183). Here the choice is made inside
libcc1d.so from the tensor layout (the sm_100 launch table in csrc/*.cu), so this module keeps
only the layer object: the filter weights are read in place by every kernel and no packed copy is
made unless a caller asks for one of the compatibility properties below.
"""

import torch

from . import _ops


def arch():
    """Compute architecture of the current CUDA device, e.g. "sm_100" (api.py:19-22)."""
    major, minor = torch.cuda.get_device_capability()
    return f"sm_{major}{minor}"


def padded_width(width):
    """Smallest power of two >= width, the row length of the padded conv-state layout."""
    return 1 << (width - 1).bit_length()


class CausalConv1d:
    """Depthwise causal conv1d layer over (dim, width) weights (api.py:186-479)."""

    def __init__(self, weight, bias=None, activation=None):
        """Args:
            weight: (dim, width) filter weights, width 2..8.
            bias: optional (dim,) bias.
            activation: None, "silu" or "swish".

        Raises:
            ValueError: bad activation or weight shape.
        """
        if activation not in (None, "silu", "swish"):
            raise ValueError(f'activation must be None, "silu" or "swish", got {activation!r}')
        if weight.dim() != 2 or not 2 <= weight.shape[1] <= 8:
            raise ValueError(
                f"weight must have shape (dim, width) with 2 <= width <= 8, got {tuple(weight.shape)}"
            )
        self.D, self.W = weight.shape
        self.has_bias, self.act = (bias is not None, None if activation is None else "silu")
        self.weight, self.bias = (weight, bias)
        self._packed = {}

    # Compatibility views of the weights (the kernels read `weight` itself).
    @property
    def wpad(self):
        """Weights zero-padded to padded_width(width) columns (update.py:626-637)."""
        if "wpad" not in self._packed:
            P = padded_width(self.W)
            self._packed["wpad"] = torch.nn.functional.pad(self.weight, (0, P - self.W)).contiguous()
        return self._packed["wpad"]

    @property
    def wflat(self):
        """The caller's (dim, width) weights as one (1, dim * width) row, or None when the
        weights carry a bias or are not contiguous (api.py:246-255)."""
        w = self.weight
        return w.view(1, -1) if self.bias is None and w.is_contiguous() else None

    def fwd(self, x, out=None, cfg=None):
        """Prefill over x of shape (batch, dim, seqlen) (api.py:257-338).

        Args:
            x: (batch, dim, seqlen), any strides.
            out: optional (batch, dim, seqlen) output; must not share storage with x.
            cfg: accepted for signature compatibility and ignored; the library picks the kernel.

        Returns:
            The output; when channels of x are adjacent (a channel-last view) it views
            (batch, seqlen, dim) storage, otherwise it is contiguous.

        Raises:
            ValueError: out shares storage with x, or has the wrong shape.
        """
        B, D, L = x.shape
        if out is None:
            if x.stride(1) == 1 and D > 1:
                out = torch.empty((B, L, D), dtype=x.dtype, device=x.device).transpose(1, 2)
            else:
                out = torch.empty((B, D, L), dtype=x.dtype, device=x.device)
        else:
            if out.untyped_storage().data_ptr() == x.untyped_storage().data_ptr():
                raise ValueError(
                    "causal_conv1d_cute prefill is out-of-place only: `out` must not share storage with `x`"
                )
            if tuple(out.shape) != (B, D, L) or out.dtype != x.dtype or out.device != x.device:
                raise ValueError(f"out must be a {x.dtype} tensor of shape {(B, D, L)} on {x.device}")
        return _ops.fwd(x, self.weight, self.bias, self.act, out)

    def update(self, x, conv_state, out=None, cfg=None):
        """Single-token decode of x (batch, dim) against conv_state (batch, dim, state_len)
        (api.py:419-479).

        state_len is width - 1 (standard layout) or padded_width(width) (padded layout: the
        history is the last width - 1 entries and the whole row shifts by one); any length
        >= width - 1 is accepted.
        """
        B, D = x.shape
        if conv_state.dim() != 3 or conv_state.shape[:2] != (B, D) or conv_state.shape[2] < self.W - 1:
            raise ValueError(f"conv_state shape {tuple(conv_state.shape)} is not ({B}, {D}, >= {self.W - 1})")
        if out is None:
            out = torch.empty((B, D), dtype=x.dtype, device=x.device)
        _ops.update(x.unsqueeze(-1), conv_state, self.weight, self.bias, self.act,
                    out.unsqueeze(-1), None, -1, None, None)
        return out

    def update_ring(
        self,
        x,
        ring_state,
        cache_seqlens,
        conv_state_indices=None,
        pad_slot_id=-1,
        out=None,
        cfg=None,
    ):
        """Single-token decode on a ring conv state (slots, width - 1, dim) (api.py:346-398)."""
        B = x.shape[0]
        dev = x.device
        seen = cache_seqlens if cache_seqlens.device == dev else cache_seqlens.to(dev)
        if seen.dtype != torch.int32:
            seen = seen.to(torch.int32)
        idx = conv_state_indices
        if idx is not None:
            idx = idx if idx.device == dev else idx.to(dev)
            if idx.dtype != torch.int32:
                idx = idx.to(torch.int32)
        elif ring_state.shape[0] < B:
            raise ValueError(f"ring_state has {ring_state.shape[0]} slots for {B} rows and no indices")
        if out is None:
            out = torch.empty((B, self.D), dtype=x.dtype, device=dev)
        return _ops.update_ring(x, ring_state, self.weight, self.bias, self.act, out, seen, idx,
                                pad_slot_id)
