"""Tensor-level calls into libcc1d.so, registered as torch.library ops (cc1d::fwd, cc1d::update,
cc1d::update_ring, cc1d::varlen, cc1d::update_unpack, cc1d::fwd_states, cc1d::to_ring,
cc1d::from_ring).

Each op passes data pointers, element strides and sizes of already-validated CUDA tensors to
one C entry point, on the current stream of the tensors' device. No host synchronisation, no
allocation: outputs are allocated by the caller. The C side picks the kernel variant for the
layout it is given.

Device status. When checks are enabled (set_device_checks(True)), every call passes a per-device
int32 status word that kernels OR a bit into when they skip an index outside the caches (a slot
outside the state cache, sequence bounds outside the packed tokens). device_status() reads and
clears it. Checks are off by default so that no call allocates anything.
"""

import torch

from . import _lib
from ._lib import check, dtype_code, load

_checks = False
_status = {}


def set_device_checks(enabled=True):
    """Turn the device-side index checks' status word on or off for later calls."""
    global _checks
    _checks = bool(enabled)


def device_status(device=None, clear=True):
    """Return the OR of the CC1D_DEV_* bits reported on device since the last clear (syncs)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    t = _status.get(dev.index)
    if t is None:
        return 0
    v = int(t.item())
    if clear:
        t.zero_()
    return v


def _status_ptr(device):
    if not _checks:
        return None
    t = _status.get(device.index)
    if t is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        t = _status[device.index] = torch.zeros(1, dtype=torch.int32, device=device)
    return t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device):
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _fwd_impl(x, weight, bias, silu, out):
    """out[b, c, t] for x, out of shape (batch, dim, seqlen), any strides (cc1d_fwd)."""
    lib = load()
    B, D, L = x.shape
    check(
        lib.cc1d_fwd(
            x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
            weight.data_ptr(), weight.stride(0), weight.stride(1),
            _ptr(bias), 0 if bias is None else bias.stride(0),
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
            B, D, L, weight.shape[1], dtype_code(x.dtype), int(bool(silu)), _stream(x.device),
        )
    )
    return out


def _fwd_states_impl(x, weight, bias, silu, out, seq_idx, initial_states, final_states):
    """Prefill with sequence ids and/or initial / final states (cc1d_fwd_states).

    seq_idx int32 (batch, seqlen) or None; initial_states / final_states (batch, dim, W-1) or None.
    """
    lib = load()
    B, D, L = x.shape
    q = (None, 0, 0) if seq_idx is None else (seq_idx.data_ptr(), *seq_idx.stride())
    i = (None, 0, 0, 0) if initial_states is None else (initial_states.data_ptr(), *initial_states.stride())
    f = (None, 0, 0, 0) if final_states is None else (final_states.data_ptr(), *final_states.stride())
    check(
        lib.cc1d_fwd_states(
            x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
            weight.data_ptr(), weight.stride(0), weight.stride(1),
            _ptr(bias), 0 if bias is None else bias.stride(0),
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
            *q, *i, *f,
            B, D, L, weight.shape[1], dtype_code(x.dtype), int(bool(silu)), _stream(x.device),
        )
    )
    return out


def _update_impl(x3, state, weight, bias, silu, out3, idx, pad, inter, iidx):
    """Decode of x3 (batch, dim, steps) into out3 of the same shape (cc1d_update).

    state is (slots, dim, state_len); inter, when given, is (inter_slots, steps, dim, W-1).
    idx / iidx are int32 CUDA tensors or None.
    """
    lib = load()
    B, D, L = x3.shape
    if inter is None:
        ip, ist, inslots = None, (0, 0, 0, 0), 0
    else:
        ip, ist, inslots = inter.data_ptr(), inter.stride(), inter.shape[0]
    check(
        lib.cc1d_update(
            x3.data_ptr(), x3.stride(0), x3.stride(1), x3.stride(2),
            state.data_ptr(), state.stride(0), state.stride(1), state.stride(2),
            state.shape[2], state.shape[0],
            weight.data_ptr(), weight.stride(0), weight.stride(1),
            _ptr(bias), 0 if bias is None else bias.stride(0),
            out3.data_ptr(), out3.stride(0), out3.stride(1), out3.stride(2),
            _ptr(idx), int(pad),
            ip, ist[0], ist[1], ist[2], ist[3], inslots, _ptr(iidx),
            B, D, L, weight.shape[1], dtype_code(x3.dtype), int(bool(silu)),
            _status_ptr(x3.device), _stream(x3.device),
        )
    )
    return out3


def _update_ring_impl(x, ring, weight, bias, silu, out, seen, idx, pad):
    """Ring decode of x (batch, dim) against ring (slots, W-1, dim) (cc1d_update_ring)."""
    lib = load()
    B, D = x.shape
    check(
        lib.cc1d_update_ring(
            x.data_ptr(), x.stride(0), x.stride(1),
            ring.data_ptr(), ring.stride(0), ring.stride(1), ring.stride(2), ring.shape[0],
            weight.data_ptr(), weight.stride(0), weight.stride(1),
            _ptr(bias), 0 if bias is None else bias.stride(0),
            out.data_ptr(), out.stride(0), out.stride(1),
            seen.data_ptr(), _ptr(idx), int(pad),
            B, D, weight.shape[1], dtype_code(x.dtype), int(bool(silu)),
            _status_ptr(x.device), _stream(x.device),
        )
    )
    return out


def _to_ring_impl(state, ring, seen):
    """Ordered state (slots, dim, W-1) -> ring state (slots, W-1, dim) (cc1d_to_ring); seen is an
    int32 CUDA tensor (slots,)."""
    lib = load()
    S, D, K = state.shape
    check(lib.cc1d_to_ring(state.data_ptr(), *state.stride(), ring.data_ptr(), *ring.stride(),
                           seen.data_ptr(), S, D, K + 1, dtype_code(state.dtype),
                           _stream(state.device)))


def _from_ring_impl(ring, state, seen):
    """Ring state (slots, W-1, dim) -> ordered state (slots, dim, W-1) (cc1d_from_ring)."""
    lib = load()
    S, D, K = state.shape
    check(lib.cc1d_from_ring(ring.data_ptr(), *ring.stride(), state.data_ptr(), *state.stride(),
                             seen.data_ptr(), S, D, K + 1, dtype_code(state.dtype),
                             _stream(state.device)))


def _varlen_impl(x, weight, bias, silu, out, qsl, cidx, hinit, states, pad):
    """Packed prefill of x (dim, ntokens) into out (dim, ntokens) (cc1d_varlen).

    qsl int32 (nseq + 1,); cidx int32 or None; hinit uint8 or None; states (slots, dim, W-1)
    or None.
    """
    lib = load()
    D, T = x.shape
    if states is None:
        sp, ss, nslots = None, (0, 0, 0), 0
    else:
        sp, ss, nslots = states.data_ptr(), states.stride(), states.shape[0]
    check(
        lib.cc1d_varlen(
            x.data_ptr(), x.stride(0), x.stride(1),
            weight.data_ptr(), weight.stride(0), weight.stride(1),
            _ptr(bias), 0 if bias is None else bias.stride(0),
            out.data_ptr(), out.stride(0), out.stride(1),
            qsl.data_ptr(), qsl.numel() - 1, T, _ptr(cidx), _ptr(hinit),
            sp, ss[0], ss[1], ss[2], nslots, int(pad),
            D, weight.shape[1], dtype_code(x.dtype), int(bool(silu)),
            _status_ptr(x.device), _stream(x.device),
        )
    )
    return out


def _update_unpack_impl(qkvz, ba, state, weight, bias, out, z, b, a, idx, heads, silu, pad):
    """Fused Gated DeltaNet decode step (cc1d_update_unpack)."""
    lib = load()
    B = qkvz.shape[0]
    D, W = weight.shape
    zdim = qkvz.shape[1] - D
    check(
        lib.cc1d_update_unpack(
            qkvz.data_ptr(), qkvz.stride(0), ba.data_ptr(), ba.stride(0),
            state.data_ptr(), state.shape[0], weight.data_ptr(), _ptr(bias),
            out.data_ptr(), z.data_ptr(), b.data_ptr(), a.data_ptr(),
            idx.data_ptr(), int(pad), B, D, zdim, int(heads), W,
            dtype_code(qkvz.dtype), dtype_code(ba.dtype), int(bool(silu)), _stream(qkvz.device),
        )
    )
    return out, z, b, a


# ---------------------------------------------------------------------------------------------
# torch.library registration: the entry points as dispatcher ops cc1d::<name>, with the mutated
# arguments (outputs and caches) marked in the schemas and fake implementations for meta/fake
# tensors (tracing, torch.compile). The CUDA implementations are the functions above. The ops are
# defined with the low-level torch.library.Library API: per call it adds about 6 us of host time,
# against about 28 us for torch.library.custom_op (measured on the host, no GPU work).
# ---------------------------------------------------------------------------------------------

_SCHEMAS = {
    "fwd": "fwd(Tensor x, Tensor weight, Tensor? bias, bool silu, Tensor(a!) out) -> ()",
    "fwd_states": (
        "fwd_states(Tensor x, Tensor weight, Tensor? bias, bool silu, Tensor(a!) out, "
        "Tensor? seq_idx, Tensor? initial_states, Tensor(b!)? final_states) -> ()"
    ),
    "update": (
        "update(Tensor x3, Tensor(a!) state, Tensor weight, Tensor? bias, bool silu, "
        "Tensor(b!) out3, Tensor? idx, int pad, Tensor(c!)? inter, Tensor? iidx) -> ()"
    ),
    "update_ring": (
        "update_ring(Tensor x, Tensor(a!) ring, Tensor weight, Tensor? bias, bool silu, "
        "Tensor(b!) out, Tensor seen, Tensor? idx, int pad) -> ()"
    ),
    "to_ring": "to_ring(Tensor state, Tensor(a!) ring, Tensor seen) -> ()",
    "from_ring": "from_ring(Tensor ring, Tensor(a!) state, Tensor seen) -> ()",
    "varlen": (
        "varlen(Tensor x, Tensor weight, Tensor? bias, bool silu, Tensor(a!) out, Tensor qsl, "
        "Tensor? cidx, Tensor? hinit, Tensor(b!)? states, int pad) -> ()"
    ),
    "update_unpack": (
        "update_unpack(Tensor qkvz, Tensor ba, Tensor(a!) state, Tensor weight, Tensor? bias, "
        "Tensor(b!) out, Tensor(c!) z, Tensor(d!) b, Tensor(e!) a, Tensor idx, int heads, "
        "bool silu, int pad) -> ()"
    ),
}
_IMPLS = {
    "fwd": _fwd_impl, "fwd_states": _fwd_states_impl, "update": _update_impl,
    "update_ring": _update_ring_impl, "to_ring": _to_ring_impl, "from_ring": _from_ring_impl,
    "varlen": _varlen_impl,
    "update_unpack": _update_unpack_impl,
}


def _no_result(*args):
    return None


def _kernel(impl):
    # The schemas return nothing: the ops write their results into the tensors they are given.
    def run(*args):
        impl(*args)

    return run


def _register():
    try:
        lib = torch.library.Library("cc1d", "DEF")
    except RuntimeError:
        # This module was already imported under another name in this process: the ops exist.
        return None
    for name, schema in _SCHEMAS.items():
        lib.define(schema)
        lib.impl(name, _kernel(_IMPLS[name]), "CUDA")
        torch.library.register_fake(f"cc1d::{name}", _no_result, lib=lib)
    return lib


_library = _register()
_op = torch.ops.cc1d


def fwd(x, weight, bias, silu, out):
    """out[b, c, t] for x, out of shape (batch, dim, seqlen), any strides (op cc1d::fwd)."""
    _op.fwd(x, weight, bias, bool(silu), out)
    return out


def fwd_states(x, weight, bias, silu, out, seq_idx, initial_states, final_states):
    """Prefill with sequence ids and/or initial / final states (op cc1d::fwd_states)."""
    _op.fwd_states(x, weight, bias, bool(silu), out, seq_idx, initial_states, final_states)
    return out


def update(x3, state, weight, bias, silu, out3, idx, pad, inter, iidx):
    """Decode of x3 (batch, dim, steps) into out3 of the same shape (op cc1d::update)."""
    _op.update(x3, state, weight, bias, bool(silu), out3, idx, int(pad), inter, iidx)
    return out3


def update_ring(x, ring, weight, bias, silu, out, seen, idx, pad):
    """Ring decode of x (batch, dim) against ring (slots, W-1, dim) (op cc1d::update_ring)."""
    _op.update_ring(x, ring, weight, bias, bool(silu), out, seen, idx, int(pad))
    return out


def to_ring(state, ring, seen):
    """Ordered state -> ring state; writes only `ring` (op cc1d::to_ring)."""
    _op.to_ring(state, ring, seen)


def from_ring(ring, state, seen):
    """Ring state -> ordered state; writes only `state` (op cc1d::from_ring)."""
    _op.from_ring(ring, state, seen)


def varlen(x, weight, bias, silu, out, qsl, cidx, hinit, states, pad):
    """Packed prefill of x (dim, ntokens) into out (dim, ntokens) (op cc1d::varlen)."""
    _op.varlen(x, weight, bias, bool(silu), out, qsl, cidx, hinit, states, int(pad))
    return out


def update_unpack(qkvz, ba, state, weight, bias, out, z, b, a, idx, heads, silu, pad):
    """Fused Gated DeltaNet decode step (op cc1d::update_unpack)."""
    _op.update_unpack(qkvz, ba, state, weight, bias, out, z, b, a, idx, int(heads), bool(silu),
                      int(pad))
    return out, z, b, a


__all__ = [
    "device_status", "from_ring", "fwd", "fwd_states", "to_ring", "set_device_checks", "update", "update_ring", "update_unpack",
    "varlen", "_lib",
]
