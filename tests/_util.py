"""Helpers shared by the tests: exact tensor <-> numpy conversion and the parity assertions.

Tolerances (stated by the task for this path): outputs within atol = rtol = 1e-2 for bf16/fp16
and 1e-5 for fp32 against the oracle; conv states, ring rows, per-step windows and every copy
bit-exact.
"""

import numpy as np
import torch

TAG = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
TOL = {torch.bfloat16: 1e-2, torch.float16: 1e-2, torch.float32: 1e-5}


def to_np(t):
    """Float tensor (any dtype/device/strides) -> float32 numpy array holding the same values."""
    if t is None:
        return None
    t = t.detach().cpu()
    if t.dtype in (torch.int32, torch.int64, torch.bool, torch.uint8):
        return t.numpy()
    return t.float().numpy()


def from_np(a, dtype, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=device, dtype=dtype)


def assert_close(got, ref, dtype, mask=None):
    """|got - ref| <= tol + tol * |ref| elementwise (ref is the oracle, float32 numpy)."""
    g = to_np(got) if isinstance(got, torch.Tensor) else np.asarray(got, np.float32)
    r = np.asarray(ref, np.float32)
    assert g.shape == r.shape, (g.shape, r.shape)
    if mask is not None:
        g, r = g[mask], r[mask]
    tol = TOL[dtype]
    bad = ~(np.abs(g - r) <= tol + tol * np.abs(r))
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tol {tol}; max err {np.abs(g - r).max()}"


def bits(t):
    t = t.detach().contiguous()
    if t.dtype == torch.float32:
        return t.view(torch.int32)
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16)
    return t


def assert_bits(a, b):
    """Bit-exact equality of two tensors (or a tensor and an oracle array of its dtype)."""
    if isinstance(b, np.ndarray):
        b = from_np(b, a.dtype, a.device)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert torch.equal(bits(a), bits(b.to(a.device))), "not bit-identical"
