"""Test cases, fp32 references and the accuracy classifier (reference testing.py:1-186).

check() classifies an output against an unrounded fp32 reference the way the reference's test
suite does: the backward error max |got - ref| / (sum_k |w_k x_k| + |b|) must stay within the
accumulation bound 1.1 * (W + 2) * 2^-(m+1) for an m-bit mantissa, else "WRONG"; within it, the
output is "ok" when its error is at most 1.5 ulp wherever |ref| >= REF_MIN, "lowprec" otherwise
(for instance a sum accumulated in 16-bit precision).
"""

from dataclasses import dataclass

import torch
import torch.nn.functional as F

MANT_BITS = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}
REF_MIN = 0.25


@dataclass(frozen=True)
class Case:
    """One configuration: kind "fwd" (prefill) or "update" (single-token decode)."""

    model: str
    kind: str
    D: int
    W: int
    B: int
    L: int = 1
    bias: bool = True
    act: str | None = None
    layout: str = "bdl"  # "bdl" contiguous (batch, dim, seqlen) or "btd" channel-last view
    dtype: torch.dtype = torch.bfloat16

    @property
    def label(self):
        a = "silu" if self.act else "none"
        if self.kind == "fwd":
            return f"{self.model} fwd D={self.D} W={self.W} B={self.B} L={self.L} {self.layout} {a}"
        return f"{self.model} upd D={self.D} W={self.W} B={self.B} {a}"

    @property
    def bytes_moved(self):
        """Minimum traffic: every input element read once, every output element written once."""
        e = torch.empty((), dtype=self.dtype).element_size()
        if self.kind == "fwd":
            return 2 * self.B * self.D * self.L * e
        return (2 * self.B * self.D * (self.W - 1) + 2 * self.B * self.D) * e


def make_inputs(case: Case, seed=0, device="cuda"):
    """Seeded inputs: dict with x, w, b (or None) and, for "update", state (batch, dim, W-1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(device=device, dtype=case.dtype, generator=g)
    w = torch.randn(case.D, case.W, **kw)
    b = torch.randn(case.D, **kw) if case.bias else None
    if case.kind == "fwd":
        if case.layout == "bdl":
            x = torch.randn(case.B, case.D, case.L, **kw)
        elif case.layout == "btd":
            x = torch.randn(case.B, case.L, case.D, **kw).transpose(1, 2)
        else:
            raise ValueError(case.layout)
        return dict(x=x, w=w, b=b)
    x = torch.randn(case.B, case.D, **kw)
    state = torch.randn(case.B, case.D, case.W - 1, **kw)
    return dict(x=x, w=w, b=b, state=state)


def _history(case, t, absval=False):
    f = (lambda v: v.float().abs()) if absval else (lambda v: v.float())
    return torch.cat([f(t["state"]), f(t["x"]).unsqueeze(-1)], dim=-1)


def reference(case: Case, t):
    """fp32 reference: the prefill output, or (output, next state) for "update"."""
    w = t["w"].float()
    b = None if t["b"] is None else t["b"].float()
    if case.kind == "fwd":
        y = F.conv1d(t["x"].float(), w.unsqueeze(1), b, padding=case.W - 1, groups=case.D)
        y = y[..., : case.L]
        return F.silu(y) if case.act else y
    full = _history(case, t)
    y = (full * w).sum(-1) + (0 if b is None else b)
    return (F.silu(y) if case.act else y, full[..., 1:].to(case.dtype))


def l1_magnitude(case: Case, t):
    """sum_k |w_k x_k| + |b| in fp32, the scale of the backward error."""
    w = t["w"].float().abs()
    b = None if t["b"] is None else t["b"].float().abs()
    if case.kind == "fwd":
        m = F.conv1d(t["x"].float().abs(), w.unsqueeze(1), b, padding=case.W - 1, groups=case.D)
        return m[..., : case.L]
    m = (_history(case, t, absval=True) * w).sum(-1)
    return m if b is None else m + b


def check(case: Case, t, got, ref32):
    """Classify got against ref32: returns (status, ulp_err, bwd_err) with status "ok",
    "lowprec" or "WRONG"."""
    got, ref32 = got.float(), ref32.float()
    err = (got - ref32).abs()
    mag = ref32.abs()
    keep = mag >= REF_MIN
    ulp = torch.pow(2.0, torch.floor(torch.log2(mag.clamp_min(REF_MIN))) - MANT_BITS[case.dtype])
    ulp_err = (err / ulp)[keep].max().item() if bool(keep.any()) else 0.0
    bwd_err = (err / l1_magnitude(case, t).clamp_min(1e-6)).max().item()
    bound = 1.1 * (case.W + 2) * 2.0 ** -(MANT_BITS[case.dtype] + 1)
    if not bwd_err <= bound:
        return ("WRONG", ulp_err, bwd_err)
    return ("ok" if ulp_err <= 1.5 else "lowprec", ulp_err, bwd_err)
