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


# ---------------------------------------------------------------------------------------------
# fp32 references of every entry point, computed with PyTorch on the tensors' own device. They
# extend reference() above (reference testing.py:105-128) to the packed, multi-step, indexed and
# ring paths, following the reference's CPU algorithm (fallback.py:49-164, functional.py:911-922):
# an unrounded fp32 output for the accuracy check and the cache writes, which are copies of the
# inputs, exactly. bench.py gates every timed path on them, and the tests use them over whole
# BASELINE-sized tensors. Outputs of skipped rows (pad slots, empty sequences) are NaN.
# ---------------------------------------------------------------------------------------------


def _conv_hist(full, w, b, silu):
    """Valid depthwise conv of full (..., D, n + W - 1) in fp32 -> (..., D, n)."""
    D, W = w.shape
    lead = full.shape[:-2]
    y = F.conv1d(full.float().reshape(-1, D, full.shape[-1]), w.float().unsqueeze(1),
                 None if b is None else b.float(), groups=D)
    y = y.reshape(*lead, D, y.shape[-1])
    return F.silu(y) if silu else y


def ref_fwd(x, w, b, silu):
    """Prefill (batch, dim, seqlen) -> fp32 output with zero history before every row."""
    W = w.shape[1]
    return _conv_hist(F.pad(x.float(), (W - 1, 0)), w, b, silu)


def ref_varlen(x, w, b, qsl, cidx, hinit, states, silu, pad=-1):
    """Packed prefill of x (dim, ntokens) -> (fp32 output, states after) (fallback.py:77-114).

    states (slots, dim, W-1) is not modified; a copy with every live sequence's final state is
    returned (None without states)."""
    D, T = x.shape
    K = w.shape[1] - 1
    out = torch.full((D, T), float("nan"), device=x.device)
    st = None if states is None else states.clone()
    bounds = [int(v) for v in qsl.tolist()]
    slots = list(range(len(bounds) - 1)) if cidx is None else [int(v) for v in cidx.tolist()]
    init = [False] * len(slots) if hinit is None else [bool(v) for v in hinit.tolist()]
    for i, slot in enumerate(slots):
        a, e = bounds[i], bounds[i + 1]
        if e <= a or (st is not None and slot == pad):
            continue
        h = st[slot] if st is not None and init[i] else x.new_zeros(D, K)
        full = torch.cat([h, x[:, a:e]], dim=1)
        out[:, a:e] = _conv_hist(full, w, b, silu)
        if st is not None:
            st[slot] = full[:, full.shape[1] - K:]
    return out, st


def ref_update(x, state, w, b, silu, idx=None, pad=-1, inter=None, iidx=None):
    """Decode of x (batch, dim) or (batch, dim, steps) against state (slots, dim, S >= W-1) ->
    (fp32 output, state after, dense per-step windows after) (fallback.py:117-164). Pad rows keep
    their state; the inputs are not modified."""
    W = w.shape[1]
    K = W - 1
    xs = x.unsqueeze(-1) if x.dim() == 2 else x
    B, D, L = xs.shape
    slots = torch.arange(B, device=x.device) if idx is None else idx.long()
    live = slots != pad
    st = state.clone()
    it = None if inter is None else inter.clone()
    full = torch.cat([state[slots.clamp_min(0)], xs], dim=-1)  # (B, D, S + L)
    out = _conv_hist(full[..., full.shape[-1] - (K + L):], w, b, silu)
    out[~live] = float("nan")
    st[slots[live]] = full[live][..., L:]
    if it is not None:
        islots = slots if iidx is None else iidx.long()
        S = state.shape[-1]
        for t in range(L):
            first = S + t + 1 - K
            it[islots[live], t] = full[live][..., first:first + K]
    return (out[..., 0] if x.dim() == 2 else out), st, it


def ref_update_ring(x, ring, w, b, silu, seen, idx=None, pad=-1):
    """Single-token decode on a ring state (slots, W-1, dim) -> (fp32 output, ring after):
    from_ring + update + overwrite of row seen % (W-1) (functional.py:911-922)."""
    K = ring.shape[1]
    B, D = x.shape
    slots = torch.arange(B, device=x.device) if idx is None else idx.long()
    live = slots != pad
    rows = (seen.long().unsqueeze(1) + torch.arange(K, device=x.device)) % K  # (B, K)
    sl = slots.clamp_min(0)
    ordered = ring[sl.unsqueeze(1), rows]  # (B, K, D), oldest first
    full = torch.cat([ordered.transpose(1, 2), x.unsqueeze(-1)], dim=-1)
    out = _conv_hist(full, w, b, silu)[..., 0]
    out[~live] = float("nan")
    rg = ring.clone()
    pos = seen.long() % K
    rg[slots[live], pos[live]] = x[live]
    return out, rg


def ref_to_ring(state, seen):
    """Ordered state (slots, dim, K) -> ring (slots, K, dim): ring row (seen + k) % K holds entry
    k (ring.py:33-49)."""
    S, D, K = state.shape
    rows = (seen.long().unsqueeze(1) + torch.arange(K, device=state.device)) % K
    ring = torch.empty(S, K, D, dtype=state.dtype, device=state.device)
    ring[torch.arange(S, device=state.device).unsqueeze(1), rows] = state.transpose(1, 2)
    return ring


def ref_from_ring(ring, seen):
    """Ring (slots, K, dim) -> ordered state (slots, dim, K) (ring.py:52-67)."""
    S, K, D = ring.shape
    rows = (seen.long().unsqueeze(1) + torch.arange(K, device=ring.device)) % K
    return ring[torch.arange(S, device=ring.device).unsqueeze(1), rows].transpose(1, 2).contiguous()


def ref_update_unpack(qkvz, ba, state, w, b, idx, heads, silu, pad=-1):
    """Fused Gated DeltaNet decode (unpack.py:33-222) -> (fp32 conv output, z, b, a, state
    after): the conv reads the leading dim columns of each row; rows whose slot is the pad id or
    outside the cache keep their state and output their conv input."""
    D = w.shape[0]
    zdim = qkvz.shape[1] - D
    x = qkvz[:, :D]
    slots = idx.long()
    valid = (slots != pad) & (slots >= 0) & (slots < state.shape[0])
    out, st, _ = ref_update(x[valid], state, w, b, silu, idx[valid])
    full = x.float().clone()
    full[valid] = out
    return (full, qkvz[:, D:D + zdim].clone(), ba[:, :heads].clone(), ba[:, heads:2 * heads].clone(),
            st)


def within(got, ref, tol):
    """|got - ref| <= tol + tol |ref| wherever ref is not NaN (NaN marks undefined outputs)."""
    got, ref = got.float(), ref.float()
    keep = ~torch.isnan(ref)
    err = (got - ref).abs()
    return bool(((err <= tol + tol * ref.abs()) | ~keep).all())


def copy_ceiling(dst, src):
    """Copy src into dst (same number of bytes, CUDA, 32-byte aligned) with the library's own
    32-byte-vector copy kernel (cc1d_copy) on the current stream: the measured ceiling that the
    streaming kernels are reported against (reference benchmarks/copy_baseline.py:38-90)."""
    from ._lib import check, load

    n = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() != n or not (src.is_contiguous() and dst.is_contiguous()):
        raise ValueError("copy_ceiling needs contiguous tensors of the same size in bytes")
    stream = torch.cuda.current_stream(src.device).cuda_stream
    check(load().cc1d_copy(dst.data_ptr(), src.data_ptr(), n, stream))
    return dst
