"""numpy restatement of the reference's CPU algorithm (test infrastructure only; see __init__).

Each function names the reference lines it follows. Reference paths are relative to the
causal-conv1d-cute project root.
"""

import numpy as np

DTYPES = ("bf16", "f16", "f32")


def round_to(a, dtype):
    """Round float values to the storage dtype (round to nearest even) and return float32.

    bf16 rounding keeps the high 16 bits of the float32 after adding 0x7FFF plus the lowest kept
    bit, the usual round-to-nearest-even on the bit pattern; NaN stays NaN.
    """
    a = np.asarray(a, dtype=np.float32)
    if dtype == "f32":
        return a.copy()
    if dtype == "f16":
        return a.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(dtype)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + ((u >> 16) & 1) + 0x7FFF) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), r).astype(np.float32)


def _silu(a):
    """x * sigmoid(x) in float64, without overflow for large |x|."""
    e = np.exp(-np.abs(a))
    return np.where(a >= 0, a / (1.0 + e), a * e / (1.0 + e))


def _conv_valid(full, w, b, silu):
    """Valid (unpadded) depthwise conv of full (D, n + W - 1) -> (D, n) in float64.

    Restates fallback._conv (fallback.py:28-46): F.conv1d over a history-prefixed sequence.
    """
    D, W = w.shape
    n = full.shape[1] - (W - 1)
    acc = np.zeros((D, max(n, 0)), dtype=np.float64)
    if b is not None:
        acc += np.asarray(b, np.float64)[:, None]
    full = np.asarray(full, np.float64)
    for k in range(W):
        acc += np.asarray(w[:, k], np.float64)[:, None] * full[:, k : k + n]
    return _silu(acc) if silu else acc


def fwd(x, w, b, silu, dtype):
    """Prefill over (batch, dim, seqlen): fallback.fwd (fallback.py:49-74).

    Zero history before every sequence, output rounded to dtype.
    """
    B, D, L = x.shape
    W = w.shape[1]
    out = np.empty((B, D, L), np.float32)
    for i in range(B):
        full = np.concatenate([np.zeros((D, W - 1), np.float32), x[i]], axis=1)
        out[i] = round_to(_conv_valid(full, w, b, silu), dtype)
    return out


def fwd_states(x, w, b, seq_idx, init, silu, dtype):
    """Prefill with the Dao-AILab causal_conv1d_fn extras, which the reference passes upstream
    (dao_compat.py:28-78) to the `causal_conv1d` package (Dao-AILab/causal-conv1d; the reference
    pins no version).

    Restates that package's published semantics. x (batch, dim, seqlen); init (batch, dim, W-1)
    or None: the history before token 0 of each row, as the reference's own varlen fallback uses a
    cached initial state (fallback.py:77-114); the final state is the last W-1 entries of
    [init | x]. seq_idx (batch, seqlen) or None: the output at token t sums only the taps whose
    token has the same id as t (a differing id contributes nothing), zero history before token 0;
    it excludes init. Returns (out rounded to dtype, final states (batch, dim, W-1)).
    """
    B, D, L = x.shape
    W = w.shape[1]
    K = W - 1
    out = np.empty((B, D, L), np.float32)
    final = np.empty((B, D, K), np.float32)
    for i in range(B):
        hist = np.zeros((D, K), np.float32) if init is None else np.asarray(init[i], np.float32)
        full = np.concatenate([hist, x[i]], axis=1)
        final[i] = full[:, -K:]
        if seq_idx is None:
            out[i] = round_to(_conv_valid(full, w, b, silu), dtype)
            continue
        q = np.asarray(seq_idx[i])
        acc = np.zeros((D, L), np.float64)
        if b is not None:
            acc += np.asarray(b, np.float64)[:, None]
        for t in range(L):
            for k in range(W):
                p = t - K + k
                if p >= 0 and q[p] == q[t]:
                    acc[:, t] += np.asarray(w[:, k], np.float64) * np.float64(x[i][:, p])
        out[i] = round_to(_silu(acc) if silu else acc, dtype)
    return out, final


def varlen(x, w, b, qsl, cidx, hinit, states, silu, pad, dtype):
    """Packed prefill: fallback.varlen (fallback.py:77-114).

    x is (dim, total_tokens). Returns (out, states') where states' is a copy of states with the
    final state of every live sequence written (None when states is None). Sequences of zero
    tokens, and sequences whose slot is pad when states are given, are skipped: their outputs are
    NaN here (undefined in the reference) and their slots unchanged.
    """
    D, T = x.shape
    W = w.shape[1]
    K = W - 1
    out = np.full((D, T), np.nan, np.float32)
    st = None if states is None else states.copy()
    nseq = len(qsl) - 1
    slots = list(range(nseq)) if cidx is None else [int(s) for s in cidx]
    inits = [False] * nseq if hinit is None else [bool(h) for h in hinit]
    for i in range(nseq):
        a, e, slot = int(qsl[i]), int(qsl[i + 1]), slots[i]
        if e <= a or (st is not None and slot == pad):
            continue
        use = st is not None and inits[i]
        init = st[slot] if use else np.zeros((D, K), np.float32)
        full = np.concatenate([init, x[:, a:e]], axis=1)
        out[:, a:e] = round_to(_conv_valid(full, w, b, silu), dtype)
        if st is not None:
            st[slot] = full[:, -K:]
    return out, st


def update(x, state, w, b, silu, idx, pad, inter, iidx, dtype):
    """Decode of one or more tokens: fallback.update (fallback.py:117-164).

    x is (batch, dim) or (batch, dim, steps); state is (slots, dim, state_len >= W-1) and the
    whole row shifts by steps. inter, when given, is a dense (slots, steps, dim, W-1) array; the
    "dedup" layout is a view of the same values and is checked through it. Returns
    (out, state', inter'); outputs of pad rows are NaN (undefined in the reference).
    """
    W = w.shape[1]
    K = W - 1
    xs = x[..., None] if x.ndim == 2 else x
    B, D, L = xs.shape
    out = np.full((B, D, L), np.nan, np.float32)
    st = state.copy()
    it = None if inter is None else inter.copy()
    slots = list(range(B)) if idx is None else [int(s) for s in idx]
    islots = slots if iidx is None else [int(s) for s in iidx]
    for i, slot in enumerate(slots):
        if slot == pad:
            continue
        full = np.concatenate([st[slot], xs[i]], axis=1)
        out[i] = round_to(_conv_valid(full[:, -(K + L):], w, b, silu), dtype)
        st[slot] = full[:, L:]
        if it is not None:
            for t in range(L):
                first = full.shape[1] - L + t + 1 - K
                it[islots[i], t] = full[:, first : first + K]
    return (out[..., 0] if x.ndim == 2 else out), st, it


def to_ring(state, seen):
    """Ordered (slots, dim, K) -> ring (slots, K, dim): ring.to_ring (ring.py:33-49).

    Row (seen + k) % K of the ring holds entry k (oldest first) of the ordered state.
    """
    S, D, K = state.shape
    ring = np.empty((S, K, D), state.dtype)
    for s in range(S):
        for k in range(K):
            ring[s, (int(seen[s]) + k) % K] = state[s, :, k]
    return ring


def from_ring(ring, seen):
    """Ring (slots, K, dim) -> ordered (slots, dim, K): ring.from_ring (ring.py:52-67)."""
    S, K, D = ring.shape
    state = np.empty((S, D, K), ring.dtype)
    for s in range(S):
        for k in range(K):
            state[s, :, k] = ring[s, (int(seen[s]) + k) % K]
    return state


def update_ring(x, ring, w, b, silu, seen, idx, pad, dtype):
    """Single-token decode on a ring state: functional.causal_conv1d_update_ring's CPU path
    (functional.py:911-922), i.e. from_ring + fallback.update + overwrite of row seen % K.

    Returns (out, ring'); outputs of pad rows are NaN.
    """
    B, D = x.shape
    K = ring.shape[1]
    rg = ring.copy()
    out = np.full((B, D), np.nan, np.float32)
    slots = list(range(B)) if idx is None else [int(s) for s in idx]
    for i, slot in enumerate(slots):
        if slot == pad:
            continue
        ordered = from_ring(rg[slot : slot + 1], seen[i : i + 1])[0]
        full = np.concatenate([ordered, x[i][:, None]], axis=1)
        out[i] = round_to(_conv_valid(full, w, b, silu)[:, 0], dtype)
        rg[slot, int(seen[i]) % K] = x[i]
    return out, rg


def update_unpack(qkvz, ba, state, w, b, idx, heads, silu, pad, dtype):
    """Fused Gated DeltaNet decode: the semantics of ConvUpdateUnpack (unpack.py:33-222).

    The conv input is the leading dim columns of each [Q|K|V|Z] row; Z is the next zdim columns,
    B and A the two halves of each [B|A] row. Rows whose slot is pad or outside the cache keep
    their state and get their conv input as output. Returns (out, z, b, a, state').
    """
    D, W = w.shape
    zdim = qkvz.shape[1] - D
    B = qkvz.shape[0]
    st = state.copy()
    out = np.empty((B, D), np.float32)
    for i in range(B):
        slot = int(idx[i])
        xr = qkvz[i, :D]
        if slot == pad or slot < 0 or slot >= st.shape[0]:
            out[i] = xr
            continue
        full = np.concatenate([st[slot], xr[:, None]], axis=1)
        out[i] = round_to(_conv_valid(full, w, b, silu)[:, 0], dtype)
        st[slot] = full[:, 1:]
    return out, qkvz[:, D : D + zdim].copy(), ba[:, :heads].copy(), ba[:, heads : 2 * heads].copy(), st
