"""CPU oracle for the depthwise causal conv1d hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the algorithm of the reference's PyTorch fallback
(causal_conv1d_cute/fallback.py) and of its ring and fused-decode semantics. It is the checker
that the CUDA kernels are compared against, and nothing else: only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may import or run anything under oracle/. The library itself never
routes through it; it raises when its CUDA extension is missing.

Parity is pinned: tests/test_oracle_golden.py checks every function here against golden vectors
that tests/golden/make_golden.py produced by running the reference package itself on the CPU.
fwd_states restates calls the reference does not run itself (it passes them to the upstream
Dao-AILab causal_conv1d package, absent here): tests/test_oracle_states.py anchors its initial and
final states and its sequence-id split on varlen (pinned above); the equality rule for sequence
ids that recur non-contiguously is the upstream's published rule, unpinned by a golden vector.

Conventions: tensors are numpy arrays of float32 holding values exactly representable in the
storage dtype ("bf16", "f16" or "f32"); results are rounded to that dtype and returned as float32.
Sums are formed in float64 (bias first, taps oldest first) and rounded once, so the oracle is at
least as accurate as the reference's float32 F.conv1d.
"""

from .restate import (  # noqa: F401
    DTYPES,
    from_ring,
    fwd,
    fwd_states,
    round_to,
    to_ring,
    update,
    update_ring,
    update_unpack,
    varlen,
)
