"""The oracle's prefill with initial / final states and sequence ids (oracle.fwd_states), anchored
on the pinned varlen restatement: a batch row with an initial state is a packed sequence with a
cached initial state, and a row split by sequence ids into contiguous runs is a packed batch of
those runs without states. Runs on the CPU."""

import numpy as np
import pytest

import oracle


def _rand(rng, *shape, dtype="bf16"):
    return oracle.round_to(rng.standard_normal(shape).astype(np.float32), dtype)


@pytest.mark.parametrize("W", [2, 4, 8])
@pytest.mark.parametrize("L", [1, 3, 7, 40])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_initial_and_final_states_match_varlen(W, L, dtype):
    rng = np.random.default_rng(W * 100 + L)
    B, D, K = 3, 16, W - 1
    x = _rand(rng, B, D, L, dtype=dtype)
    w = _rand(rng, D, W, dtype=dtype)
    b = _rand(rng, D, dtype=dtype)
    init = _rand(rng, B, D, K, dtype=dtype)
    out, fin = oracle.fwd_states(x, w, b, None, init, True, dtype)
    packed = np.concatenate(list(x), axis=1)  # (D, B * L)
    qsl = np.arange(B + 1) * L
    v_out, v_st = oracle.varlen(packed, w, b, qsl, np.arange(B), np.ones(B, bool), init.copy(),
                                True, -1, dtype)
    np.testing.assert_array_equal(out, np.stack(np.split(v_out, B, axis=1)))
    np.testing.assert_array_equal(fin, v_st)
    # Without initial states the history is zeros: the plain prefill.
    out0, fin0 = oracle.fwd_states(x, w, b, None, None, True, dtype)
    np.testing.assert_array_equal(out0, oracle.fwd(x, w, b, True, dtype))
    full = np.concatenate([np.zeros((B, D, K), np.float32), x], axis=2)
    np.testing.assert_array_equal(fin0, full[:, :, -K:])


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_contiguous_sequence_ids_match_varlen(W):
    rng = np.random.default_rng(W)
    B, D, L = 2, 8, 50
    x = _rand(rng, B, D, L)
    w = _rand(rng, D, W)
    lens = [[1, 2, 17, 30], [50]]
    seq = np.stack([np.repeat(np.arange(len(r)) + 10 * i, r) for i, r in enumerate(lens)])
    out, _ = oracle.fwd_states(x, w, None, seq, None, False, "bf16")
    for i, r in enumerate(lens):
        qsl = np.concatenate([[0], np.cumsum(r)])
        v_out, _ = oracle.varlen(x[i], w, None, qsl, None, None, None, False, -1, "bf16")
        np.testing.assert_array_equal(out[i], v_out)


def test_recurring_sequence_id_follows_the_equality_rule():
    """Ids [0, 1, 0]: the third token's first tap reaches the first token across the second."""
    x = np.array([[[1.0, 2.0, 4.0]]], np.float32)
    w = np.array([[1.0, 10.0, 100.0]], np.float32)
    out, _ = oracle.fwd_states(x, w, None, np.array([[0, 1, 0]]), None, False, "f32")
    np.testing.assert_array_equal(out[0, 0], [100.0, 200.0, 1.0 * 1 + 4.0 * 100])
