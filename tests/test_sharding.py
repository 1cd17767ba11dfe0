"""The multi-GPU path (channel-slice sharding, all-gather check, max-over-ranks timing) with two
gloo ranks on the CPU. The per-rank compute is the oracle, so no GPU is needed; the kernels' own
sharded runs are checked by bench.py on the GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from causal_conv1d_cute import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _prefill(x, w, b):
    """Oracle prefill on torch CPU tensors, x (B, D, L)."""
    y = oracle.fwd(x.numpy(), w.numpy(), b.numpy(), True, "f32")
    return torch.from_numpy(y)


def _varlen_states(x, w, states, qsl):
    """Oracle varlen returning the updated state cache (slots, D, K)."""
    _, st = oracle.varlen(x.numpy(), w.numpy(), None, qsl.numpy(), None,
                          np.ones(len(qsl) - 1, np.uint8), states.numpy(), False, -1, "f32")
    return torch.from_numpy(st)


def _varlen_both(x, w, states, qsl):
    """Oracle varlen returning (output, updated state cache)."""
    out, st = oracle.varlen(x.numpy(), w.numpy(), None, qsl.numpy(), None,
                            np.ones(len(qsl) - 1, np.uint8), states.numpy(), False, -1, "f32")
    return torch.from_numpy(out), torch.from_numpy(st)


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        D = 64
        x = torch.randn(2, D, 37, generator=g)
        w = torch.rand(D, 4, generator=g) - 0.5
        b = torch.randn(D, generator=g)
        ok1 = shard.sharded_equals_unsharded(_prefill, [x, w, b], [1, 0, 0], 1, rank, world, "cpu")
        qsl = torch.tensor([0, 3, 20, 21], dtype=torch.int32)
        xv = torch.randn(D, 21, generator=g)
        st = torch.randn(3, D, 3, generator=g)
        ok2 = shard.sharded_equals_unsharded(
            lambda a, ww, s, q: _varlen_states(a, ww, s, q), [xv, w, st, qsl], [0, 0, 1, None], 1,
            rank, world, "cpu")
        # Several outputs: the output and the state cache of a packed prefill.
        ok3 = shard.sharded_equals_unsharded(
            lambda a, ww, s, q: _varlen_both(a, ww, s, q), [xv, w, st, qsl], [0, 0, 1, None],
            (0, 1), rank, world, "cpu")
        # A deliberately wrong shard (a planted mistake in the oracle output) must be caught.
        bad = shard.sharded_equals_unsharded(
            lambda a, ww, bb: _prefill(a, ww, bb) + (rank == 1) * (a.shape[1] < D), [x, w, b],
            [1, 0, 0], 1, rank, world, "cpu")
        slowest = shard.max_over_ranks(1.0 + rank, "cpu", world)
        result[rank] = (ok1, ok2 and ok3, bad, slowest)
    finally:
        dist.destroy_process_group()


def test_channel_slices():
    assert shard.channel_slice(8192, 3, 8) == (3072, 4096)
    with pytest.raises(ValueError):
        shard.channel_slice(100, 0, 8)
    t = torch.arange(24).view(2, 12)
    assert torch.equal(shard.shard(t, 1, 1, 3), t[:, 4:8])


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(result)
    for r in range(2):
        ok1, ok2, bad, slowest = res[r]
        assert ok1 and ok2
        assert not bad
        assert slowest == 2.0
