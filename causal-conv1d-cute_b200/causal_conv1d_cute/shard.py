"""Channel-slice sharding across the GPUs of one box (tensor-parallel layout).

A depthwise conv has no cross-channel term, so a layer whose D channels are split over N ranks
runs with no exchange at all: rank r owns channels [r D/N, (r + 1) D/N) of the weights, the bias,
every conv-state / ring / per-step cache and the activations. These helpers compute the slices and
check, with one all-gather, that the sharded results equal the unsharded ones bit for bit. They
work with any torch.distributed backend (NCCL on GPUs, gloo on CPU).
"""

import torch
import torch.distributed as dist


def channel_slice(dim, rank, world):
    """The (lo, hi) channel range that `rank` owns; dim must divide evenly."""
    if dim % world:
        raise ValueError(f"{dim} channels do not split evenly over {world} ranks")
    per = dim // world
    return rank * per, (rank + 1) * per


def shard(t, axis, rank, world):
    """The rank's channel slice of tensor t along `axis` (a view)."""
    lo, hi = channel_slice(t.shape[axis], rank, world)
    return t.narrow(axis, lo, hi - lo)


def gather_channels(local, axis, world, group=None):
    """All-gather every rank's slice and concatenate along the channel axis."""
    local = local.contiguous()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.cat(parts, dim=axis)


def max_over_ranks(value, device, world, group=None):
    """Max of a float over ranks (the time of a step is the slowest rank's)."""
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sharded_equals_unsharded(run, inputs, axes, out_axis, rank, world, device, group=None):
    """Run `run` on this rank's channel slice of every input, gather the outputs and compare them
    with `run` on the full inputs (rank 0), bit for bit. Returns the verdict on every rank.

    Args:
        run: callable(*tensors) -> output tensor, or a tuple of output tensors (for instance an
            output and a state cache the call updated).
        inputs: full (unsharded) tensors, identical on every rank.
        axes: channel axis of each input (None: replicated, passed whole).
        out_axis: channel axis of the output, or a tuple with one axis per output.
    """
    mine = run(*[t if a is None else shard(t, a, rank, world) for t, a in zip(inputs, axes)])
    single = not isinstance(mine, (tuple, list))
    mine = (mine,) if single else tuple(mine)
    oax = (out_axis,) if single else tuple(out_axis)
    if len(oax) != len(mine):
        raise ValueError(f"{len(mine)} outputs but {len(oax)} output axes")
    full = [gather_channels(m, a, world, group) for m, a in zip(mine, oax)]
    ok = True
    if rank == 0:
        ref = run(*inputs)
        ref = (ref,) if single else tuple(ref)
        ok = all(f.shape == r.shape and torch.equal(f, r.contiguous()) for f, r in zip(full, ref))
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())
