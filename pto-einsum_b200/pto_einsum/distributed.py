"""Batch-axis sharding of one einsum over the GPUs of a node.

One process per GPU (torchrun). The output's leading axis is split into
contiguous, near-equal shards, one per rank; every operand that carries that
axis is sliced the same way, operands without it are replicated. Each rank
runs the ordinary single-GPU path on its shard: there is no collective on the
data path. ``gather=True`` (off by default) assembles the full result on
every rank with one all-gather (NCCL over NVLink on GPUs, gloo on CPU),
padded to equal shard sizes and trimmed afterwards.

The reference is single-device; this module has no reference counterpart.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence, Tuple

import torch

from .planner import split_equation


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[begin, end) of rank's contiguous share of n items (sizes differ by <= 1)."""
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_plan(equation: str, shape0: Sequence[int], shape1: Sequence[int]):
    """Sharded axis of each operand: (label, axis in in0 or None, axis in in1 or None, size)."""
    a, b, o = split_equation(equation)
    if not o:
        raise ValueError(f"'{equation}' has a scalar output; nothing to shard")
    label = o[0]
    ax0 = a.index(label) if label in a else None
    ax1 = b.index(label) if label in b else None
    size = shape0[ax0] if ax0 is not None else shape1[ax1]
    return label, ax0, ax1, int(size)


def shard_operands(equation: str, a: torch.Tensor, b: torch.Tensor, rank: int, world: int):
    """Slice the operands for `rank` (contiguous shards of the output's leading axis)."""
    _, ax0, ax1, size = shard_plan(equation, a.shape, b.shape)
    lo, hi = shard_bounds(size, world, rank)
    if ax0 is not None:
        a = a.narrow(ax0, lo, hi - lo)
    if ax1 is not None:
        b = b.narrow(ax1, lo, hi - lo)
    return a.contiguous(), b.contiguous()


def sharded_einsum(equation: str, a_local: torch.Tensor, b_local: torch.Tensor, *, full_size: int,
                   gather: bool = False, group=None,
                   compute: Optional[Callable[[str, torch.Tensor, torch.Tensor], torch.Tensor]] = None):
    """Run this rank's shard; optionally all-gather the full output.

    `full_size` is the unsharded length of the output's leading axis. `compute`
    defaults to the CUDA einsum of this package.
    """
    import torch.distributed as dist
    if compute is None:
        from .builder import einsum as compute
    out = compute(equation, a_local, b_local)
    if not gather:
        return out
    world = dist.get_world_size(group)
    rest = tuple(out.shape[1:])
    shard = -(-full_size // world)
    if full_size % world == 0:
        # equal shards: gather straight into the result, no padding or copies
        full = torch.empty((full_size,) + rest, dtype=out.dtype, device=out.device)
        _all_gather_into(full, out.contiguous(), group)
        return full
    # unequal shards: gather padded shards, then drop each rank's padding
    pad = torch.zeros((shard,) + rest, dtype=out.dtype, device=out.device)
    pad[: out.shape[0]] = out
    buf = torch.empty((world * shard,) + rest, dtype=out.dtype, device=out.device)
    _all_gather_into(buf, pad, group)
    pieces = []
    for r in range(world):
        lo, hi = shard_bounds(full_size, world, r)
        pieces.append(buf[r * shard: r * shard + (hi - lo)])
    return torch.cat(pieces, dim=0)


def _all_gather_into(dst: torch.Tensor, src: torch.Tensor, group) -> None:
    """dst = concatenation of every rank's src along dim 0 (one collective)."""
    import torch.distributed as dist
    try:
        dist.all_gather_into_tensor(dst, src, group=group)
    except (RuntimeError, NotImplementedError):
        # backends without the fused form (older gloo): gather into views of dst
        dist.all_gather(list(dst.chunk(dist.get_world_size(group), dim=0)), src, group=group)
