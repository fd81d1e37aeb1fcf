"""Batch x head sharding of the KDA core over the GPUs of one node.

Every (batch, head) recurrence of ``kda_chunkwise`` / ``kda_recurrent`` is
independent (``kimi_linear/kda.py:140-182`` and ``:207-216`` mix no heads and
no sequences), so a job splits into contiguous slices of the batch -- or, when
the batch does not divide evenly and the heads do, of the heads -- with no
collective on the data path.  The only exchange is the optional final gather
of the outputs and final states to one rank (point-to-point sends over
NCCL/NVLink on GPUs, gloo on CPU).

One process per GPU (``torchrun``); ``torch.distributed`` supplies the ranks.
The functions here are plain host logic on tensors; which kernel computes a
shard is the caller's choice (``fn``), by default :func:`ops.kda_chunkwise`.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Shard:
    """The slice ``[start, stop)`` of dimension ``dim`` ("batch" or "head")
    that rank ``rank`` of ``world`` owns."""

    dim: str
    start: int
    stop: int
    world: int
    rank: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Balanced contiguous split of ``n`` items: the first ``n % world``
    ranks get one item more.  Ranks past ``n`` get an empty range."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def plan(B: int, H: int, world: int, rank: int) -> Shard:
    """Which dimension to split: the batch when it divides evenly (whole
    sequences per rank, contiguous in every tensor), else the heads when they
    do, else whichever is at least ``world`` long (uneven split), else the
    longer one."""
    if B % world == 0:
        dim = "batch"
    elif H % world == 0:
        dim = "head"
    elif B >= world:
        dim = "batch"
    elif H >= world:
        dim = "head"
    else:
        dim = "batch" if B >= H else "head"
    start, stop = bounds(B if dim == "batch" else H, world, rank)
    return Shard(dim, start, stop, world, rank)


def take(x, shard: Shard, kind: str):
    """This rank's view of a full tensor.  ``kind`` "seq" for ``[B, T, H, ...]``
    (q, k, v, g, beta, o) and "state" for ``[B, H, K, V]``."""
    if x is None:
        return None
    if shard.dim == "batch":
        return x[shard.start:shard.stop]
    if kind == "seq":
        return x[:, :, shard.start:shard.stop]
    if kind == "state":
        return x[:, shard.start:shard.stop]
    raise ValueError(f"unknown tensor kind {kind!r}")


def plan_like(q, world: int, rank: int) -> Shard:
    """:func:`plan` for the shape of ``q`` ``[B, T, H, K]``."""
    return plan(q.shape[0], q.shape[2], world, rank)


def gather(local, full_shape, shard: Shard, kind: str, dst: int = 0, group=None):
    """Collect every rank's ``local`` slice into a full tensor on rank ``dst``.

    Point-to-point: each other rank sends its slice (made contiguous) once;
    ``dst`` receives each directly into the full tensor when that slice is
    contiguous there (batch shards) and through a staging buffer otherwise
    (head shards).  Returns the full tensor on ``dst`` and ``None`` elsewhere.
    Every rank must call it with the same ``full_shape``, ``kind`` and ``dst``.
    """
    import torch.distributed as dist

    world, rank = shard.world, shard.rank
    if world == 1:
        return local
    if rank != dst:
        if local.numel():
            dist.send(local.contiguous(), dst, group=group)
        return None
    full = torch.empty(full_shape, dtype=local.dtype, device=local.device)
    take(full, shard, kind).copy_(local)
    for r in range(world):
        if r == dst:
            continue
        other = Shard(shard.dim, *bounds(full_shape[0] if shard.dim == "batch" else
                                         full_shape[2 if kind == "seq" else 1], world, r),
                      world, r)
        view = take(full, other, kind)
        if view.numel() == 0:
            continue
        if view.is_contiguous():
            dist.recv(view, r, group=group)
        else:
            buf = torch.empty(view.shape, dtype=view.dtype, device=view.device)
            dist.recv(buf, r, group=group)
            view.copy_(buf)
    return full


def chunkwise_sharded(q, k, v, g, beta, initial_state=None, chunk_size=64, state_dtype=None,
                      *, rank: int, world: int, group=None, gather_to: int | None = 0, fn=None):
    """Run this rank's share of one ``kda_chunkwise`` job over full-size inputs.

    Every rank passes the same full tensors (e.g. generated from one seed);
    the rank computes only its slice with ``fn`` (default
    :func:`ops.kda_chunkwise`).  With ``gather_to`` set, the outputs and final
    states are gathered to that rank, which returns the full ``(o, S)``; the
    other ranks return ``(None, None)``.  With ``gather_to=None`` every rank
    returns its own ``(o, S)`` slice.  Returns ``(o, S, shard)``.
    """
    if fn is None:
        from .ops import kda_chunkwise as fn
    shard = plan_like(q, world, rank)
    args = [take(t, shard, "seq") for t in (q, k, v, g, beta)]
    s0 = take(initial_state, shard, "state")
    o, S = fn(*args, initial_state=s0, chunk_size=chunk_size, state_dtype=state_dtype)
    if gather_to is None:
        return o, S, shard
    B, T, H = q.shape[:3]
    V, K = v.shape[-1], q.shape[-1]
    o_full = gather(o, (B, T, H, V), shard, "seq", dst=gather_to, group=group)
    S_full = gather(S, (B, H, K, V), shard, "state", dst=gather_to, group=group)
    return o_full, S_full, shard
