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


def _shard_of(full_shape, shard: Shard, kind: str, r: int) -> Shard:
    """Rank ``r``'s shard of a full tensor of ``full_shape`` (same split as ``shard``)."""
    n = full_shape[0] if shard.dim == "batch" else full_shape[2 if kind == "seq" else 1]
    return Shard(shard.dim, *bounds(n, shard.world, r), shard.world, r)


def gather_many(items, shard: Shard, dst: int = 0, group=None):
    """Collect several sharded tensors on rank ``dst`` with all transfers in
    flight at once.

    ``items`` is a list of ``(local, full, kind, t_range)``: ``local`` this
    rank's slice, ``full`` the destination tensor on ``dst`` (ignored
    elsewhere), ``kind`` "seq" / "state", ``t_range`` ``(t0, t1)`` to place a
    time segment of a "seq" tensor (``None``: the whole time axis).  Every
    rank posts its sends and ``dst`` posts one receive per (item, peer) in a
    single ``batch_isend_irecv``, so the peers' slices arrive concurrently
    (NCCL runs the group as one launch) instead of one after another.
    Receives land in place when the destination view is contiguous and go
    through a staging buffer otherwise.  Returns the work handles and a list of
    ``(staging, view)`` copies that :func:`finish` completes; nothing is
    waited for here, so the caller can overlap the transfers with compute.
    """
    import torch.distributed as dist

    world, rank = shard.world, shard.rank
    ops, copies = [], []
    for local, full, kind, t_range in items:
        if rank != dst:
            if local.numel():
                ops.append(dist.P2POp(dist.isend, local.contiguous(), dst, group=group))
            continue
        for r in range(world):
            view = take(full, _shard_of(full.shape, shard, kind, r), kind)
            if t_range is not None:
                view = view[:, t_range[0]:t_range[1]]
            if r == rank:
                view.copy_(local)
                continue
            if view.numel() == 0:
                continue
            if view.is_contiguous():
                ops.append(dist.P2POp(dist.irecv, view, r, group=group))
            else:
                buf = torch.empty(view.shape, dtype=view.dtype, device=view.device)
                ops.append(dist.P2POp(dist.irecv, buf, r, group=group))
                copies.append((buf, view))
    works = dist.batch_isend_irecv(ops) if ops else []
    return works, copies


def finish(pending):
    """Wait for :func:`gather_many` transfers and place staged receives."""
    works, copies = pending
    for w in works:
        w.wait()
    for buf, view in copies:
        view.copy_(buf)


def gather(local, full_shape, shard: Shard, kind: str, dst: int = 0, group=None):
    """Collect every rank's ``local`` slice into a full tensor on rank ``dst``
    (:func:`gather_many` for one tensor, waited for).  Returns the full tensor
    on ``dst`` and ``None`` elsewhere.  Every rank must call it with the same
    ``full_shape``, ``kind`` and ``dst``."""
    if shard.world == 1:
        return local
    full = None
    if shard.rank == dst:
        full = torch.empty(full_shape, dtype=local.dtype, device=local.device)
    finish(gather_many([(local, full, kind, None)], shard, dst, group))
    return full


def chunkwise_sharded(q, k, v, g, beta, initial_state=None, chunk_size=64, state_dtype=None,
                      *, rank: int, world: int, group=None, gather_to: int | None = 0, fn=None,
                      segments: int = 1):
    """Run this rank's share of one ``kda_chunkwise`` job over full-size inputs.

    Every rank passes the same full tensors (e.g. generated from one seed);
    the rank computes only its slice with ``fn`` (default
    :func:`ops.kda_chunkwise`).  With ``gather_to`` set, the outputs and final
    states are gathered to that rank, which returns the full ``(o, S)``; the
    other ranks return ``(None, None)``.  With ``gather_to=None`` every rank
    returns its own ``(o, S)`` slice.  Returns ``(o, S, shard)``.

    ``segments > 1`` splits the time axis into that many pieces (at multiples
    of ``chunk_size``): piece i + 1 starts from piece i's final state, which is
    exact because the chunkwise recurrence carries only the state
    (``kda.py:140-182``), and piece i's outputs are sent while piece i + 1
    computes, so the gather overlaps the compute.
    """
    shard = plan_like(q, world, rank)
    local = [take(t, shard, "seq") for t in (q, k, v, g, beta)]
    o, S = run_shard(*local, take(initial_state, shard, "state"), shard=shard,
                     full_bth=tuple(q.shape[:3]), chunk_size=chunk_size,
                     state_dtype=state_dtype, group=group, gather_to=gather_to, fn=fn,
                     segments=segments)
    return o, S, shard


def run_shard(q, k, v, g, beta, s0, *, shard: Shard, full_bth, chunk_size=64, state_dtype=None,
              group=None, gather_to: int | None = 0, fn=None, segments: int = 1):
    """:func:`chunkwise_sharded` for a rank that already holds its slices
    (``q`` .. ``beta`` ``[B_r, T, H_r, D]``, ``s0`` ``[B_r, H_r, K, V]`` or None)
    of a job of full shape ``full_bth = (B, T, H)``.  Returns ``(o, S)``: the
    full tensors on ``gather_to``, ``(None, None)`` on the other ranks, or this
    rank's slices when ``gather_to`` is None."""
    if fn is None:
        from .ops import kda_chunkwise as fn
    B, T, H = full_bth
    V, K = v.shape[-1], q.shape[-1]
    world, rank = shard.world, shard.rank
    args = (q, k, v, g, beta)
    gathering = gather_to is not None and world > 1
    segments = max(1, min(int(segments), max(1, T // max(1, chunk_size))))
    if segments == 1 or not gathering:
        o, S = fn(*args, initial_state=s0, chunk_size=chunk_size, state_dtype=state_dtype)
        if not gathering:
            return o, S
        o_full = S_full = None
        if rank == gather_to:
            o_full = torch.empty((B, T, H, V), dtype=o.dtype, device=o.device)
            S_full = torch.empty((B, H, K, V), dtype=S.dtype, device=S.device)
        finish(gather_many([(o, o_full, "seq", None), (S, S_full, "state", None)], shard,
                           gather_to, group))
        return o_full, S_full
    # time segments at chunk boundaries
    nchunks = T // chunk_size
    cuts = [chunk_size * (nchunks * i // segments) for i in range(segments)] + [T]
    o_full = S_full = None
    pending = []
    S = s0
    for i in range(segments):
        t0, t1 = cuts[i], cuts[i + 1]
        o_i, S = fn(*(a[:, t0:t1] for a in args), initial_state=S, chunk_size=chunk_size,
                    state_dtype=state_dtype)
        if rank == gather_to and o_full is None:
            o_full = torch.empty((B, T, H, V), dtype=o_i.dtype, device=o_i.device)
        pending.append(gather_many([(o_i, o_full, "seq", (t0, t1))], shard, gather_to, group))
    if rank == gather_to:
        S_full = torch.empty((B, H, K, V), dtype=S.dtype, device=S.device)
    pending.append(gather_many([(S, S_full, "state", None)], shard, gather_to, group))
    for pnd in pending:
        finish(pnd)
    if rank != gather_to:
        return None, None
    return o_full, S_full
