"""Batch x head sharding with a final gather (``sharding.py``), on CPU.

Two to four ``gloo`` ranks (spawned processes) each compute their slice of one
``kda_chunkwise`` job and gather ``o`` and ``S`` to rank 0, which compares
them with the unsharded result.  The per-shard compute is the numpy oracle
(the CUDA kernels need a GPU); what is under test is the host logic: the
split, the views, and the point-to-point gather, including uneven and
head-wise splits and a rank that fails before the gather.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch

from conftest import REPO, pkg

CASES = [
    # (B, T, H, world): batch even, heads (B odd), uneven batch, heads with B=1
    (4, 32, 2, 2),
    (3, 32, 2, 2),
    (3, 32, 3, 2),
    (1, 32, 4, 4),
]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_fn(q, k, v, g, beta, initial_state=None, chunk_size=16, state_dtype=None):
    from oracle import kda_oracle as O
    B, T, H, K = q.shape
    V = v.shape[-1]
    if B == 0 or H == 0:
        return (torch.empty(B, T, H, V), torch.empty(B, H, K, V))
    s0 = None if initial_state is None else initial_state.numpy()
    o, S = O.kda_chunkwise(q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta.numpy(),
                           initial_state=s0, chunk_size=chunk_size, state_dtype="f32")
    return torch.from_numpy(np.ascontiguousarray(o)), torch.from_numpy(np.ascontiguousarray(S))


def _worker(rank, world, port, case, mode, out_path):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "tests"))
    ok = False
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=10))
        kb = pkg()
        B, T, H = case
        x = kb.synth.make_inputs(B, T, H, 16, 16, dtype=torch.float32, seed=3, s0_std=0.02)
        if mode == "lost" and rank == 1:
            raise SystemExit(3)           # leaves before the gather, on the host
        o, S, shard = kb.sharding.chunkwise_sharded(
            x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], chunk_size=16,
            rank=rank, world=world, fn=_oracle_fn, segments=2 if mode == "seg" else 1)
        if rank == 0:
            o_ref, S_ref = _oracle_fn(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"],
                                      chunk_size=16)
            assert o.shape == o_ref.shape and S.shape == S_ref.shape
            # time segments restart the chunk loop from a carried state: equal
            # to rounding only (fp32 everywhere here)
            tol = 0.0 if mode != "seg" else 1e-5
            assert torch.allclose(o, o_ref, rtol=0, atol=tol), float((o - o_ref).abs().max())
            assert torch.allclose(S, S_ref, rtol=0, atol=tol), float((S - S_ref).abs().max())
            assert shard.dim == kb.sharding.plan(B, H, world, 0).dim
        else:
            assert o is None and S is None
        ok = True
    except SystemExit:
        raise
    except Exception:
        if mode != "lost":
            traceback.print_exc()
    finally:
        if rank == 0:
            with open(out_path, "w") as f:
                f.write("ok" if ok else "failed")
    sys.exit(0 if ok else 1)


def _run(world, case, mode, tmp_path):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = str(tmp_path / f"r0_{mode}.txt")
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, mode, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs], open(out).read() if os.path.exists(out) else ""


@pytest.mark.parametrize("case", CASES)
def test_sharded_equals_unsharded(case, tmp_path):
    B, T, H, world = case
    codes, r0 = _run(world, (B, T, H), "ok", tmp_path)
    assert r0 == "ok" and codes == [0] * world, (codes, r0)


@pytest.mark.parametrize("case", [CASES[0], CASES[3]])
def test_segmented_gather_overlapping_compute(case, tmp_path):
    """Two time segments per rank, the first one's outputs sent while the
    second computes (batch and head splits)."""
    B, T, H, world = case
    codes, r0 = _run(world, (B, T, H), "seg", tmp_path)
    assert r0 == "ok" and codes == [0] * world, (codes, r0)


def test_lost_rank_fails_the_gather_instead_of_hanging(tmp_path):
    """Rank 1 exits before its send: rank 0's receive must end with an error
    (process-group timeout or closed connection), not wait forever."""
    codes, r0 = _run(2, (4, 32, 2), "lost", tmp_path)
    assert codes[1] == 3
    assert codes[0] == 1 and r0 == "failed", (codes, r0)


def test_plan_and_bounds():
    S = pkg().sharding
    assert [S.bounds(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert S.bounds(2, 4, 3) == (2, 2)                          # empty shard
    assert S.plan(8, 16, 8, 5).dim == "batch" and S.plan(8, 16, 8, 5).size == 1
    assert S.plan(1, 16, 8, 0).dim == "head" and S.plan(1, 16, 8, 0).size == 2
    assert S.plan(3, 5, 2, 1).dim == "batch"
    covered = sorted(i for r in range(3) for i in range(*S.bounds(7, 3, r)))
    assert covered == list(range(7))
    x = torch.arange(2 * 3 * 4 * 5).reshape(2, 3, 4, 5)
    sh = S.Shard("head", 1, 3, 2, 0)
    assert S.take(x, sh, "seq").shape == (2, 3, 2, 5)
    assert S.take(x, sh, "state").shape == (2, 2, 4, 5)
    with pytest.raises(ValueError):
        S.bounds(4, 2, 2)
