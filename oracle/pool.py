"""Run the KDA oracle over many (b, h) recurrences at once -- TEST INFRASTRUCTURE.

Every (b, h) head of ``kda_chunkwise`` (``kimi_linear/kda.py:58-185``) is an
independent recurrence (no term of ``kda.py:140-182`` couples heads or batch
rows), so the oracle of a large case can be split per head and run on several
host cores.  Workers are started with the ``spawn`` method, which is safe after
CUDA has been initialised in the parent.

Used by the full-size parity tests and by the CPU legs of ``bench.py``; the
product path never imports it.
"""

from __future__ import annotations

import os

import numpy as np

from . import kda_oracle as O


def _one_head(args):
    q, k, v, g, beta, s0, chunk_size, state_dtype, v_dtype = args
    return O.kda_chunkwise(q, k, v, g, beta, initial_state=s0, chunk_size=chunk_size,
                           state_dtype=state_dtype, v_dtype=v_dtype)


def chunkwise_by_head(q, k, v, g, beta, initial_state=None, chunk_size=64, state_dtype=None,
                      v_dtype=None, procs=None):
    """``kda_oracle.kda_chunkwise`` evaluated head by head in a spawn pool.

    Arguments and results are those of ``kda_oracle.kda_chunkwise`` (numpy
    arrays ``[B,T,H,D]``, ``[B,T,H]``, ``[B,H,K,V]``).  ``procs`` defaults to the
    host's core count (at most the number of heads).
    """
    import multiprocessing as mp
    from concurrent.futures import ProcessPoolExecutor

    B, T, H, _ = q.shape
    jobs = []
    for b in range(B):
        for h in range(H):
            s0 = None if initial_state is None else initial_state[b:b + 1, h:h + 1]
            jobs.append((q[b:b + 1, :, h:h + 1], k[b:b + 1, :, h:h + 1], v[b:b + 1, :, h:h + 1],
                         g[b:b + 1, :, h:h + 1], beta[b:b + 1, :, h:h + 1], s0, chunk_size,
                         state_dtype, v_dtype))
    n = max(1, min(procs or os.cpu_count() or 1, len(jobs)))
    if n == 1:
        res = [_one_head(j) for j in jobs]
    else:
        # one BLAS thread per worker: the workers already fill the cores
        keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
        old = {key: os.environ.get(key) for key in keys}
        os.environ.update({key: "1" for key in keys})
        try:
            # an executor raises (BrokenProcessPool) when a worker cannot start,
            # where a multiprocessing.Pool would keep respawning it forever
            with ProcessPoolExecutor(n, mp_context=mp.get_context("spawn")) as ex:
                res = list(ex.map(_one_head, jobs))
        finally:
            for key, val in old.items():
                if val is None:
                    os.environ.pop(key, None)
                else:
                    os.environ[key] = val
    V = v.shape[-1]
    K = q.shape[-1]
    o = np.empty((B, T, H, V), dtype=res[0][0].dtype)
    S = np.empty((B, H, K, V), dtype=res[0][1].dtype)
    for i, (oh, Sh) in enumerate(res):
        b, h = divmod(i, H)
        o[b, :, h] = oh[0, :, 0]
        S[b, h] = Sh[0, 0]
    return o, S
