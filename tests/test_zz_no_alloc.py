"""The allocation-free chunkwise entry point, checked against the normal one.

``kda_chunkwise_fwd_noalloc`` exists for callers that must not allocate device
memory while running: a host that reserves all of its GPU memory up front, an
engine plugin whose enqueue step may not call cudaMalloc, or a C caller with
no device allocator.  Instead of a caller-provided workspace it uses a fixed
32 MiB scratch array inside the library.  This test calls it through the C ABI
twice in a row on the same inputs (the second call runs on the scratch the
first one left behind) and compares both results with ``kda_chunkwise_fwd``
within the parity tolerance of the GPU tests (2e-3 relative for fp16 inputs
with an fp32 state).  It also checks that a problem too large for the scratch
is refused with KDA_ERR_WORKSPACE instead of running.

The file name sorts last, so a run that stops at the first failure has already
run every other test; the tests also pass on their own in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def _noalloc_call(kb, x, dev):
    """Outputs are allocated here by the test; the entry point allocates nothing."""
    ops, lib = kb.ops, kb._lib
    _, q, k, v, g, beta, s0, o, S = ops._prepare(
        "noalloc", x["q"], x["k"], x["v"], x["g"], x["beta"], x["S0"], torch.float32)
    args = lib.KdaArgs()
    ops._fill(args, q, k, v, g, beta, s0, o, S, 64)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = lib.load().kda_chunkwise_fwd_noalloc(ctypes.byref(args), ctypes.c_void_p(stream))
    return st, o, S


def test_noalloc_entry_point_matches_allocating_one(cuda_dev):
    kb = pkg()
    x = kb.synth.make_inputs(2, 448, 4, 128, 128, dtype=torch.float16, seed=21, s0_std=0.02,
                             device=cuda_dev)
    assert kb.chunkwise_path(x["q"], x["k"], x["v"], x["g"], x["beta"],
                             initial_state=x["S0"], state_dtype=torch.float32) == "tcgen05"
    o_ref, S_ref = kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                    initial_state=x["S0"], state_dtype=torch.float32)
    for _ in range(2):
        st, o, S = _noalloc_call(kb, x, cuda_dev)
        assert st == 0, kb._lib.status_string(st)
        torch.cuda.synchronize()
        assert _rel(o, o_ref) < 2e-3
        assert _rel(S, S_ref) < 2e-3
    assert kb.device_error() == 0


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_dev):
    """The scratch holds 407 chunk images of 64 rows (82,432 bytes each): one
    head of 407 x 64 tokens runs, one of 408 x 64 tokens is refused."""
    kb = pkg()
    for n_chunks, ok in ((407, True), (408, False)):
        x = kb.synth.make_inputs(1, 64 * n_chunks, 1, 128, 128, dtype=torch.float16,
                                 seed=22, device=cuda_dev)
        st, o, S = _noalloc_call(kb, x, cuda_dev)
        if ok:
            assert st == 0, kb._lib.status_string(st)
            o_ref, S_ref = kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                            state_dtype=torch.float32)
            torch.cuda.synchronize()
            assert _rel(o, o_ref) < 2e-3 and _rel(S, S_ref) < 2e-3
        else:
            assert st == kb._lib.KDA_ERR_WORKSPACE
