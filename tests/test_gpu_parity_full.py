"""GPU parity against the oracle at the full BASELINE sizes, and on the rare
branch of the tensor-core path that handles steep decays.

* configs[1] exactly: B=1, T=4096, H=16, K=V=128, fp16 q/k/v, zero S0, fp32
  state (``kimi_linear/kda.py:58-185`` with its fp16-transient arithmetic,
  restated by ``oracle/kda_oracle.py``).
* configs[3] at its full sequence length: one batch row of B=8, T=32768,
  H=16, bf16 q/k/v, S0 ~ N(0, 0.02) in fp32.  The reference crashes on bf16
  ``kda_chunkwise`` inputs (``kda.py:173``); its oracle runs the bf16 values
  through the fp32-transient path ``kda.py:116`` intends and rounds the output
  to bf16.  This pins the long carry of the fp32 state through 512 chunks.
* steep decays: gates scaled so that the total decay of many 16-row blocks is
  below -80 (the tensor-core prep takes those channels out of the blocked
  Gram product and adds their exact pair terms, ``kda.py:153-168``).

The oracle runs head by head in a spawn pool (``oracle/pool.py``).  Bars are
those of the task: 2e-3 relative Frobenius error on o and on S for fp16/bf16
inputs with an fp32 state.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import pool as OP

pytestmark = pytest.mark.gpu

TOL = 2e-3


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return ((a - b).norm() / b.norm()).item()


def _np(t):
    return None if t is None else t.detach().float().cpu().numpy()


def test_config1_exact_vs_oracle(cuda_dev):
    kb = pkg()
    x = kb.synth.make_config(1, seed=3)                 # B=1, T=4096, H=16, fp16
    ro, rS = OP.chunkwise_by_head(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(),
                                  x["g"].numpy(), x["beta"].numpy(), chunk_size=64,
                                  state_dtype="f32")
    d = {n: t.to(cuda_dev) for n, t in x.items() if t is not None}
    assert kb.chunkwise_path(d["q"], d["k"], d["v"], d["g"], d["beta"],
                             state_dtype=torch.float32) == "tcgen05"
    o, S = kb.kda_chunkwise(d["q"], d["k"], d["v"], d["g"], d["beta"], chunk_size=64,
                            state_dtype=torch.float32)
    eo, eS = rel(o.float(), ro.astype(np.float32)), rel(S, rS)
    assert eo < TOL, eo
    assert eS < TOL, eS


def test_config3_full_length_one_batch_row_vs_oracle(cuda_dev):
    kb = pkg()
    x = kb.synth.make_config(3, seed=5, B=1, device=cuda_dev)   # T=32768, H=16, bf16, S0
    assert x["q"].dtype == torch.bfloat16 and x["S0"] is not None
    ro, rS = OP.chunkwise_by_head(_np(x["q"]), _np(x["k"]), _np(x["v"]), _np(x["g"]),
                                  _np(x["beta"]), initial_state=_np(x["S0"]), chunk_size=64,
                                  state_dtype="f32", v_dtype="bf16")
    assert kb.chunkwise_path(x["q"], x["k"], x["v"], x["g"], x["beta"],
                             initial_state=x["S0"], state_dtype=torch.float32) == "tcgen05"
    o, S = kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                            initial_state=x["S0"], chunk_size=64, state_dtype=torch.float32)
    eo, eS = rel(o.float(), ro), rel(S, rS)
    assert eo < TOL, eo
    assert eS < TOL, eS


def _steep_blocks(g, limit=80.0):
    """Number of (b, h, 16-row block, channel) whose total decay, from the
    block's first row to the next block's first row, is below -limit (the
    prep kernel's test; the last block of a chunk stops at the chunk end)."""
    B, T, H, K = g.shape
    x = g.double().reshape(B, T // 64, 4, 16, H, K)
    z = x[:, :, :, 1:].sum(3)                                   # rows 16r+1 .. 16r+15
    nxt = torch.zeros_like(x[:, :, :, 0])
    nxt[:, :, :3] = x[:, :, 1:, 0]                              # row 16r+16 (same chunk)
    return int(((z + nxt) < -limit).sum())


@pytest.mark.parametrize("dtype,scale", [(torch.float16, 3.0), (torch.float16, 12.0),
                                         (torch.bfloat16, 5.0)])
def test_steep_decay_blocks_vs_oracle(dtype, scale, cuda_dev):
    kb = pkg()
    x = kb.synth.make_inputs(1, 512, 2, 128, 128, dtype=dtype, seed=41, s0_std=0.02)
    x["g"] = x["g"] * scale
    n_steep = _steep_blocks(x["g"])
    total = x["g"].numel() // 16
    assert 0 < n_steep < total, (n_steep, total)                # both branches run
    vd = "bf16" if dtype == torch.bfloat16 else None
    ro, rS = OP.chunkwise_by_head(_np(x["q"]) if vd else x["q"].numpy(),
                                  _np(x["k"]) if vd else x["k"].numpy(),
                                  _np(x["v"]) if vd else x["v"].numpy(),
                                  x["g"].numpy(), x["beta"].numpy(),
                                  initial_state=x["S0"].numpy(), chunk_size=64,
                                  state_dtype="f32", v_dtype=vd)
    d = {n: t.to(cuda_dev) for n, t in x.items()}
    assert kb.chunkwise_path(d["q"], d["k"], d["v"], d["g"], d["beta"],
                             initial_state=d["S0"], state_dtype=torch.float32) == "tcgen05"
    o, S = kb.kda_chunkwise(d["q"], d["k"], d["v"], d["g"], d["beta"], initial_state=d["S0"],
                            chunk_size=64, state_dtype=torch.float32)
    eo, eS = rel(o.float(), ro.astype(np.float32)), rel(S, rS)
    assert eo < TOL, eo
    assert eS < TOL, eS
    assert kb.device_error() == 0
