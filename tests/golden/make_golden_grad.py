"""Generate golden KDA gradients from the reference implementation's autograd.

Run in a checkout that has the reference source (Lazy-Hakimi/-kimi-linear-)::

    python tests/golden/make_golden_grad.py --reference <path-to-reference-checkout>

For every case it draws seeded inputs with ``synth.make_inputs`` plus seeded
output gradients ``do`` / ``dS``, runs the reference's ``kda_recurrent``
(``kimi_linear/kda.py:188``) -- or ``kda_chunkwise`` (``kda.py:58``) where the
case says so -- on CPU tensors with ``requires_grad``, calls
``torch.autograd.backward`` on ``(o, S)`` with ``(do, dS)`` and stores inputs
and the leaf gradients in ``tests/golden/grad_<case>.npz``.  bf16 values are
stored as float32 arrays (exact); gradients are stored in the leaf's dtype
rounded the same way.

Consumed by ``tests/test_oracle_grad_golden.py`` (pins the numpy backward
oracle) and ``tests/test_gpu_grad.py`` (pins the ``kda_backward`` kernel).
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

# name: (fn, B, T, H, K, V, chunk, dtype, s0_std, state_dtype, with_dS)
CASES = {
    # config-0 head shape, several 64-step checkpoints and a ragged tail
    "grad_f32_k32_t150": ("rec", 1, 150, 2, 32, 32, None, torch.float32, 0.02, None, True),
    # K != V, no initial state, no state gradient
    "grad_f32_k64_v32": ("rec", 1, 70, 2, 64, 32, None, torch.float32, None, None, False),
    # the 1.5B head shape
    "grad_f32_k128": ("rec", 1, 66, 1, 128, 128, None, torch.float32, 0.02, None, True),
    # fp16 activations, fp32 master state
    "grad_f16_k128": ("rec", 1, 40, 2, 128, 64, None, torch.float16, 0.02, torch.float32,
                      True),
    # bf16 activations, fp32 master state
    "grad_bf16_k64": ("rec", 2, 33, 2, 64, 64, None, torch.bfloat16, 0.02, torch.float32,
                      True),
    # autograd through the chunkwise kernel (the function the prefill path
    # runs).  chunk 16: with 64-token chunks these gates span more than 88 in
    # cumulative log decay inside a chunk, and the reference's fp32 path
    # overflows exp() in masked entries (kda.py:159-162 clamps for fp16 only),
    # which turns 2-30% of its dq/dk/dg/dbeta into NaN; at 16 it stays finite
    "grad_chunk_f32_k64": ("chunk", 1, 128, 1, 64, 64, 16, torch.float32, 0.02, None, True),
}


def _np(t):
    if t is None:
        return None
    return t.detach().float().numpy() if t.dtype != torch.float32 else t.detach().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the reference checkout (contains kimi_linear/)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, REPO)
    kda = importlib.import_module("kimi_linear.kda")
    synth = importlib.import_module("-kimi-linear-_b200.synth")
    torch.set_num_threads(os.cpu_count() or 1)
    dname = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}
    for name, (fn, B, T, H, K, V, C, dt, s0, sdt, with_dS) in CASES.items():
        x = synth.make_inputs(B, T, H, K, V, dtype=dt, seed=0, s0_std=s0)
        gen = torch.Generator().manual_seed(1)
        do = torch.randn(B, T, H, V, generator=gen).to(dt)
        dS = torch.randn(B, H, K, V, generator=gen) * 0.1 if with_dS else None
        leaves = {n: x[n].clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")}
        S0 = x["S0"].clone().requires_grad_(True) if x["S0"] is not None else None
        if fn == "rec":
            o, S = kda.kda_recurrent(leaves["q"], leaves["k"], leaves["v"], leaves["g"],
                                     leaves["beta"], state=S0, state_dtype=sdt)
        else:
            o, S = kda.kda_chunkwise(leaves["q"], leaves["k"], leaves["v"], leaves["g"],
                                     leaves["beta"], initial_state=S0, chunk_size=C,
                                     state_dtype=sdt)
        outs, grads = [o], [do]
        if dS is not None:
            outs.append(S)
            grads.append(dS.to(S.dtype))
        torch.autograd.backward(outs, grads)
        arrays = {n: _np(x[n]) for n in ("q", "k", "v", "g", "beta")}
        arrays["do"] = _np(do)
        if dS is not None:
            arrays["dS"] = _np(dS.to(S.dtype))
        if S0 is not None:
            arrays["S0"] = _np(x["S0"])
            arrays["dS0"] = _np(S0.grad)
        for n in ("q", "k", "v", "g", "beta"):
            arrays[f"d{n}"] = _np(leaves[n].grad)
        meta = np.array([B, T, H, K, V, -1 if C is None else C], dtype=np.int64)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"), meta=meta, fn=np.array(fn),
            dtype=np.array(dname[dt]),
            state_dtype=np.array("" if sdt is None else dname[sdt]), **arrays)
        print(f"{name}: wrote {sorted(arrays)}")


if __name__ == "__main__":
    main()
