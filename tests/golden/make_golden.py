"""Generate the golden KDA vectors from the reference implementation itself.

Run in a checkout that has the reference source (Lazy-Hakimi/-kimi-linear-)
importable; the default location is the ``--reference`` argument::

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

For every case it draws seeded inputs with ``synth.make_inputs`` and calls the
reference's ``kimi_linear.kda.kda_chunkwise`` (``kda.py:58``) and
``kimi_linear.kda.kda_recurrent`` (``kda.py:188``) on CPU tensors, then stores
inputs and outputs in ``tests/golden/<case>.npz``.  bf16 tensors are stored as
float32 arrays (exact).  The reference chunkwise kernel raises on bf16 values
(``kda.py:173``), so its bf16 golden output is the reference run on the
fp32-upcast bf16 values with the output rounded to bf16 -- the arithmetic
``kda.py:116`` intends for non-fp16 inputs.

The files are consumed by ``tests/test_oracle_golden.py`` (pins the numpy
oracle) and ``tests/test_gpu_parity.py`` (pins the CUDA kernels).
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

# name: (B, T, H, K, V, chunk, dtype, s0_std, state_dtype)
CASES = {
    # BASELINE config 0 exactly: fp32, S0 = 0, seed 0
    "c0_f32": (2, 256, 2, 32, 32, 64, torch.float32, None, None),
    # config 0 shapes with a non-zero initial state (Eq. 8 carry-in)
    "c0_f32_s0": (2, 256, 2, 32, 32, 64, torch.float32, 0.02, None),
    # fp16 q/k/v, fp32 master state, the reference's fp16-transient path
    "f16_k64_c64": (1, 128, 2, 64, 64, 64, torch.float16, 0.02, torch.float32),
    # the 1.5B head shape, two chunks
    "f16_k128_c64": (1, 128, 2, 128, 128, 64, torch.float16, 0.02, torch.float32),
    # tiny-config chunk size, fp16 state returned (state_dtype=None)
    "f16_c16_f16state": (2, 48, 2, 32, 32, 16, torch.float16, None, None),
    # chunk 128 (the 1.5B config's chunk_size), fp32
    "f32_c128": (1, 256, 1, 64, 64, 128, torch.float32, 0.02, None),
    # T < chunk: the module passes C = T (kda.py:513-514)
    "f32_c40": (1, 40, 2, 32, 32, 40, torch.float32, None, None),
    # K != V
    "f32_k32_v64": (1, 64, 2, 32, 64, 32, torch.float32, 0.02, None),
    # bf16 q/k/v with fp32 state; odd T for the recurrent kernel
    "bf16_k64": (2, 64, 2, 64, 64, 32, torch.bfloat16, 0.02, torch.float32),
}
# cases whose q/k/v/g/beta are those of another case (loaded from there)
SHARED_INPUTS = {"c0_f32_s0": "c0_f32"}
# recurrent-only cases (T not a multiple of any chunk)
REC_CASES = {
    "rec_f32_t37": (2, 37, 2, 32, 32, None, torch.float32, 0.02, None),
    "rec_bf16_t5": (1, 5, 3, 64, 32, None, torch.bfloat16, 0.02, torch.float32),
    "rec_f16_t1": (2, 1, 2, 128, 128, None, torch.float16, 0.02, torch.float32),
}


def _np(t):
    if t is None:
        return None
    return t.detach().float().numpy() if t.dtype == torch.bfloat16 else t.detach().numpy()


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
    for name, (B, T, H, K, V, C, dt, s0, sdt) in {**CASES, **REC_CASES}.items():
        x = synth.make_inputs(B, T, H, K, V, dtype=dt, seed=0, s0_std=s0)
        rec = {}
        o_r, S_r = kda.kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                     state=x["S0"], state_dtype=sdt)
        rec.update(o_rec=_np(o_r), S_rec=_np(S_r))
        if C is not None:
            if dt == torch.bfloat16:
                o_c, S_c = kda.kda_chunkwise(x["q"].float(), x["k"].float(), x["v"].float(),
                                             x["g"], x["beta"], initial_state=x["S0"],
                                             chunk_size=C, state_dtype=sdt)
                o_c = o_c.to(torch.bfloat16)
            else:
                o_c, S_c = kda.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                                             initial_state=x["S0"], chunk_size=C,
                                             state_dtype=sdt)
            rec.update(o_chunk=_np(o_c), S_chunk=_np(S_c))
        arrays = {k: _np(v) for k, v in x.items() if v is not None}
        if name in SHARED_INPUTS:
            # same seed and draw order as the named case: q..beta are identical,
            # only S0 (drawn last) is new, so the inputs are not stored twice
            arrays = {"S0": arrays["S0"]}
        arrays.update(rec)
        meta = np.array([B, T, H, K, V, -1 if C is None else C], dtype=np.int64)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"), meta=meta,
            dtype=np.array(dname[dt]),
            state_dtype=np.array("" if sdt is None else dname[sdt]),
            s0=np.array(s0 is not None),
            inputs_from=np.array(SHARED_INPUTS.get(name, "")), **arrays)
        print(f"{name}: wrote {sorted(arrays)}")


if __name__ == "__main__":
    main()
