"""Golden vectors for the fused KDA prologue / epilogue, made by the reference.

Run in a checkout that has the reference source importable::

    python tests/golden/make_golden_fused.py --reference <path-to-reference-checkout>

For each case it builds the reference's own ``KimiDeltaAttention``
(``kimi_linear/kda.py:331``) from the tiny test configuration with the KDA
head shape overridden, gives it seeded random weights, and runs its own
``_projections`` (``kda.py:399-461``) and ``_output`` (``kda.py:464-470``) on
CPU.  Stored per case (``tests/golden/fused_<case>.npz``):

* the projection-GEMM outputs the module computed (``q_in``, ``k_in``,
  ``v_in``, ``gk``, ``beta_logit``, ``og``) -- the inputs of the fused
  kernels, so a GPU test compares the kernels alone, not cuBLAS against CPU
  GEMMs;
* the module parameters the kernels read (conv weights and biases,
  ``A_log``, ``dt_bias``, the head-wise RMSNorm weight, eps values);
* the conv history passed in (if any) and the reference outputs ``q, k, v,
  g, beta`` and the new conv cache of ``_projections``;
* ``o_core`` (random, the input of ``_output``) and ``y``: the input the
  reference's ``_output`` hands to ``o_proj`` (captured with a forward hook).

bf16 tensors are stored as float32 arrays (exact).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import zlib

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (B, T, head_dim, heads, dtype, mode)  mode: prefill | history | decode
CASES = {
    "fused_f32_d32_prefill": (2, 40, 32, 2, torch.float32, "prefill"),
    "fused_f32_d128_history": (2, 19, 128, 2, torch.float32, "history"),
    "fused_f32_d128_decode": (3, 1, 128, 2, torch.float32, "decode"),
    "fused_bf16_d128_prefill": (1, 70, 128, 2, torch.bfloat16, "prefill"),
    "fused_bf16_d64_decode": (2, 1, 64, 3, torch.bfloat16, "decode"),
}


def _np(t):
    if t is None:
        return None
    t = t.detach()
    return t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    kda_mod = importlib.import_module("kimi_linear.kda")
    cfgmod = importlib.import_module("kimi_linear.configuration")
    with open(os.path.join(args.reference, "configs", "kimi_linear_tiny_test.json")) as f:
        base = json.load(f)

    for name, (B, T, hd, H, dt, mode) in CASES.items():
        vals = json.loads(json.dumps(base))
        la = vals["linear_attn"]
        la.update(num_heads=H, head_dim=hd, value_head_dim=hd)
        cfg = cfgmod.KimiLinearConfig(vals)
        gen = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        m = kda_mod.KimiDeltaAttention(cfg)
        with torch.no_grad():
            for p in m.parameters():
                p.copy_(torch.randn(p.shape, generator=gen) * 0.3)
            # the static decay parameters in their usual ranges
            m.A_log.copy_(torch.log(torch.empty(m.A_log.shape).uniform_(1, 16, generator=gen)))
            m.dt_bias.copy_(torch.log(torch.expm1(torch.empty(m.dt_bias.shape).uniform_(
                1e-3, 0.1, generator=gen))))
        m = m.to(dt)
        d = vals["hidden_size"]
        x = torch.randn(B, T, d, generator=gen).to(dt)
        keep = la["conv_size"] - 1
        D = H * hd
        hist = None
        if mode in ("history", "decode"):
            hist = {n: (torch.randn(B, keep, D, generator=gen) * 0.5).to(dt) for n in "qkv"}
        with torch.no_grad():
            q_in, k_in, v_in = m.in_proj_q(x), m.in_proj_k(x), m.in_proj_v(x)
            gk = m.gk_proj(x)
            beta_logit = m.beta_proj(x)
            og = m.og_proj(x)
            q, k, v, g, beta, new_conv = m._projections(
                x, conv_cache=hist, use_cache=mode != "prefill")
            o_core = (torch.randn(B, T, H, hd, generator=gen) * 0.5).to(dt)
            captured = {}
            h = m.o_proj.register_forward_hook(lambda mod, inp, out: captured.update(y=inp[0]))
            m._output(o_core, x)
            h.remove()
        arrays = dict(
            q_in=q_in, k_in=k_in, v_in=v_in, gk=gk, beta_logit=beta_logit, og=og,
            w_q=m.conv_q.conv.weight, w_k=m.conv_k.conv.weight, w_v=m.conv_v.conv.weight,
            b_q=m.conv_q.conv.bias, b_k=m.conv_k.conv.bias, b_v=m.conv_v.conv.bias,
            A_log=m.A_log, dt_bias=m.dt_bias, norm_w=m.g_norm.weight,
            q=q, k=k, v=v, g=g, beta=beta, o_core=o_core, y=captured["y"])
        if hist is not None:
            arrays.update(hist_q=hist["q"], hist_k=hist["k"], hist_v=hist["v"])
        if new_conv is not None:
            arrays.update(new_q=new_conv["q"], new_k=new_conv["k"], new_v=new_conv["v"])
        out = {n: _np(t) for n, t in arrays.items() if t is not None}
        meta = dict(B=B, T=T, H=H, head_dim=hd, conv_size=la["conv_size"],
                    l2norm_eps=vals["l2norm_eps"], rms_eps=vals["rms_norm_eps"],
                    dtype={torch.float32: "f32", torch.bfloat16: "bf16"}[dt], mode=mode)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=np.array(json.dumps(meta)),
                            **out)
        print(f"{name}: {sorted(out)}")


if __name__ == "__main__":
    main()
