"""Generate golden static-buffer MLA decode steps from the reference module.

Run in a checkout that has the reference source (Lazy-Hakimi/-kimi-linear-)::

    python tests/golden/make_golden_mla.py --reference <path-to-reference-checkout>

For every case it builds the reference's ``kimi_linear.mla.MLA`` (NoPE, seeded
random init) in the case's dtype on CPU, draws ``q_nope``, ``c_kv`` and a
partly filled latent buffer, and calls ``MLA._decode_step_static``
(``kimi_linear/mla.py:117``) with ``use_cache=True``.  It stores the inputs,
``kv_b_proj.weight``, ``o_proj.weight``, the input of ``o_proj`` (captured with
a forward pre-hook: the attention core's output), the module's output and
the advanced position in ``tests/golden/mla_<case>.npz`` (bf16 values as
float32 arrays).  Consumed by ``tests/test_oracle_mla_golden.py`` and
``tests/test_gpu_mla.py``.
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (dtype, B, L, H, KVL, DN, DV, hidden, pos)
CASES = {
    "mla_f16_h16": (torch.float16, 2, 200, 16, 128, 32, 32, 64, 150),
    "mla_bf16_last": (torch.bfloat16, 1, 70, 16, 256, 32, 16, 64, 69),
    "mla_f16_first": (torch.float16, 3, 64, 4, 64, 16, 16, 32, 0),
}


def _np(t):
    return t.detach().float().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the reference checkout (contains kimi_linear/)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    MLA = importlib.import_module("kimi_linear.mla").MLA
    dname = {torch.float16: "f16", torch.bfloat16: "bf16"}
    for name, (dt, B, L, H, KVL, DN, DV, hidden, pos) in CASES.items():
        torch.manual_seed(0)
        cfg = types.SimpleNamespace(
            full_attn_config=dict(num_heads=H, q_lora_rank=32, kv_lora_rank=KVL,
                                  qk_nope_head_dim=DN, qk_rope_head_dim=0, v_head_dim=DV,
                                  rope_theta=10000.0, qkv_bias=False, o_bias=False),
            hidden_size=hidden, rms_norm_eps=1e-6, max_position_embeddings=4096)
        m = MLA(cfg).to(dt).eval()
        gen = torch.Generator().manual_seed(1)
        q_nope = (torch.randn(B, 1, H, DN, generator=gen) * 0.5).to(dt)
        c_kv = torch.randn(B, 1, KVL, generator=gen).to(dt)
        buf = torch.zeros(B, L, KVL, dtype=dt)
        buf[:, :pos] = torch.randn(B, pos, KVL, generator=gen).to(dt)
        state = {"c_kv_buf": buf.clone(), "pos": torch.tensor([pos], dtype=torch.int64)}
        x = torch.zeros(B, 1, hidden, dtype=dt)
        seen = []
        hook = m.o_proj.register_forward_pre_hook(lambda mod, inp: seen.append(inp[0].clone()))
        with torch.no_grad():
            out, st = m._decode_step_static(x, q_nope, None, c_kv, None, state, True)
        hook.remove()
        arrays = dict(q_nope=_np(q_nope), c_kv=_np(c_kv), kv_buf=_np(buf),
                      w=_np(m.kv_b_proj.weight), o_w=_np(m.o_proj.weight),
                      attn_out=_np(seen[0]), out=_np(out),
                      kv_buf_after_row=_np(st["c_kv_buf"][:, pos]))
        meta = np.array([B, L, H, KVL, DN, DV, hidden, pos, int(st["pos"].item())],
                        dtype=np.int64)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=meta,
                            dtype=np.array(dname[dt]), scale=np.array(m.scale), **arrays)
        print(f"{name}: wrote {sorted(arrays)}")


if __name__ == "__main__":
    main()
