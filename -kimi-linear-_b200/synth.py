"""Seeded synthetic KDA inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved anywhere in this path).

Draw order from one generator (fixed, so every consumer sees identical
tensors for a seed): q, k, v, A_log, x, dt, beta, then S0 when requested.

* ``q, k ~ N(0, 1)``, L2-normalised over the head dimension (the module applies
  ``l2norm`` before the core, ``kimi_linear/kda.py:449-450``);
* ``v ~ N(0, 1)``;
* ``A_log = log U(1, 16)`` per ``[H, K]`` channel;
* ``x ~ N(0, 1)`` of shape ``[B, T, H, K]``;
* ``dt_bias = log(expm1(U(1e-3, 0.1)))`` per ``[H, K]`` channel;
* ``g = -exp(A_log) * softplus(x + dt_bias)`` in fp32 (``kda.py:460``);
* ``beta = sigmoid(N(0, 1))`` of shape ``[B, T, H]`` in fp32 (``kda.py:452``);
* ``S0 ~ N(0, std)`` of shape ``[B, H, K, V]`` in fp32 when ``s0_std`` is set.

q is NOT pre-scaled: both reference kernels apply ``K^-0.5`` internally
(``kda.py:132,199``) and so do the CUDA kernels.

Generation runs in fp32 on ``device`` (CPU by default, so that the oracle and
the kernel see the same tensors); q/k/v are then cast to ``dtype``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

# BASELINE configurations (shape dictionaries); C is the reference chunk_size.
CONFIGS = {
    0: dict(B=2, T=256, H=2, K=32, V=32, C=64, dtype=torch.float32, s0_std=None),
    1: dict(B=1, T=4096, H=16, K=128, V=128, C=64, dtype=torch.float16, s0_std=None),
    2: dict(B=64, T=1, H=16, K=128, V=128, C=64, dtype=torch.float16, s0_std=0.02,
            steps=1024),
    3: dict(B=8, T=32768, H=16, K=128, V=128, C=64, dtype=torch.bfloat16, s0_std=0.02),
}


def make_inputs(B, T, H, K, V, dtype=torch.float32, seed=0, s0_std=None,
                device="cpu", generator=None):
    """Return ``dict(q, k, v, g, beta, S0)`` on ``device``.

    ``generator`` may be passed to continue an existing random stream (used by
    the decode benchmark to draw one token after another).
    """
    gen = generator
    if gen is None:
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed))
    f32 = dict(dtype=torch.float32, device=device, generator=gen)
    q = torch.randn(B, T, H, K, **f32)
    k = torch.randn(B, T, H, K, **f32)
    v = torch.randn(B, T, H, V, **f32)
    a_log = torch.log(torch.empty(H, K, dtype=torch.float32, device=device).uniform_(
        1.0, 16.0, generator=gen))
    x = torch.randn(B, T, H, K, **f32)
    dt = torch.empty(H, K, dtype=torch.float32, device=device).uniform_(
        1e-3, 0.1, generator=gen)
    dt_bias = torch.log(torch.expm1(dt))
    braw = torch.randn(B, T, H, **f32)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True))
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True))
    g = -torch.exp(a_log) * F.softplus(x + dt_bias)
    beta = torch.sigmoid(braw)
    S0 = None
    if s0_std is not None:
        S0 = torch.randn(B, H, K, V, **f32) * float(s0_std)
    return dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), g=g.float(),
                beta=beta.float(), S0=S0)


def make_config(cfg_id, seed=0, device="cpu", **override):
    """Inputs of BASELINE config ``cfg_id`` (fields may be overridden)."""
    c = dict(CONFIGS[cfg_id])
    c.update(override)
    return make_inputs(c["B"], c["T"], c["H"], c["K"], c["V"], dtype=c["dtype"],
                       seed=seed, s0_std=c["s0_std"], device=device)
