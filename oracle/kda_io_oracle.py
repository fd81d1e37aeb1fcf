"""CPU oracle for the fused KDA prologue / epilogue -- TEST INFRASTRUCTURE ONLY.

numpy restatement of the elementwise part of the reference's KDA block around
the core (Lazy-Hakimi/-kimi-linear-):

* ``prologue`` -- ``KimiDeltaAttention._projections`` after its projection
  GEMMs (``kimi_linear/kda.py:399-461``): causal depthwise ``ShortConv``
  (``kda.py:282-310``), SiLU, per-head ``l2norm`` (``kda.py:313-325``), the
  log decay ``g = -exp(A_log) * softplus(gk + dt_bias)`` and
  ``beta = sigmoid(beta_logit)``, plus the new conv cache;
* ``epilogue`` -- ``KimiDeltaAttention._output`` before ``o_proj``
  (``kda.py:464-470``) with ``HeadwiseRMSNorm`` (``kda.py:258-279``).

Only ``tests/`` may import it; it checks the CUDA kernels of
``-kimi-linear-_b200/csrc/kda_io.cu`` and is pinned against vectors made by the
reference module itself (``tests/golden/make_golden_fused.py``).

Dtype handling follows the reference: values are carried as float32 arrays;
``dtype`` ("f32" / "f16" / "bf16") names the tensor dtype of the module, and
every intermediate the reference materialises in that dtype (conv output,
SiLU output, normalised q/k, RMSNorm output, gated output) is rounded to it.
"""

from __future__ import annotations

import numpy as np

from .kda_oracle import round_bf16

_F32 = np.float32


def rnd(x, dtype):
    """Round float32 values to ``dtype`` and return float32."""
    x = np.asarray(x, dtype=_F32)
    if dtype == "f16":
        return x.astype(np.float16).astype(_F32)
    if dtype == "bf16":
        return round_bf16(x)
    return x


def short_conv(x, w, b, hist, dtype):
    """Causal depthwise conv (``kda.py:282-310``) of ``x`` [B, T, D].

    ``w`` [D, cs] (the ``nn.Conv1d`` weight without its middle axis), ``b``
    [D] or None, ``hist`` [B, cs-1, D] (the conv cache) or None for zero
    left padding.  Returns (out [B, T, D] rounded to ``dtype``, full input
    [B, cs-1+T, D] with the history prepended)."""
    B, T, D = x.shape
    cs = w.shape[1]
    keep = cs - 1
    pad = np.zeros((B, keep, D), _F32) if hist is None else np.asarray(hist, _F32)
    full = np.concatenate([pad, np.asarray(x, _F32)], axis=1)
    out = np.zeros((B, T, D), _F32)
    for j in range(cs):
        out += full[:, j:j + T, :] * w[:, j].astype(_F32)
    if b is not None:
        out += b.astype(_F32)
    return rnd(out, dtype), full


def silu(x):
    x = np.asarray(x, _F32)
    return x / (_F32(1) + np.exp(-x))


def l2norm(x, eps, dtype):
    """``kda.py:313-325``: fp32 reduction over the last axis, rsqrt clamped
    at 1 / eps, result in the input dtype."""
    x = np.asarray(x, _F32)
    ss = (x * x).sum(-1, keepdims=True, dtype=_F32)
    with np.errstate(divide="ignore"):
        rstd = np.minimum(_F32(1) / np.sqrt(ss), _F32(1.0 / eps))
    return rnd(x * rstd, dtype)


def softplus(x):
    """torch.nn.functional.softplus with beta 1, threshold 20."""
    x = np.asarray(x, _F32)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(_F32)


def sigmoid(x):
    x = np.asarray(x, _F32)
    return (_F32(1) / (_F32(1) + np.exp(-x))).astype(_F32)


def prologue(q_in, k_in, v_in, gk, beta_logit, w, b, A_log, dt_bias, H, K, V, eps, dtype,
             hist=None, want_cache=False):
    """Outputs of ``_projections`` from its GEMM outputs (``kda.py:443-461``).

    ``w`` / ``b`` / ``hist``: dicts keyed "q", "k", "v".  Returns
    (q, k, v, g, beta, new_cache or None)."""
    B, T, _ = q_in.shape
    outs, fulls = {}, {}
    for n, x in (("q", q_in), ("k", k_in), ("v", v_in)):
        c, full = short_conv(x, w[n], b.get(n) if b else None,
                             None if hist is None else hist[n], dtype)
        outs[n] = rnd(silu(c), dtype)
        fulls[n] = full
    q = l2norm(outs["q"].reshape(B, T, H, K), eps, dtype)
    k = l2norm(outs["k"].reshape(B, T, H, K), eps, dtype)
    v = outs["v"].reshape(B, T, H, V)
    g = (-np.exp(np.asarray(A_log, _F32)) *
         softplus(np.asarray(gk, _F32).reshape(B, T, H, K) + np.asarray(dt_bias, _F32)))
    beta = sigmoid(beta_logit)
    cache = None
    if want_cache:
        keep = w["q"].shape[1] - 1
        cache = {n: fulls[n][:, fulls[n].shape[1] - keep:] for n in "qkv"}
    return q, k, v, g.astype(_F32), beta, cache


def epilogue(o_core, og, weight, eps, dtype):
    """The tensor ``_output`` hands to ``o_proj`` (``kda.py:464-469``):
    head-wise RMSNorm (fp32, weight [H, V]) in ``dtype``, times
    sigmoid(og) in fp32, in ``dtype``; returned as [B, T, H*V]."""
    B, T, H, V = o_core.shape
    x = np.asarray(o_core, _F32)
    r = _F32(1) / np.sqrt((x * x).mean(-1, keepdims=True, dtype=_F32) + _F32(eps))
    n = rnd(x * r * np.asarray(weight, _F32), dtype)
    gate = sigmoid(np.asarray(og, _F32).reshape(B, T, H, V))
    return rnd(n * gate, dtype).reshape(B, T, H * V)
