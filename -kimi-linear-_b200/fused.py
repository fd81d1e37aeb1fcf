"""Fused prologue / epilogue of the KDA block (``csrc/kda_io.cu``).

Around the KDA core, ``KimiDeltaAttention`` (``kimi_linear/kda.py:331``) runs
a chain of elementwise passes over HBM:

* ``_projections`` (``kda.py:399-461``): after the q/k/v, gate and beta
  projection GEMMs -- causal ShortConv (``kda.py:282-310``), SiLU, per-head
  ``l2norm`` (``kda.py:313-325``), ``g = -exp(A_log) * softplus(gk + dt_bias)``,
  ``beta = sigmoid(beta_logit)`` and the conv cache;
* ``_output`` (``kda.py:464-470``): head-wise RMSNorm (``kda.py:258-279``)
  and the sigmoid output gate before ``o_proj``.

:func:`kda_prologue` and :func:`kda_epilogue` do each in one kernel.
:func:`projections` / :func:`output` are drop-ins for the two module methods
(same arguments and returns; the module's own ``nn.Linear`` GEMMs still run),
and :func:`install_module` patches them onto the class.  Forward only, CUDA
tensors only, K == V in {32, 64, 128}; anything else raises (no fallback).

Deliberate difference: with ``use_cache`` and a prefill shorter than
``conv_size - 1`` tokens and no history, the reference returns a conv cache
with fewer than ``conv_size - 1`` rows (``kda.py:437``), which its own decode
step cannot consume; here the cache always has ``conv_size - 1`` rows, the
missing ones zero (the conv's zero left padding).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _DT, _call, _check_tensors


def _rows(t):
    """(batch, time) strides of a [B, T, D] tensor with a unit last stride."""
    return (ctypes.c_int64 * 2)(t.stride(0), t.stride(1))


def _last_contig(t):
    return t if t.stride(-1) == 1 else t.contiguous()


def _f32(t, cache=None):
    """``t`` as a contiguous fp32 tensor, memoised per parameter version."""
    if t is None:
        return None
    if cache is None or torch.is_grad_enabled():
        return t.detach().float().contiguous()
    key = (id(t), t._version, t.data_ptr(), t.device)
    hit = cache.get(id(t))
    if hit is not None and hit[0] == key:
        return hit[1]
    val = t.detach().float().contiguous()
    cache[id(t)] = (key, val)
    return val


def kda_prologue(q_in, k_in, v_in, gk, beta_logit, conv_w, conv_b, A_log, dt_bias,
                 num_heads, head_dim, value_head_dim, l2norm_eps, conv_cache=None,
                 want_cache=False):
    """q, k, v, g, beta (and the new conv cache) from the projection outputs.

    ``q_in``/``k_in`` [B, T, H*K], ``v_in`` [B, T, H*V], ``gk`` [B, T, H*K],
    ``beta_logit`` [B, T, H]; ``conv_w`` / ``conv_b``: (q, k, v) triples of the
    ``nn.Conv1d`` weights [D, 1, cs] and biases [D] (or None); ``conv_cache``:
    dict of histories [B, cs-1, D] or None.  Returns ``(q, k, v, g, beta,
    new_cache)``: q, k [B, T, H, K] and v [B, T, H, V] in q_in's dtype, g
    [B, T, H, K] and beta [B, T, H] fp32, new_cache a dict (``want_cache``) or
    None.
    """
    fn = "kda_prologue"
    hist = None if conv_cache is None else [conv_cache[n] for n in "qkv"]
    dev = _check_tensors(fn, [("q_in", q_in), ("k_in", k_in), ("v_in", v_in), ("gk", gk),
                              ("beta_logit", beta_logit)] +
                         ([] if hist is None else [(f"conv_cache[{n}]", h)
                                                   for n, h in zip("qkv", hist)]))
    B, T, _ = q_in.shape
    H, K, V = int(num_heads), int(head_dim), int(value_head_dim)
    io = q_in.dtype
    if k_in.dtype != io or v_in.dtype != io or (hist and any(h.dtype != io for h in hist)):
        raise TypeError(f"{fn}: q_in, k_in, v_in and the conv cache must share one dtype")
    if gk.dtype != beta_logit.dtype:
        beta_logit = beta_logit.to(gk.dtype)
    q_in, k_in, v_in, gk, beta_logit = (_last_contig(t) for t in (q_in, k_in, v_in, gk,
                                                                   beta_logit))
    ws = [w.reshape(w.shape[0], -1) for w in conv_w]
    cs = ws[0].shape[1]
    keep = cs - 1
    if hist is not None:
        hist = [_last_contig(h) for h in hist]
        for h in hist:
            if h.shape[1] != keep or h.stride(1) != h.shape[2]:
                raise RuntimeError(f"{fn}: conv cache must be [B, {keep}, D] with row stride D")
    q = torch.empty(B, T, H, K, device=dev, dtype=io)
    k = torch.empty(B, T, H, K, device=dev, dtype=io)
    v = torch.empty(B, T, H, V, device=dev, dtype=io)
    g = torch.empty(B, T, H, K, device=dev, dtype=torch.float32)
    beta = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    new = None
    if want_cache:
        new = {n: torch.empty(B, keep, D, device=dev, dtype=io)
               for n, D in (("q", H * K), ("k", H * K), ("v", H * V))}
    if B * T == 0:
        if new is not None and hist is not None:
            for n, h in zip("qkv", hist):
                new[n].copy_(h)
        elif new is not None:
            for t in new.values():
                t.zero_()
        return q, k, v, g, beta, new
    a = _lib.KdaPrologueArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V = B, T, H, K, V
    a.conv_size = cs
    a.io_dtype = _DT[io]
    a.gate_dtype = _DT[gk.dtype]
    a.l2norm_eps = float(l2norm_eps)
    a.q_in, a.q_in_stride = q_in.data_ptr(), _rows(q_in)
    a.k_in, a.k_in_stride = k_in.data_ptr(), _rows(k_in)
    a.v_in, a.v_in_stride = v_in.data_ptr(), _rows(v_in)
    keepalive = [_f32(w) for w in ws] + [_f32(b) if b is not None else None
                                         for b in (conv_b or (None, None, None))]
    for i in range(3):
        a.conv_w[i] = keepalive[i].data_ptr()
        a.conv_b[i] = keepalive[3 + i].data_ptr() if keepalive[3 + i] is not None else None
        a.hist[i] = hist[i].data_ptr() if hist is not None else None
        a.hist_batch_stride[i] = hist[i].stride(0) if hist is not None else 0
        a.new_hist[i] = new["qkv"[i]].data_ptr() if new is not None else None
    a.gk, a.gk_stride = gk.data_ptr(), _rows(gk)
    a.beta_logit, a.beta_logit_stride = beta_logit.data_ptr(), _rows(beta_logit)
    A32, d32 = _f32(A_log), _f32(dt_bias)
    a.A_log, a.dt_bias = A32.data_ptr(), d32.data_ptr()
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g)):
        setattr(a, name, t.data_ptr())
        setattr(a, f"{name}_stride", (ctypes.c_int64 * 4)(*t.stride()))
    a.beta, a.beta_stride = beta.data_ptr(), (ctypes.c_int64 * 3)(*beta.stride())
    _call(fn, _lib.load().kda_prologue_fwd, a, dev)
    return q, k, v, g, beta, new


def kda_epilogue(o_core, og, weight, eps):
    """``(rmsnorm_head(o_core) * weight).to(dtype) * sigmoid(og)``, in o_core's
    dtype, as [B, T, H*V] (the input of ``o_proj``).  ``og`` [B, T, H*V],
    ``weight`` [H, V]."""
    fn = "kda_epilogue"
    dev = _check_tensors(fn, [("o_core", o_core), ("og", og), ("weight", weight)])
    B, T, H, V = o_core.shape
    io = o_core.dtype
    if og.dtype != io:
        og = og.to(io)
    o_core, og = _last_contig(o_core), _last_contig(og)
    y = torch.empty(B, T, H * V, device=dev, dtype=io)
    if B * T * H == 0:
        return y
    w32 = _f32(weight)
    a = _lib.KdaEpilogueArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.V = B, T, H, V
    a.io_dtype = _DT[io]
    a.eps = float(eps)
    a.o, a.o_stride = o_core.data_ptr(), (ctypes.c_int64 * 4)(*o_core.stride())
    a.og, a.og_stride = og.data_ptr(), _rows(og)
    a.weight = w32.data_ptr()
    a.y, a.y_stride = y.data_ptr(), _rows(y)
    _call(fn, _lib.load().kda_epilogue_fwd, a, dev)
    return y


def _module_cache(m):
    c = getattr(m, "_b200_cast_cache", None)
    if c is None:
        c = {}
        m._b200_cast_cache = c
    return c


def projections(module, x, conv_cache=None, use_cache=False):
    """Drop-in for ``KimiDeltaAttention._projections`` (``kda.py:399-461``)."""
    m = module
    cache = _module_cache(m)
    keep = max(m.conv_size - 1, 0)
    q_in, k_in, v_in = m.in_proj_q(x), m.in_proj_k(x), m.in_proj_v(x)
    gk = m.gk_proj(x)
    beta_logit = m.beta_proj(x)
    hist = conv_cache if (use_cache and conv_cache is not None and keep > 0) else None
    ws = [_f32(c.conv.weight, cache) for c in (m.conv_q, m.conv_k, m.conv_v)]
    bs = [_f32(c.conv.bias, cache) if c.conv.bias is not None else None
          for c in (m.conv_q, m.conv_k, m.conv_v)]
    q, k, v, g, beta, new = kda_prologue(
        q_in, k_in, v_in, gk, beta_logit, ws, bs, _f32(m.A_log, cache), _f32(m.dt_bias, cache),
        m.num_heads, m.head_dim, m.value_head_dim, m.l2norm_eps, conv_cache=hist,
        want_cache=use_cache)
    return q, k, v, g, beta, new


def output(module, o_core, x):
    """Drop-in for ``KimiDeltaAttention._output`` (``kda.py:464-470``)."""
    m = module
    og = m.og_proj(x)
    y = kda_epilogue(o_core, og, _f32(m.g_norm.weight, _module_cache(m)), m.g_norm.eps)
    return m.o_proj(y)


_saved = []


def install_module(cls=None):
    """Route ``cls._projections`` / ``cls._output`` (default: the reference's
    ``kimi_linear.kda.KimiDeltaAttention``) through :func:`projections` and
    :func:`output`.  Returns the patched class; :func:`uninstall_module`
    restores the originals."""
    if cls is None:
        import importlib
        cls = importlib.import_module("kimi_linear.kda").KimiDeltaAttention
    _lib.load()
    for name, fn in (("_projections", projections), ("_output", output)):
        _saved.append((cls, name, cls.__dict__.get(name)))
        setattr(cls, name, fn)
    return cls


def uninstall_module():
    while _saved:
        cls, name, fn = _saved.pop()
        if fn is None:
            delattr(cls, name)
        else:
            setattr(cls, name, fn)
