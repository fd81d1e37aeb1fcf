"""Single-token MLA decode over a static latent buffer (``csrc/mla_decode.cu``).

Drop-in for ``MLA._decode_step_static`` (``kimi_linear/mla.py:117-181``), the
graph-capturable decode step ``GraphedDecoder`` runs for every MLA layer
(``kimi_linear/graph_decode.py``): the module's own projections and ``o_proj``
still run; everything between them -- writing the new latent at ``pos``, the
absorbed-form attention over the whole buffer with the ``pos`` mask, the
``W_v`` projection and ``pos += 1`` -- is one C-ABI call (three kernels) that
reads ``pos`` from device memory, so a replayed graph picks up its current
value exactly as the reference's ``index_copy_`` / mask do.

Numerics follow the reference: ``q_lat = q_nope W_nope`` and the scores in
fp32, softmax in fp32, ``p`` and ``mixed = p kv_buf`` in the buffer's dtype,
``mixed W_v^T`` in fp32, the result in the activation dtype.

Supported: NoPE layers (``qk_rope_head_dim == 0``, the configuration of the
paper and of ``configs/kimi_linear_1p5b_dense.json``), fp16/bf16 activations,
``num_heads <= 16``, ``kv_lora_rank`` in {64, 128, 256, 512}.  Anything else
raises (no fallback); CUDA tensors only.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _DT, _call, _check_tensors

_SUPPORTED_KVL = (64, 128, 256, 512)


def _s(t, n):
    return (ctypes.c_int64 * n)(*t.stride())


def mla_decode_core(q_nope, c_kv, kv_buf, pos, w, num_heads, nope_dim, v_dim, scale):
    """The attention core of one static-buffer decode step.

    ``q_nope`` [B, 1, H, DN] (or [B, H, DN]), ``c_kv`` [B, 1, KVL] (or
    [B, KVL]), ``kv_buf`` [B, L, KVL] (updated in place at ``pos``), ``pos``
    int64 [1] on the device (advanced by one), ``w`` = ``kv_b_proj.weight``
    [H*(DN+DV), KVL].  Returns ``attn_out`` [B, 1, H*DV] in ``q_nope``'s dtype
    (the input of ``o_proj``)."""
    fn = "mla_decode_core"
    dev = _check_tensors(fn, [("q_nope", q_nope), ("c_kv", c_kv), ("kv_buf", kv_buf),
                              ("w", w)])
    if not isinstance(pos, torch.Tensor) or pos.device != dev or pos.dtype != torch.int64 \
            or pos.numel() != 1:
        raise RuntimeError(f"{fn}: pos must be an int64 tensor of one element on {dev}")
    io = kv_buf.dtype
    if io not in (torch.float16, torch.bfloat16):
        raise TypeError(f"{fn}: the B200 MLA decode kernel needs fp16 or bf16 (got {io})")
    B, L, KVL = kv_buf.shape
    H, DN, DV = int(num_heads), int(nope_dim), int(v_dim)
    if KVL not in _SUPPORTED_KVL or H > 16:
        raise RuntimeError(f"{fn}: kv_lora_rank {KVL} / num_heads {H} not supported "
                           f"(kv_lora_rank in {_SUPPORTED_KVL}, num_heads <= 16)")
    qn = q_nope.reshape(B, H, DN) if q_nope.dim() == 4 else q_nope
    ck = c_kv.reshape(B, KVL) if c_kv.dim() == 3 else c_kv
    if qn.dtype != io:
        qn = qn.to(io)
    if ck.dtype != io:
        ck = ck.to(io)
    if w.dtype != io:
        w = w.to(io)
    if tuple(w.shape) != (H * (DN + DV), KVL):
        raise RuntimeError(f"{fn}: kv_b_proj.weight shape {tuple(w.shape)} != "
                           f"{(H * (DN + DV), KVL)}")
    out = torch.empty(B, H, DV, device=dev, dtype=io)
    a = _lib.MlaDecodeArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.L, a.H, a.KVL, a.DN, a.DV = B, L, H, KVL, DN, DV
    a.io_dtype = _DT[io]
    a.scale = float(scale)
    a.q_nope, a.q_nope_stride = qn.data_ptr(), _s(qn, 3)
    a.c_kv, a.c_kv_stride = ck.data_ptr(), _s(ck, 2)
    a.kv_buf, a.kv_buf_stride = kv_buf.data_ptr(), _s(kv_buf, 3)
    a.pos = pos.data_ptr()
    a.w, a.w_stride = w.data_ptr(), _s(w, 2)
    a.out, a.out_stride = out.data_ptr(), _s(out, 3)
    lib = _lib.load()
    need = int(lib.mla_decode_workspace_bytes(ctypes.byref(a)))
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), need
    _call(fn, lib.mla_decode_fwd, a, dev)
    return out.reshape(B, 1, H * DV)


def _weight(module, dtype):
    """``kv_b_proj.weight`` in ``dtype``, cast once per parameter version."""
    w = module.kv_b_proj.weight
    if w.dtype == dtype:
        return w.detach()
    cache = module.__dict__.setdefault("_b200_w_cache", {})
    key = (w._version, w.data_ptr(), dtype)
    hit = cache.get("kv_b")
    if hit is None or hit[0] != key:
        hit = (key, w.detach().to(dtype))
        cache["kv_b"] = hit
    return hit[1]


def decode_step_static(module, x, q_nope, q_rope, c_kv, k_rope, state, use_cache):
    """Drop-in for ``MLA._decode_step_static`` (``kimi_linear/mla.py:117``):
    same arguments, same returns, same in-place updates of ``state``."""
    if x.shape[1] != 1:
        raise RuntimeError("the static-buffer path is single-token decode only")
    if module.qk_rope_head_dim != 0:
        raise NotImplementedError(
            "decode_step_static: the B200 MLA decode kernel covers NoPE layers "
            "(qk_rope_head_dim == 0) only")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, q_nope, c_kv)):
        raise RuntimeError("decode_step_static is forward-only (decode); call under no_grad")
    attn_out = mla_decode_core(q_nope, c_kv, state["c_kv_buf"], state["pos"],
                               _weight(module, x.dtype), module.num_heads,
                               module.qk_nope_head_dim, module.v_head_dim, module.scale)
    out = module.o_proj(attn_out.to(x.dtype))
    if use_cache:
        return out, state
    return out


_saved = []


def install_mla(cls=None):
    """Route ``cls._decode_step_static`` (default: the reference's
    ``kimi_linear.mla.MLA``) through :func:`decode_step_static`.  Returns the
    patched class; :func:`uninstall_mla` restores the original."""
    if cls is None:
        import importlib
        cls = importlib.import_module("kimi_linear.mla").MLA
    _lib.load()
    _saved.append((cls, cls.__dict__.get("_decode_step_static")))
    cls._decode_step_static = decode_step_static
    return cls


def uninstall_mla():
    while _saved:
        cls, fn = _saved.pop()
        if fn is None:
            delattr(cls, "_decode_step_static")
        else:
            cls._decode_step_static = fn
