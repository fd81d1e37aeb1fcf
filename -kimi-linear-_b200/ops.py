"""Reference-signature KDA entry points backed by the sm_100a CUDA library.

``kda_chunkwise`` and ``kda_recurrent`` take exactly the arguments of
``kimi_linear/kda.py:58-59`` and ``kimi_linear/kda.py:188`` and return the same
``(o, S)`` pair with the same shapes and dtypes:

* ``o`` is ``[B, T, H, V]`` in ``v.dtype`` (``kda.py:185,219``);
* ``S`` is ``[B, H, K, V]`` in ``state_dtype or v.dtype``;
* ``initial_state`` / ``state`` may be ``None`` (zero state) and is never
  modified (the reference clones it, ``kda.py:137,205``);
* ``q`` is scaled by ``K^-0.5`` inside the kernel (``kda.py:132,199``);
* ``g`` and ``beta`` are promoted to fp32 as the reference does
  (``kda.py:119-120,202-203``);
* ``tile_size`` only tuned the reference's CPU/GPU memory use
  (``kda.py:101-103``); it is accepted and has no effect here;
* ``T % chunk_size != 0`` raises ``RuntimeError`` like the reference's
  reshape (``kda.py:124``).

Everything runs on the current CUDA stream of the inputs' device: no host
synchronisation, no host reads of device values, outputs from PyTorch's
caching allocator -- so the calls can be captured in a CUDA graph
(``kimi_linear/graph_decode.py:269-289``).  There is no CPU path: CPU tensors
raise.

Gradients: the reference's trainers differentiate through both functions with
torch autograd.  When grad mode is on and an input requires grad, the call
runs the same forward kernel inside :class:`_KdaFunction`, whose backward is
the ``kda_backward`` kernel -- the exact reverse-mode gradient of the token
recurrence that both functions compute (``kda.py:207-216``).  It supports
K in {32, 64, 128} and V % 16 == 0 and raises otherwise.  One deliberate
difference: for fp16 outputs ``kda_recurrent`` clamps ``o`` to the fp16 range
(``kda.py:217-218``) and autograd zeroes the gradient of clamped entries; the
kernel passes every entry's gradient through (the two differ only where the
output overflowed fp16).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
       torch.bfloat16: _lib.DTYPE_BF16}


class KdaError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, code: int):
        self.code = int(code)
        super().__init__(f"{fn}: {_lib.status_string(code)} (status {code})")


def _check_tensors(fn, tensors):
    dev = None
    for name, t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{fn}: {name} must be a torch.Tensor")
        if t.device.type != "cuda":
            raise RuntimeError(
                f"{fn}: {name} is on {t.device}; the B200 KDA kernels need CUDA tensors "
                f"(there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{fn}: {name} is on {t.device}, expected {dev}")
        if t.dtype not in _DT:
            raise TypeError(f"{fn}: {name} has unsupported dtype {t.dtype}")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for _, t in tensors):
        raise RuntimeError(
            f"{fn}: the B200 KDA kernels are forward-only; call under torch.no_grad() "
            f"or detach the inputs")
    return dev


def _inner_contig(t):
    return t if t.stride(-1) == 1 or t.numel() == 0 else t.contiguous()


def _strides(t, n):
    s = list(t.stride())
    return (ctypes.c_int64 * n)(*s)


def _fill(args, q, k, v, g, beta, state_in, o, state_out, chunk_size):
    B, T, H, K = q.shape
    V = v.shape[-1]
    args.abi_version = _lib.ABI_VERSION
    args.B, args.T, args.H, args.K, args.V = B, T, H, K, V
    args.chunk_size = int(chunk_size)
    args.io_dtype = _DT[v.dtype]
    args.state_out_dtype = _DT[state_out.dtype]
    args.scale = float(K) ** -0.5
    args.flags = 0
    args.q, args.q_stride = q.data_ptr(), _strides(q, 4)
    args.k, args.k_stride = k.data_ptr(), _strides(k, 4)
    args.v, args.v_stride = v.data_ptr(), _strides(v, 4)
    args.g, args.g_stride = g.data_ptr(), _strides(g, 4)
    args.beta, args.beta_stride = beta.data_ptr(), _strides(beta, 3)
    if state_in is not None:
        args.state_in = state_in.data_ptr()
        args.state_in_stride = _strides(state_in, 4)
        args.state_in_dtype = _DT[state_in.dtype]
    else:
        args.state_in = None
        args.state_in_dtype = _lib.DTYPE_F32
    args.o, args.o_stride = o.data_ptr(), _strides(o, 4)
    args.state_out, args.state_out_stride = state_out.data_ptr(), _strides(state_out, 4)
    args.workspace = None
    args.workspace_bytes = 0


def _prepare(fn, q, k, v, g, beta, state, state_dtype, inplace=False):
    dev = _check_tensors(fn, [("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta),
                              ("state", state)])
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4 or g.dim() != 4 or beta.dim() != 3:
        raise RuntimeError(f"{fn}: expected q,k,g [B,T,H,K], v [B,T,H,V], beta [B,T,H]")
    B, T, H, K = q.shape
    V = v.shape[-1]
    if (k.shape != q.shape or g.shape != q.shape or v.shape[:3] != q.shape[:3]
            or beta.shape != q.shape[:3]):
        raise RuntimeError(
            f"{fn}: shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)} "
            f"g{tuple(g.shape)} beta{tuple(beta.shape)}")
    if state is not None and tuple(state.shape) != (B, H, K, V):
        raise RuntimeError(f"{fn}: state shape {tuple(state.shape)} != {(B, H, K, V)}")
    io = v.dtype
    # the kernels read q/k in v's dtype (the module always passes one dtype)
    q = _inner_contig(q if q.dtype == io else q.to(io))
    k = _inner_contig(k if k.dtype == io else k.to(io))
    v = _inner_contig(v)
    g = _inner_contig(g.float())              # kda.py:119,202
    beta = _inner_contig(beta.float())        # kda.py:120,203
    if beta.numel() and beta.stride(-1) != 1:
        beta = beta.contiguous()
    sdt = state_dtype or io
    if sdt not in _DT:
        raise TypeError(f"{fn}: unsupported state_dtype {sdt}")
    o = torch.empty(B, T, H, V, device=dev, dtype=io)
    if inplace and state is not None:
        # the new state overwrites `state` (every kernel reads the state tile it
        # owns before writing it, so exact aliasing is safe)
        if state.dtype != sdt:
            raise TypeError(f"{fn}: inplace needs state.dtype == state_dtype or v.dtype "
                            f"({state.dtype} vs {sdt})")
        if state.stride(-1) != 1:
            raise RuntimeError(f"{fn}: inplace needs a unit innermost state stride")
        return dev, q, k, v, g, beta, state, o, state
    if state is not None:
        state = _inner_contig(state)
    S = torch.empty(B, H, K, V, device=dev, dtype=sdt)
    return dev, q, k, v, g, beta, state, o, S


def _call(fn_name, entry, args, dev):
    stream = torch.cuda.current_stream(dev).cuda_stream
    if torch.cuda.current_device() != dev.index:
        with torch.cuda.device(dev):
            st = entry(ctypes.byref(args), ctypes.c_void_p(stream))
    else:
        st = entry(ctypes.byref(args), ctypes.c_void_p(stream))
    if st != _lib.KDA_OK:
        raise KdaError(fn_name, st)


def kda_chunkwise(q, k, v, g, beta, initial_state=None, chunk_size=64, tile_size=0,
                  state_dtype=None, *, inplace=False):
    """Chunkwise KDA forward -- drop-in for ``kimi_linear/kda.py:58``.

    ``inplace=True`` (not in the reference; off by default) writes the final
    state into ``initial_state`` and returns that tensor, instead of a new one
    (the reference clones the state, ``kda.py:137``)."""
    if _needs_grad(q, k, v, g, beta, initial_state):
        if inplace:
            raise RuntimeError("kda_chunkwise: inplace=True cannot record gradients")
        return _with_grad("kda_chunkwise", q, k, v, g, beta, initial_state,
                          lambda *t: chunkwise_impl(*t, chunk_size, state_dtype))
    return chunkwise_impl(q, k, v, g, beta, initial_state, chunk_size, state_dtype,
                          inplace=inplace)


def chunkwise_impl(q, k, v, g, beta, initial_state=None, chunk_size=64, state_dtype=None,
                   force_simt=False, inplace=False):
    """``kda_chunkwise`` with an implementation switch: ``force_simt=True``
    runs the CUDA-core kernel even where the tcgen05 kernel applies (both
    are complete implementations; the switch exists to cross-check them)."""
    C = int(chunk_size)
    if C == 0:
        raise ZeroDivisionError("integer division or modulo by zero")  # T // C, kda.py:114
    T = q.shape[1] if q.dim() == 4 else 0
    if C < 0 or T % C != 0:
        raise RuntimeError(
            f"kda_chunkwise: T={T} is not a multiple of chunk_size={C} "
            f"(the reference's reshape fails here too)")
    dev, q, k, v, g, beta, s0, o, S = _prepare("kda_chunkwise", q, k, v, g, beta,
                                               initial_state, state_dtype, inplace)
    if o.numel() == 0 and S.numel() == 0:
        return o, S
    if T == 0 and S is s0:
        return o, S                                    # nothing to do, state unchanged
    lib = _lib.load()
    args = _lib.KdaArgs()
    _fill(args, q, k, v, g, beta, s0, o, S, C)
    if force_simt:
        args.flags = _lib.FLAG_FORCE_SIMT
    need = lib.kda_chunkwise_workspace_bytes(ctypes.byref(args))
    if need:
        ws = torch.empty(int(need), dtype=torch.uint8, device=dev)
        args.workspace = ws.data_ptr()
        args.workspace_bytes = int(need)
    _call("kda_chunkwise", lib.kda_chunkwise_fwd, args, dev)
    return o, S


def kda_recurrent(q, k, v, g, beta, state=None, state_dtype=None, *, inplace=False):
    """Token-recurrent KDA forward -- drop-in for ``kimi_linear/kda.py:188``.

    ``inplace=True`` (not in the reference; off by default) writes the new
    state into ``state`` and returns that tensor: a decoder that keeps its
    state in a static buffer (``GraphedDecoder``, ``graph_decode.py:262``) then
    needs no copy-back -- its ``copy_`` becomes a copy onto itself."""
    if _needs_grad(q, k, v, g, beta, state):
        if inplace:
            raise RuntimeError("kda_recurrent: inplace=True cannot record gradients")
        return _with_grad("kda_recurrent", q, k, v, g, beta, state,
                          lambda *t: kda_recurrent(*t, state_dtype))
    dev, q, k, v, g, beta, s0, o, S = _prepare("kda_recurrent", q, k, v, g, beta,
                                               state, state_dtype, inplace)
    if o.numel() == 0 and S.numel() == 0:
        return o, S
    lib = _lib.load()
    args = _lib.KdaArgs()
    _fill(args, q, k, v, g, beta, s0, o, S, 1)
    _call("kda_recurrent", lib.kda_recurrent_fwd, args, dev)
    return o, S


def _needs_grad(*ts):
    return torch.is_grad_enabled() and any(
        isinstance(t, torch.Tensor) and t.requires_grad for t in ts)


class _KdaFunction(torch.autograd.Function):
    """Forward: one of the forward kernels (``run``); backward: ``kda_backward``.

    Inputs arrive in the dtypes the kernels read (q, k in v's dtype; g, beta
    fp32); the conversions before :meth:`apply` are ordinary differentiable
    torch ops, so autograd casts each gradient back to the caller's dtype."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, state, run):
        o, S = run(q, k, v, g, beta, state)
        ctx.save_for_backward(q, k, v, g, beta, state)
        ctx.set_materialize_grads(False)
        return o, S

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, do, dS):
        q, k, v, g, beta, state = ctx.saved_tensors
        grads = kda_backward(q, k, v, g, beta, state, do, dS)
        need = ctx.needs_input_grad
        out = [gr if need[i] else None for i, gr in enumerate(grads)]
        return (*out, None)


def kda_backward(q, k, v, g, beta, state, do, dS):
    """Gradients ``(dq, dk, dv, dg, dbeta, dstate)`` of the KDA forward
    ``(o, S) = f(q, k, v, g, beta, state)`` for output gradients ``do``
    (of ``o``, or None) and ``dS`` (of the returned state, or None).

    ``q``, ``k``, ``v`` share one dtype; ``g``, ``beta`` fp32; ``state`` is
    None (zero initial state, ``dstate`` None) or [B, H, K, V] in any
    supported dtype.  dq, dk, dv come back in v's dtype, dg and dbeta fp32,
    dstate in ``state``'s dtype.  For V <= 128 the library runs the chunkwise
    backward (64-token chunks in parallel, two short state chains); wider V
    runs the token-serial kernels, whose per-16-column partial sums the library
    adds up in the same call."""
    fn = "kda_backward"
    dev = _check_tensors(fn, [("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta),
                              ("state", state), ("do", do), ("dS", dS)])
    B, T, H, K = q.shape
    V = v.shape[-1]
    io = v.dtype
    if q.dtype != io or k.dtype != io or g.dtype != torch.float32 or \
            beta.dtype != torch.float32:
        raise TypeError(f"{fn}: q, k, v must share one dtype and g, beta be fp32")
    q, k, v, g = (_inner_contig(t) for t in (q, k, v, g))
    beta = beta if beta.numel() == 0 or beta.stride(-1) == 1 else beta.contiguous()
    if state is not None:
        state = _inner_contig(state)
    if do is None:
        do = torch.zeros(B, T, H, V, device=dev, dtype=io)
    else:
        do = _inner_contig(do.to(io))
    if dS is not None:
        dS = _inner_contig(dS.float())
    dv = torch.empty(B, T, H, V, device=dev, dtype=torch.float32)
    dstate = (torch.empty(B, H, K, V, device=dev, dtype=torch.float32)
              if state is not None else None)
    if B * T * H == 0:
        if dstate is not None:
            dstate.copy_(dS if dS is not None else torch.zeros_like(dstate))
        z = torch.zeros(B, T, H, K, device=dev, dtype=torch.float32)
        return (z.to(io), z.to(io), dv.zero_().to(io), z,
                torch.zeros(B, T, H, device=dev, dtype=torch.float32),
                None if state is None else dstate.to(state.dtype))
    # V <= 128: the chunkwise kernels write the final gradients; wider V runs
    # the token-serial kernels, which write per-16-column partial sums that the
    # library then adds up (both in the same call)
    if V > 128:
        nvt = V // 16
        dq_p = torch.empty(nvt, B, T, H, K, device=dev, dtype=torch.float32)
        dk_p = torch.empty_like(dq_p)
        dg_p = torch.empty_like(dq_p)
        db_p = torch.empty(nvt, B, T, H, device=dev, dtype=torch.float32)
    lib = _lib.load()
    ck_n = int(lib.kda_backward_ckpt_floats(B, H, T, K, V))
    ckpt = torch.empty(max(ck_n, 4), device=dev, dtype=torch.float32)
    a = _lib.KdaBackwardArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V = B, T, H, K, V
    a.io_dtype = _DT[io]
    a.scale = float(K) ** -0.5
    a.q, a.q_stride = q.data_ptr(), _strides(q, 4)
    a.k, a.k_stride = k.data_ptr(), _strides(k, 4)
    a.v, a.v_stride = v.data_ptr(), _strides(v, 4)
    a.g, a.g_stride = g.data_ptr(), _strides(g, 4)
    a.beta, a.beta_stride = beta.data_ptr(), _strides(beta, 3)
    if state is not None:
        a.state_in, a.state_in_stride = state.data_ptr(), _strides(state, 4)
        a.state_in_dtype = _DT[state.dtype]
        a.dstate_in, a.dstate_in_stride = dstate.data_ptr(), _strides(dstate, 4)
    else:
        a.state_in_dtype = _lib.DTYPE_F32
    a.dout, a.dout_stride = do.data_ptr(), _strides(do, 4)
    if dS is not None:
        a.dstate_out, a.dstate_out_stride = dS.data_ptr(), _strides(dS, 4)
    if V > 128:
        a.dq_part, a.dk_part = dq_p.data_ptr(), dk_p.data_ptr()
        a.dg_part, a.dbeta_part = dg_p.data_ptr(), db_p.data_ptr()
    a.dv, a.dv_stride = dv.data_ptr(), _strides(dv, 4)
    a.ckpt, a.ckpt_floats = ckpt.data_ptr(), ck_n
    dq = torch.empty(B, T, H, K, device=dev, dtype=io)
    dk = torch.empty_like(dq)
    dg = torch.empty(B, T, H, K, device=dev, dtype=torch.float32)
    db = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    a.dq, a.dq_stride = dq.data_ptr(), _strides(dq, 4)
    a.dk, a.dk_stride = dk.data_ptr(), _strides(dk, 4)
    a.dg, a.dg_stride = dg.data_ptr(), _strides(dg, 4)
    a.dbeta, a.dbeta_stride = db.data_ptr(), _strides(db, 3)
    _call(fn, lib.kda_backward, a, dev)
    return (dq, dk, dv.to(io), dg, db,
            None if state is None else dstate.to(state.dtype))


def _with_grad(fn, q, k, v, g, beta, state, run):
    """Route a call that needs gradients through :class:`_KdaFunction`."""
    _check_grad_inputs(fn, q, k, v, g, beta, state)
    io = v.dtype
    q = q if q.dtype == io else q.to(io)
    k = k if k.dtype == io else k.to(io)
    return _KdaFunction.apply(q, k, v, g.float(), beta.float(), state, run)


def _check_grad_inputs(fn, q, k, v, g, beta, state):
    with torch.no_grad():
        _check_tensors(fn, [("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta),
                            ("state", state)])


def device_error(clear=True):
    """The kernels' device error word (0 = no bounded wait ever gave up)."""
    return int(_lib.load().kda_device_error(1 if clear else 0))


def chunkwise_path(q, k, v, g, beta, initial_state=None, chunk_size=64, state_dtype=None):
    """Which kernel ``kda_chunkwise`` runs for these inputs: "tcgen05" or "simt"."""
    dev, q, k, v, g, beta, s0, o, S = _prepare("chunkwise_path", q, k, v, g, beta,
                                               initial_state, state_dtype)
    lib = _lib.load()
    args = _lib.KdaArgs()
    _fill(args, q, k, v, g, beta, s0, o, S, int(chunk_size))
    r = lib.kda_chunkwise_path(ctypes.byref(args))
    if r < 0:
        raise KdaError("chunkwise_path", -r)
    return "tcgen05" if r == 1 else "simt"
