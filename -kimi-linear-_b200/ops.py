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
(``kimi_linear/graph_decode.py:269-289``).  The kernels are forward-only: a
call that would need gradients raises instead of returning values autograd
cannot differentiate.  There is no CPU path: CPU tensors raise.
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
    dev, q, k, v, g, beta, s0, o, S = _prepare("kda_recurrent", q, k, v, g, beta,
                                               state, state_dtype, inplace)
    if o.numel() == 0 and S.numel() == 0:
        return o, S
    lib = _lib.load()
    args = _lib.KdaArgs()
    _fill(args, q, k, v, g, beta, s0, o, S, 1)
    _call("kda_recurrent", lib.kda_recurrent_fwd, args, dev)
    return o, S


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
