"""CPU oracle for the Kimi Delta Attention (KDA) core -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the two reference kernels of Lazy-Hakimi/-kimi-linear-:

* ``kda_chunkwise``  -- ``kimi_linear/kda.py:58-185`` (chunk-parallel Eq. 6-9)
* ``kda_recurrent``  -- ``kimi_linear/kda.py:188-219`` (token recurrence, Eq. 1)

It is the parity checker for the CUDA kernels in ``-kimi-linear-_b200/csrc``.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it; the product path never calls it (the package raises
when its CUDA library is missing instead of falling back to anything here).

Pinning: ``tests/test_oracle_golden.py`` checks this module against golden
vectors produced by running the reference functions themselves
(``tests/golden/make_golden.py``, committed together with the ``.npz`` files).

Dtype semantics follow the reference exactly, because fp16 inputs take a
different arithmetic path there:

* ``td`` (the transient dtype) is fp16 when ``v`` is fp16, else fp32
  (``kda.py:115-116``); ``g``/``beta`` are promoted to fp32 (``kda.py:119-120``).
* fp16 transients: the pair decay ``exp(gc_c - gc_i)`` is formed in fp32,
  clamped at 11, rounded to fp16 and exponentiated in fp16 (``kda.py:159-162``);
  the masked products are fp16, reduced in fp32 (``kda.py:164,167``); the GEMMs
  take fp16 operands with fp32 accumulation and an fp16 result
  (``kda.py:172-182``).
* The carried state ``S`` is fp32 throughout (``kda.py:134-137,180-182``).

numpy has no bfloat16: a bf16 tensor is passed as a float32 array holding
bf16-representable values together with ``v_dtype="bf16"``; outputs in bf16
come back the same way (float32 arrays rounded to bf16, round-to-nearest-even).
The reference's ``kda_chunkwise`` raises on bf16 ``v`` (``kda.py:173``: fp32
``M`` times bf16 ``v``); for bf16 this oracle runs the fp32-transient path on
the bf16 values, which is the arithmetic ``kda.py:116`` intends for non-fp16
inputs, and rounds the output to bf16.
"""

from __future__ import annotations

import numpy as np

FP16_MAX_SAFE = 60000.0  # kimi_linear/fp16.py:97, applied at kda.py:217-218

_F32 = np.float32
_F16 = np.float16


# --------------------------------------------------------------------------- #
# dtype helpers
# --------------------------------------------------------------------------- #
def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round a float32 array to the nearest bfloat16 value (ties to even).

    Returns float32 storage.  NaN stays NaN; +-inf stays +-inf.
    """
    x = np.ascontiguousarray(x, dtype=_F32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(_F32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def _dtype_name(a: np.ndarray, override: str | None) -> str:
    if override is not None:
        if override not in ("f32", "f16", "bf16"):
            raise ValueError(f"unknown dtype name {override!r}")
        return override
    if a.dtype == _F16:
        return "f16"
    if a.dtype == _F32:
        return "f32"
    raise TypeError(f"unsupported array dtype {a.dtype}")


def cast_to(x: np.ndarray, name: str) -> np.ndarray:
    """Cast float data to the storage dtype ``name`` (the ``tensor.to(dtype)``
    of ``kda.py:185,219``)."""
    if name == "f32":
        return np.asarray(x, dtype=_F32)
    if name == "f16":
        return np.asarray(x, dtype=_F32).astype(_F16)
    return round_bf16(np.asarray(x, dtype=_F32))


def _mm(a: np.ndarray, b: np.ndarray, td) -> np.ndarray:
    """Batched GEMM with ``td`` operands: fp32 accumulation, one rounding of
    the result to ``td`` (the CPU ``bmm`` of the reference)."""
    out = np.matmul(a.astype(_F32), b.astype(_F32))
    return out.astype(td)


def _unit_lower_inverse(L: np.ndarray) -> np.ndarray:
    """``(I + L)^{-1}`` for strictly lower-triangular ``L`` (``[..., C, C]``).

    Forward substitution row by row, fp32: the restatement of
    ``torch.linalg.solve_triangular(eye + L, eye, upper=False,
    unitriangular=True)`` at ``kda.py:170``.
    """
    C = L.shape[-1]
    X = np.zeros_like(L, dtype=_F32)
    for c in range(C):
        row = np.zeros(L.shape[:-2] + (C,), dtype=_F32)
        row[..., c] = 1.0
        if c:
            # X[c, :] = e_c - sum_{i<c} L[c, i] X[i, :]
            row -= np.einsum("...i,...ij->...j", L[..., c, :c], X[..., :c, :])
        X[..., c, :] = row
    return X


# --------------------------------------------------------------------------- #
# kda_chunkwise  (kimi_linear/kda.py:58-185)
# --------------------------------------------------------------------------- #
def kda_chunkwise(q, k, v, g, beta, initial_state=None, chunk_size=64, tile_size=0,
                  state_dtype=None, v_dtype=None):
    """Chunkwise KDA forward.

    Args mirror ``kda_chunkwise`` (``kda.py:58-59``).  ``q``/``k``/``g`` are
    ``[B,T,H,K]``, ``v`` ``[B,T,H,V]``, ``beta`` ``[B,T,H]``, ``initial_state``
    ``[B,H,K,V]``.  ``state_dtype`` / ``v_dtype`` are dtype names ("f32",
    "f16", "bf16"); ``v_dtype`` defaults to the numpy dtype of ``v``.
    ``tile_size`` only changes the reference's summation blocking
    (``kda.py:130,150``) and is accepted and ignored.

    Returns ``(o [B,T,H,V], S [B,H,K,V])`` cast to ``v_dtype`` and
    ``state_dtype or v_dtype`` like ``kda.py:185``.
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = int(chunk_size)
    if C <= 0 or T % C != 0:
        # kda.py:124 -- the reshape to [B, NT, C, H, D] fails
        raise RuntimeError(f"T={T} is not a multiple of chunk_size={C}")
    NT = T // C
    out_name = _dtype_name(v, v_dtype)
    td = _F16 if out_name == "f16" else _F32          # kda.py:116

    def stor(x):  # storage dtype of q/k/v inside the kernel (td for fp16, else fp32)
        return np.asarray(x, dtype=td) if td == _F16 else np.asarray(x, dtype=_F32)

    qs, ks, vs = stor(q), stor(k), stor(v)
    g32 = np.asarray(g, dtype=_F32)                    # kda.py:119
    b32 = np.asarray(beta, dtype=_F32)                 # kda.py:120

    def ch(x):  # [B,T,H,D] -> [B,H,NT,C,D]  (kda.py:123-124)
        return x.reshape(B, NT, C, H, x.shape[-1]).transpose(0, 3, 1, 2, 4)

    qc, kc, vc, gch = ch(qs), ch(ks), ch(vs), ch(g32)
    bc = b32.reshape(B, NT, C, H).transpose(0, 3, 1, 2)  # [B,H,NT,C]  kda.py:127
    gc = np.cumsum(gch, axis=-2, dtype=_F32)             # kda.py:129
    q_scale = K ** -0.5                                  # kda.py:132
    tri_le = np.tril(np.ones((C, C), dtype=bool))        # i <= c
    tri_lt = np.tril(np.ones((C, C), dtype=bool), -1)    # i <  c

    if initial_state is None:
        S = np.zeros((B, H, K, V), dtype=_F32)           # kda.py:135
    else:
        S = np.array(initial_state, dtype=_F32, copy=True)  # kda.py:137
    o = np.empty((B, H, NT, C, V), dtype=td)

    # exp(gc_c - gc_i) overflows for i > c; those entries are masked by the
    # tril below exactly as in the reference (kda.py:165,168)
    with np.errstate(over="ignore", invalid="ignore"):
        return _chunk_loop(qc, kc, vc, gc, bc, S, o, NT, C, K, q_scale, td, tri_le, tri_lt,
                           B, H, V, out_name, state_dtype)


def _chunk_loop(qc, kc, vc, gc, bc, S, o, NT, C, K, q_scale, td, tri_le, tri_lt,
                B, H, V, out_name, state_dtype):
    for n in range(NT):                                   # kda.py:140
        # kda.py:141 -- the python-float scale multiplies in fp32, one rounding to td
        q_n = (qc[:, :, n].astype(_F32) * _F32(q_scale)).astype(td)
        k_n, v_n = kc[:, :, n], vc[:, :, n]
        g_n, b_n = gc[:, :, n], bc[:, :, n]
        exp_g = np.exp(g_n)                               # fp32 (0,1]  kda.py:144

        # pairwise decay D[c, i, :] = exp(gc_c - gc_i)   kda.py:159-162
        D = g_n[..., :, None, :] - g_n[..., None, :, :]
        if td == _F16:
            # fp16 exp = exp of the fp16 value evaluated in fp32, rounded once
            # (numpy's own float16 exp loses subnormals, torch's does not)
            D = np.minimum(D, _F32(11.0))
            D = np.exp(D.astype(_F16).astype(_F32)).astype(_F16)
        else:
            D = np.exp(D)
        # masked product-sums, fp32 reduction       kda.py:164-168
        kk = (k_n[..., :, None, :] * k_n[..., None, :, :] * D).sum(-1, dtype=_F32)
        L = np.where(tri_lt, kk * b_n[..., :, None], _F32(0.0)).astype(_F32)
        qk = (q_n[..., :, None, :] * k_n[..., None, :, :] * D).sum(-1, dtype=_F32)
        Aout = np.where(tri_le, qk, _F32(0.0)).astype(td)
        del D, kk, qk

        # UT transform                               kda.py:170-173
        M = _unit_lower_inverse(L)
        M = (M * b_n[..., None, :]).astype(td)
        w_n = _mm(M, (exp_g.astype(td) * k_n).astype(td), td)
        u_n = _mm(M, v_n, td)

        # output + state carry                       kda.py:176-182
        S_h = S.astype(td)
        pseudo_v = (u_n - _mm(w_n, S_h, td)).astype(td)
        o[:, :, n] = (_mm((q_n * exp_g.astype(td)).astype(td), S_h, td)
                      + _mm(Aout, pseudo_v, td)).astype(td)
        g_last = g_n[..., -1, :]
        S = S * np.exp(g_last)[..., None]
        kbar = (np.exp(g_n[..., -1:, :] - g_n).astype(td) * k_n).astype(td)
        S = (S + _mm(np.swapaxes(kbar, -1, -2), pseudo_v, td).astype(_F32)).astype(_F32)

    o = o.transpose(0, 2, 3, 1, 4).reshape(B, NT * C, H, V)   # kda.py:184
    return cast_to(o, out_name), cast_to(S, state_dtype or out_name)


# --------------------------------------------------------------------------- #
# kda_recurrent  (kimi_linear/kda.py:188-219)
# --------------------------------------------------------------------------- #
def kda_recurrent(q, k, v, g, beta, state=None, state_dtype=None, v_dtype=None):
    """Token-by-token KDA recurrence (paper Eq. 1), all arithmetic in fp32.

    Per token (``kda.py:207-216``): ``S <- Diag(exp g) S``;
    ``S <- S - beta k (k^T S)``; ``S <- S + beta k v^T``; ``o = S^T q`` with ``q``
    pre-scaled by ``K^-0.5`` (``kda.py:199``).  fp16 outputs are clamped to
    +-60000 (``kda.py:217-218``).
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    out_name = _dtype_name(v, v_dtype)
    q32 = np.asarray(q, dtype=_F32) * _F32(K ** -0.5)
    k32 = np.asarray(k, dtype=_F32)
    v32 = np.asarray(v, dtype=_F32)
    g32 = np.asarray(g, dtype=_F32)
    b32 = np.asarray(beta, dtype=_F32)
    S = (np.zeros((B, H, K, V), dtype=_F32) if state is None
         else np.array(state, dtype=_F32, copy=True))
    o = np.zeros((B, T, H, V), dtype=_F32)
    for t in range(T):
        S = S * np.exp(g32[:, t])[..., None]
        k_t = k32[:, t]
        b_t = b32[:, t][..., None]                       # [B,H,1]
        kS = np.einsum("bhk,bhkv->bhv", k_t, S)
        S = S - b_t[..., None] * k_t[..., None] * kS[..., None, :]
        S = S + b_t[..., None] * k_t[..., None] * v32[:, t][..., None, :]
        o[:, t] = np.einsum("bhk,bhkv->bhv", q32[:, t], S)
    if out_name == "f16":
        o = np.clip(o, -FP16_MAX_SAFE, FP16_MAX_SAFE)
    return cast_to(o, out_name), cast_to(S, state_dtype or out_name)


# --------------------------------------------------------------------------- #
# gradient of kda_recurrent / kda_chunkwise (torch autograd in the reference)
# --------------------------------------------------------------------------- #
def kda_backward(q, k, v, g, beta, state=None, do=None, dS=None):
    """Reverse-mode gradient of the token recurrence ``kda.py:207-216``, float64.

    The reference's trainers get these gradients from torch autograd through
    ``kda_recurrent`` (``kda.py:188-219``) or ``kda_chunkwise`` (``kda.py:58-185``,
    the same function).  This restates the chain rule of one step backwards::

        St = Diag(a) S_{t-1}, x = k^T St, u = beta (v - x), S_t = St + k u^T,
        o = S_t^T q'                         (a = exp g, q' = K^-0.5 q)

        dS += q' do^T;  dq' = S_t do;  du = dS^T k;  dv = beta du;
        dbeta = du . (v - x);  dx = -beta du;  dk = dS u + St dx;
        dSt = dS + k dx^T;  dg = rowsum(dSt (.) St);  dS_{t-1} = Diag(a) dSt

    ``do`` [B,T,H,V] / ``dS`` [B,H,K,V] may be None (zero).  Returns float64
    ``(dq, dk, dv, dg, dbeta, dstate)``; ``dstate`` is None without ``state``.
    Inputs are read as float32 values, like the reference (``kda.py:199-203``).
    The fp16 output clamp (``kda.py:217-218``) is not differentiated through.
    """
    f = np.float64
    B, T, H, K = q.shape
    V = v.shape[-1]
    sc = f(_F32(K ** -0.5))
    qs = np.asarray(q, dtype=_F32).astype(f) * sc
    k64 = np.asarray(k, dtype=_F32).astype(f)
    v64 = np.asarray(v, dtype=_F32).astype(f)
    al = np.exp(np.asarray(g, dtype=_F32).astype(f))
    b64 = np.asarray(beta, dtype=_F32).astype(f)
    do64 = (np.zeros((B, T, H, V)) if do is None
            else np.asarray(do, dtype=_F32).astype(f))
    S = (np.zeros((B, H, K, V)) if state is None
         else np.asarray(state, dtype=_F32).astype(f))
    prev, us, xs = [], [], []
    for t in range(T):                         # forward, keeping S_{t-1}, u, v - x
        prev.append(S)
        St = S * al[:, t][..., None]
        x = np.einsum("bhk,bhkv->bhv", k64[:, t], St)
        vmx = v64[:, t] - x
        u = b64[:, t][..., None] * vmx
        S = St + k64[:, t][..., None] * u[..., None, :]
        us.append(u)
        xs.append(vmx)
    dq = np.zeros((B, T, H, K)); dk = np.zeros((B, T, H, K)); dg = np.zeros((B, T, H, K))
    dv = np.zeros((B, T, H, V)); db = np.zeros((B, T, H))
    dSt_acc = np.zeros((B, H, K, V)) if dS is None else np.asarray(dS, dtype=_F32).astype(f)
    for t in range(T - 1, -1, -1):
        kt, at, bt = k64[:, t], al[:, t], b64[:, t]
        St = prev[t] * at[..., None]
        Snew = St + kt[..., None] * us[t][..., None, :]
        dSt_acc = dSt_acc + qs[:, t][..., None] * do64[:, t][..., None, :]
        dq[:, t] = np.einsum("bhkv,bhv->bhk", Snew, do64[:, t]) * sc
        du = np.einsum("bhkv,bhk->bhv", dSt_acc, kt)
        dv[:, t] = bt[..., None] * du
        db[:, t] = np.einsum("bhv,bhv->bh", du, xs[t])
        dx = -bt[..., None] * du
        dk[:, t] = (np.einsum("bhkv,bhv->bhk", dSt_acc, us[t])
                    + np.einsum("bhkv,bhv->bhk", St, dx))
        dSt = dSt_acc + kt[..., None] * dx[..., None, :]
        dg[:, t] = np.einsum("bhkv,bhkv->bhk", dSt, St)
        dSt_acc = dSt * at[..., None]
    return dq, dk, dv, dg, db, (None if state is None else dSt_acc)


# --------------------------------------------------------------------------- #
# comparison metric
# --------------------------------------------------------------------------- #
def rel_err(a, b) -> float:
    """Relative Frobenius error ``||a - b|| / ||b||`` computed in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    if den == 0.0:
        return float(num)
    return float(num / den)
