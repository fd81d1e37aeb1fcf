"""CPU oracle of the static-buffer MLA decode step -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the attention core of ``MLA._decode_step_static``
(``kimi_linear/mla.py:117-181``) for NoPE layers (``qk_rope_head_dim == 0``):
everything between the projections and ``o_proj``.  It is the parity checker
of ``csrc/mla_decode.cu``; only ``tests/`` may import it.

Rounding points follow the reference: ``q_latent`` and the scores in fp32
(``mla.py:149-152``), softmax in fp32 (``:163``), ``p`` cast to the buffer's
dtype and ``mixed = p @ kv_buf`` returned in that dtype (``:164``), then
``mixed.float() @ W_v^T`` in fp32 (``:165-166``) and the result in the
activation dtype (``:168``).  bf16 arrays are float32 arrays holding bf16
values, as in ``kda_oracle``.

Pinned by ``tests/test_oracle_mla_golden.py`` against outputs of the
reference module itself (``tests/golden/make_golden_mla.py``).
"""

from __future__ import annotations

import numpy as np

from .kda_oracle import cast_to

_F32 = np.float32


def mla_decode_static(q_nope, c_kv, kv_buf, pos, w, num_heads, nope_dim, v_dim, scale,
                      dtype):
    """One decode step.  ``q_nope`` [B, 1, H, DN], ``c_kv`` [B, 1, KVL],
    ``kv_buf`` [B, L, KVL] (not modified), ``pos`` int, ``w`` =
    ``kv_b_proj.weight`` [H*(DN+DV), KVL], ``dtype`` "f16" or "bf16" (the
    activation and buffer dtype).  Returns ``(attn_out [B, 1, H*DV], kv_buf
    after the write at pos, pos + 1)``."""
    B, L, KVL = kv_buf.shape
    H, DN, DV = int(num_heads), int(nope_dim), int(v_dim)
    buf = np.array(kv_buf, dtype=_F32, copy=True)
    buf[:, pos] = np.asarray(c_kv, dtype=_F32).reshape(B, KVL)            # index_copy_ (:142)
    W = np.asarray(w, dtype=_F32).reshape(H, DN + DV, KVL)
    W_nope, W_v = W[:, :DN], W[:, DN:]                                     # :147
    qn = np.asarray(q_nope, dtype=_F32).reshape(B, H, DN)
    q_lat = np.einsum("bhd,hdc->bhc", qn, W_nope).astype(_F32)            # :149-150
    scores = np.einsum("bhc,blc->bhl", q_lat, buf).astype(_F32) * _F32(scale)   # :151-157
    invalid = np.arange(L) > pos                                           # :160-162
    scores[:, :, invalid] = -np.inf
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp((scores - m).astype(np.float64))
    p = (e / e.sum(axis=-1, keepdims=True)).astype(_F32)                   # :163
    p_t = cast_to(p, dtype).astype(np.float64)                             # p.to(buf.dtype)
    mixed = cast_to(np.einsum("bhl,blc->bhc", p_t, buf.astype(np.float64)).astype(_F32),
                    dtype)                                                 # :164
    out = np.einsum("bhc,hvc->bhv", mixed.astype(_F32), W_v).astype(_F32)  # :165-166
    out = cast_to(out, dtype).reshape(B, 1, H * DV)                        # :167-168
    return out, cast_to(buf, dtype), pos + 1
