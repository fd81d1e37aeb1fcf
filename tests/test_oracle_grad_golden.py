"""Pin the numpy backward oracle (``oracle/kda_oracle.py:kda_backward``) against
gradients from the reference's own autograd (``tests/golden/make_golden_grad.py``).
CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import grad_cases, load_grad
from oracle import kda_oracle as ko

# the oracle works in float64 on the fp32 input values; the reference's
# autograd in fp32 (fp16/bf16 leaves round their gradients)
TOL = {"f32": 2e-5, "f16": 2e-3, "bf16": 1e-2}
TOL_CHUNK = 1e-4      # autograd through the chunkwise algebra (solve, cumsum, exp)


@pytest.mark.parametrize("name", grad_cases())
def test_oracle_backward_matches_reference_autograd(name):
    c = load_grad(name)
    got = ko.kda_backward(c["q"], c["k"], c["v"], c["g"], c["beta"], c.get("S0"),
                          c["do"], c.get("dS"))
    tol = TOL_CHUNK if c["fn"] == "chunk" else TOL[c["dtype"]]
    for n, a in zip(("dq", "dk", "dv", "dg", "dbeta", "dS0"), got):
        if n == "dS0" and "S0" not in c:
            assert a is None
            continue
        want = c[n]
        if c["dtype"] != "f32" and n in ("dq", "dk", "dv"):
            a = ko.cast_to(a.astype(np.float32), c["dtype"])
        err = ko.rel_err(a, want)
        assert err < tol, f"{name} {n}: rel err {err:.3e} >= {tol}"


def test_oracle_backward_finite_difference():
    """Independent of the fixtures: directional derivative of the oracle's own
    forward (float64) against the oracle's backward."""
    rng = np.random.default_rng(3)
    B, T, H, K, V = 1, 9, 1, 32, 16
    q = rng.standard_normal((B, T, H, K))
    k = rng.standard_normal((B, T, H, K))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, V))
    g = -np.abs(rng.standard_normal((B, T, H, K))) * 0.1
    beta = rng.uniform(0.1, 0.9, (B, T, H))
    S0 = rng.standard_normal((B, H, K, V)) * 0.1
    do = rng.standard_normal((B, T, H, V))
    dS = rng.standard_normal((B, H, K, V))

    def fwd(q, k, v, g, beta, S0):
        sc = K ** -0.5
        S = S0.copy()
        o = np.zeros((B, T, H, V))
        for t in range(T):
            St = S * np.exp(g[:, t])[..., None]
            x = np.einsum("bhk,bhkv->bhv", k[:, t], St)
            S = St + k[:, t][..., None] * (beta[:, t][..., None] * (v[:, t] - x))[..., None, :]
            o[:, t] = np.einsum("bhk,bhkv->bhv", q[:, t] * sc, S)
        return (o * do).sum() + (S * dS).sum()

    # float32-exact inputs so the oracle's float32 read changes nothing
    xs = [a.astype(np.float32).astype(np.float64) for a in (q, k, v, g, beta, S0)]
    grads = ko.kda_backward(*xs, do.astype(np.float32), dS.astype(np.float32))
    do_, dS_ = do.astype(np.float32).astype(np.float64), dS.astype(np.float32).astype(np.float64)
    do, dS = do_, dS_
    eps = 1e-6
    for i, gr in enumerate(grads):
        d = rng.standard_normal(xs[i].shape)
        xp = [a.copy() for a in xs]; xm = [a.copy() for a in xs]
        xp[i] += eps * d; xm[i] -= eps * d
        fd = (fwd(*xp) - fwd(*xm)) / (2 * eps)
        an = float((gr * d).sum())
        assert abs(fd - an) <= 1e-6 * max(1.0, abs(an)), (i, fd, an)
