"""GPU parity of the KDA backward kernel (``csrc/kda_backward.cu``), reached
through torch autograd on ``kda_recurrent`` / ``kda_chunkwise`` exactly as the
reference's trainers differentiate the reference functions.

Bars (written here): fp32 gradients within 2e-5 relative Frobenius error of
the reference's autograd; fp16/bf16 leaves (whose gradients autograd rounds to
the leaf dtype) within 5e-3; the fp32 dg, dbeta and initial-state gradients
within 2e-5 for every input dtype.  Evidence:

1. the reference's own autograd gradients (tests/golden/grad_*.npz);
2. the numpy backward oracle on fresh seeded inputs (ragged T, K != V,
   no state, no output-gradient on one side);
3. at the prefill benchmark size (B=1, T=4096, H=16, K=V=128, fp16): the
   exact identities of a function linear in (v, S0) and in q, plus the oracle
   on one head.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import grad_cases, load_grad, pkg
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TOL_F32 = 2e-5
TOL_LOW = 5e-3


def rel(a, b):
    a = a.detach().double().cpu() if isinstance(a, torch.Tensor) else torch.as_tensor(a).double()
    b = b.detach().double().cpu() if isinstance(b, torch.Tensor) else torch.as_tensor(b).double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den else 1.0)


def _t(a, dev, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)


def _run(kb, fn, x, S0, sdt, C, do, dS):
    leaves = {n: x[n].clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")}
    s0 = None if S0 is None else S0.clone().requires_grad_(True)
    if fn == "chunk":
        o, S = kb.kda_chunkwise(leaves["q"], leaves["k"], leaves["v"], leaves["g"],
                                leaves["beta"], initial_state=s0, chunk_size=C, state_dtype=sdt)
    else:
        o, S = kb.kda_recurrent(leaves["q"], leaves["k"], leaves["v"], leaves["g"],
                                leaves["beta"], state=s0, state_dtype=sdt)
    outs, grads = [], []
    if do is not None:
        outs.append(o); grads.append(do)
    if dS is not None:
        outs.append(S); grads.append(dS.to(S.dtype))
    torch.autograd.backward(outs, grads)
    out = {f"d{n}": leaves[n].grad for n in leaves}
    out["dS0"] = None if s0 is None else s0.grad
    return out, o, S


@pytest.mark.parametrize("name", grad_cases())
def test_backward_vs_reference_autograd(name, cuda_dev):
    c = load_grad(name)
    dt = TORCH_DT[c["dtype"]]
    x = {n: _t(c[n], cuda_dev, dt) for n in ("q", "k", "v")}
    x.update(g=_t(c["g"], cuda_dev, torch.float32), beta=_t(c["beta"], cuda_dev, torch.float32))
    S0 = _t(c["S0"], cuda_dev, torch.float32) if "S0" in c else None
    sdt = TORCH_DT[c["state_dtype"]] if c["state_dtype"] else None
    do = _t(c["do"], cuda_dev, dt)
    dS = _t(c["dS"], cuda_dev, torch.float32) if "dS" in c else None
    got, _, _ = _run(pkg(), c["fn"], x, S0, sdt, c["C"], do, dS)
    for n in ("dq", "dk", "dv", "dg", "dbeta", "dS0"):
        if n == "dS0" and S0 is None:
            assert got[n] is None
            continue
        a = got[n]
        assert a.dtype == (dt if n in ("dq", "dk", "dv") else torch.float32), n
        assert torch.isfinite(a).all(), n
        tol = TOL_LOW if (c["dtype"] != "f32" and n in ("dq", "dk", "dv")) else TOL_F32
        assert rel(a.float(), c[n]) < tol, (name, n, rel(a.float(), c[n]))


CASES = [
    # B, T, H, K, V, dtype, s0, with_do, with_dS
    (2, 131, 2, 32, 48, torch.float32, True, True, True),
    (1, 200, 3, 64, 16, torch.bfloat16, False, True, False),
    (1, 97, 2, 128, 128, torch.float16, True, False, True),
    (1, 64, 1, 128, 32, torch.float32, True, True, True),
    (3, 1, 2, 64, 64, torch.float32, True, True, True),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}T{c[1]}H{c[2]}K{c[3]}V{c[4]}")
def test_backward_vs_oracle(case, cuda_dev):
    B, T, H, K, V, dt, s0, wdo, wdS = case
    kb = pkg()
    x = kb.synth.make_inputs(B, T, H, K, V, dtype=dt, seed=5, s0_std=0.02 if s0 else None,
                             device=cuda_dev)
    gen = torch.Generator(device=cuda_dev).manual_seed(9)
    do = torch.randn(B, T, H, V, device=cuda_dev, generator=gen).to(dt) if wdo else None
    dS = torch.randn(B, H, K, V, device=cuda_dev, generator=gen) * 0.1 if wdS else None
    got, _, _ = _run(kb, "rec", x, x["S0"], torch.float32 if dt != torch.float32 else None,
                     None, do, dS)
    np_ = lambda t: None if t is None else t.detach().float().cpu().numpy()  # noqa: E731
    want = O.kda_backward(np_(x["q"]), np_(x["k"]), np_(x["v"]), np_(x["g"]), np_(x["beta"]),
                          np_(x["S0"]), np_(do), np_(dS))
    for n, w in zip(("dq", "dk", "dv", "dg", "dbeta", "dS0"), want):
        if w is None:
            assert got[n] is None
            continue
        if dt != torch.float32 and n in ("dq", "dk", "dv"):
            w = O.cast_to(w.astype(np.float32), "f16" if dt == torch.float16 else "bf16")
            tol = TOL_LOW
        else:
            tol = TOL_F32
        assert rel(got[n].float(), w) < tol, (n, rel(got[n].float(), w))


def _steep_blocks_bwd(g, C=64):
    """(b, h, chunk, 16-row block, channel) count whose decay inside the block,
    g summed over its rows 2 .. 16, is below -80: the chunkwise backward leaves
    those out of its anchored block GEMMs and adds their pair terms exactly."""
    B, T, H, K = g.shape
    Tp = -(-T // C) * C
    x = torch.zeros(B, Tp, H, K, dtype=torch.float64, device=g.device)
    x[:, :T] = g.double()
    x = x.reshape(B, Tp // 16, 16, H, K)
    return int((x[:, :, 1:].sum(2) < -80).sum()), x[:, :, 0].numel()


@pytest.mark.parametrize("scale", [8.0, 20.0])
def test_backward_steep_decay_blocks_vs_oracle(scale, cuda_dev):
    kb = pkg()
    x = kb.synth.make_inputs(1, 192, 2, 64, 32, dtype=torch.float32, seed=8, s0_std=0.02,
                             device=cuda_dev)
    x["g"] = x["g"] * scale
    n_steep, total = _steep_blocks_bwd(x["g"])
    assert 0 < n_steep < total, (n_steep, total)
    gen = torch.Generator(device=cuda_dev).manual_seed(12)
    do = torch.randn(1, 192, 2, 32, device=cuda_dev, generator=gen)
    dS = torch.randn(1, 2, 64, 32, device=cuda_dev, generator=gen) * 0.1
    got, _, _ = _run(kb, "chunk", x, x["S0"], None, 64, do, dS)
    np_ = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    want = O.kda_backward(np_(x["q"]), np_(x["k"]), np_(x["v"]), np_(x["g"]), np_(x["beta"]),
                          np_(x["S0"]), np_(do), np_(dS))
    for n, w in zip(("dq", "dk", "dv", "dg", "dbeta", "dS0"), want):
        assert torch.isfinite(got[n]).all(), n
        assert rel(got[n].float(), w) < TOL_F32, (n, rel(got[n].float(), w))


def test_chunkwise_and_recurrent_share_the_gradient(cuda_dev):
    """Both functions are one function: the same backward through either."""
    kb = pkg()
    x = kb.synth.make_inputs(1, 256, 2, 128, 128, dtype=torch.float16, seed=2, s0_std=0.02,
                             device=cuda_dev)
    do = torch.randn(1, 256, 2, 128, device=cuda_dev).half()
    a, _, _ = _run(kb, "chunk", x, x["S0"], torch.float32, 64, do, None)
    b, _, _ = _run(kb, "rec", x, x["S0"], torch.float32, None, do, None)
    for n in a:
        assert torch.equal(a[n], b[n]), n


def test_full_size_identities_and_one_head(cuda_dev):
    """Prefill benchmark size.  With q, k, g, beta fixed, (o, S) is linear in
    (v, S0), so f = <do, o> + <dS, S> equals <dv, v> + <dS0, S0>; and o is
    linear in q, so <do, o> = <dq, q>.  One head's full gradient is checked
    against the oracle."""
    kb = pkg()
    B, T, H, K, V = 1, 4096, 16, 128, 128
    x = kb.synth.make_inputs(B, T, H, K, V, dtype=torch.float32, seed=0, s0_std=0.02,
                             device=cuda_dev)
    gen = torch.Generator(device=cuda_dev).manual_seed(4)
    do = torch.randn(B, T, H, V, device=cuda_dev, generator=gen)
    dS = torch.randn(B, H, K, V, device=cuda_dev, generator=gen) * 0.1
    got, o, S = _run(kb, "chunk", x, x["S0"], None, 64, do, dS)
    f = (do.double() * o.double()).sum() + (dS.double() * S.double()).sum()
    lin = (got["dv"].double() * x["v"].double()).sum() + \
        (got["dS0"].double() * x["S0"].double()).sum()
    assert abs((f - lin) / f).item() < 1e-4
    fo = (do.double() * o.double()).sum()
    assert abs((fo - (got["dq"].double() * x["q"].double()).sum()) / fo).item() < 1e-4
    h = 5
    np_ = lambda t: t.detach().float().cpu().numpy()[:, :, h:h + 1]  # noqa: E731
    want = O.kda_backward(np_(x["q"]), np_(x["k"]), np_(x["v"]), np_(x["g"]), np_(x["beta"]),
                          x["S0"][:, h:h + 1].cpu().numpy(), np_(do),
                          dS[:, h:h + 1].cpu().numpy())
    for n, w in zip(("dq", "dk", "dv", "dg", "dbeta"), want):
        assert rel(got[n][:, :, h], w[:, :, 0]) < 1e-4, (n, rel(got[n][:, :, h], w[:, :, 0]))
    assert rel(got["dS0"][:, h], want[5][:, 0]) < 1e-4
