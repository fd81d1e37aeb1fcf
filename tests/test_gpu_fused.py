"""Fused prologue / epilogue kernels (``csrc/kda_io.cu``) on the GPU, through
the C ABI.

* against vectors made by the reference module's own ``_projections`` /
  ``_output`` (``tests/golden/make_golden_fused.py``), fed the same
  projection-GEMM outputs;
* against the numpy oracle at the 1.5B head shape in fp16 over several token
  tiles, with a conv history;
* the module drop-ins ``projections`` / ``output`` on a module shaped like
  ``KimiDeltaAttention`` (attribute names of ``kda.py:331-390``), against the
  same math written with torch ops, for prefill then one decode step.

Tolerances: 1e-5 relative for fp32, 2e-3 for fp16 / bf16 (north_star).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from conftest import fused_cases, load_fused, pkg
from oracle import kda_io_oracle as IO
from oracle.kda_oracle import rel_err

pytestmark = pytest.mark.gpu
TOL = {"f32": 1e-5, "bf16": 2e-3, "f16": 2e-3}
TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("name", fused_cases())
def test_prologue_vs_reference_golden(name, cuda_dev):
    d = load_fused(name)
    m = d["meta"]
    dt = TDT[m["dtype"]]
    t = lambda key, dtype=dt: torch.from_numpy(d[key]).to(cuda_dev, dtype)  # noqa: E731
    hist = {n: t(f"hist_{n}") for n in "qkv"} if "hist_q" in d else None
    q, k, v, g, beta, new = pkg().kda_prologue(
        t("q_in"), t("k_in"), t("v_in"), t("gk"), t("beta_logit"),
        [t(f"w_{n}") for n in "qkv"], [t(f"b_{n}") for n in "qkv"], t("A_log"), t("dt_bias"),
        m["H"], m["head_dim"], m["head_dim"], m["l2norm_eps"], conv_cache=hist,
        want_cache=m["mode"] != "prefill")
    torch.cuda.synchronize()
    tol = TOL[m["dtype"]]
    for key, got in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        assert tuple(got.shape) == d[key].shape, key
        assert rel(got.float(), d[key]) < tol, (key, rel(got.float(), d[key]))
    if m["mode"] != "prefill":
        for n in "qkv":
            assert torch.equal(new[n].float().cpu(), torch.from_numpy(d[f"new_{n}"])), n


@pytest.mark.parametrize("name", fused_cases())
def test_epilogue_vs_reference_golden(name, cuda_dev):
    d = load_fused(name)
    m = d["meta"]
    dt = TDT[m["dtype"]]
    y = pkg().kda_epilogue(torch.from_numpy(d["o_core"]).to(cuda_dev, dt),
                           torch.from_numpy(d["og"]).to(cuda_dev, dt),
                           torch.from_numpy(d["norm_w"]).to(cuda_dev), m["rms_eps"])
    torch.cuda.synchronize()
    assert tuple(y.shape) == d["y"].shape
    assert rel(y.float(), d["y"]) < TOL[m["dtype"]]


def test_prologue_epilogue_vs_oracle_fp16_1p5b_heads(cuda_dev):
    """B=2, T=300 (five token tiles, ragged last), H=4, K=V=128, fp16, with a
    conv history, against the oracle."""
    g = torch.Generator().manual_seed(21)
    B, T, H, K, cs = 2, 300, 4, 128, 4
    D = H * K
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    q_in, k_in, v_in, gk = (r(B, T, D).half() for _ in range(4))
    beta_logit = r(B, T, H).half()
    ws = [r(D, 1, cs) * 0.4 for _ in range(3)]
    bs = [r(D) * 0.1 for _ in range(3)]
    A_log = torch.log(torch.empty(H, K).uniform_(1, 16, generator=g))
    dt_bias = torch.log(torch.expm1(torch.empty(H, K).uniform_(1e-3, 0.1, generator=g)))
    hist = {n: r(B, cs - 1, D).half() for n in "qkv"}
    dev = lambda t: t.to(cuda_dev)  # noqa: E731
    q, k, v, gg, beta, new = pkg().kda_prologue(
        dev(q_in), dev(k_in), dev(v_in), dev(gk), dev(beta_logit), [dev(w) for w in ws],
        [dev(b) for b in bs], dev(A_log), dev(dt_bias), H, K, K, 1e-6,
        conv_cache={n: dev(h) for n, h in hist.items()}, want_cache=True)
    n = lambda t: t.float().numpy()  # noqa: E731
    ro = IO.prologue(n(q_in), n(k_in), n(v_in), n(gk), n(beta_logit),
                     {c: n(w).reshape(D, cs) for c, w in zip("qkv", ws)},
                     {c: n(b) for c, b in zip("qkv", bs)}, n(A_log), n(dt_bias), H, K, K,
                     1e-6, "f16", hist={c: n(h) for c, h in hist.items()}, want_cache=True)
    for got, want in zip((q, k, v, gg, beta), ro[:5]):
        assert rel(got.float(), want) < 2e-3
    for c in "qkv":
        assert torch.equal(new[c].cpu(), torch.from_numpy(ro[5][c]).half())
    o_core = r(B, T, H, K).half()
    og = r(B, T, D).half()
    w = r(H, K) * 0.5 + 1
    y = pkg().kda_epilogue(dev(o_core), dev(og), dev(w), 1e-6)
    assert rel(y.float(), IO.epilogue(n(o_core), n(og), n(w), 1e-6, "f16")) < 2e-3


class _Conv(nn.Module):
    def __init__(self, D, cs):
        super().__init__()
        self.conv = nn.Conv1d(D, D, cs, groups=D, bias=True)


class _Norm(nn.Module):
    def __init__(self, H, V):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(H, V))
        self.eps = 1e-6


class _KdaLike(nn.Module):
    """The attributes ``projections`` / ``output`` read, named as in
    ``KimiDeltaAttention.__init__`` (``kda.py:331-390``)."""

    def __init__(self, d=96, H=2, K=64, cs=4, rank=16):
        super().__init__()
        self.num_heads, self.head_dim, self.value_head_dim, self.conv_size = H, K, K, cs
        self.l2norm_eps = 1e-6
        self.in_proj_q, self.in_proj_k, self.in_proj_v = (nn.Linear(d, H * K) for _ in range(3))
        self.conv_q, self.conv_k, self.conv_v = (_Conv(H * K, cs) for _ in range(3))
        self.gk_proj = nn.Sequential(nn.Linear(d, rank), nn.Linear(rank, H * K))
        self.A_log = nn.Parameter(torch.log(torch.empty(H, K).uniform_(1, 16)))
        self.dt_bias = nn.Parameter(torch.full((H, K), -3.0))
        self.beta_proj = nn.Linear(d, H)
        self.og_proj = nn.Sequential(nn.Linear(d, rank), nn.Linear(rank, H * K))
        self.g_norm = _Norm(H, K)
        self.o_proj = nn.Linear(H * K, d)


def _torch_projections(m, x, hist):
    """The reference's _projections math in torch ops (test-side restatement)."""
    B, T, _ = x.shape
    H, K = m.num_heads, m.head_dim
    keep = m.conv_size - 1
    outs, new = [], {}
    for n, lin, cv in (("q", m.in_proj_q, m.conv_q), ("k", m.in_proj_k, m.conv_k),
                       ("v", m.in_proj_v, m.conv_v)):
        xi = lin(x)
        full = torch.cat([hist[n], xi], 1) if hist is not None else F.pad(xi, (0, 0, keep, 0))
        c = F.conv1d(full.transpose(1, 2), cv.conv.weight, cv.conv.bias,
                     groups=full.shape[-1]).transpose(1, 2)
        outs.append(F.silu(c).view(B, T, H, K))
        new[n] = full[:, -keep:]

    def l2(t):
        tf = t.float()
        return (tf * (tf * tf).sum(-1, keepdim=True).rsqrt().clamp(max=1 / m.l2norm_eps)).to(t.dtype)
    beta = torch.sigmoid(m.beta_proj(x).float())
    g = -torch.exp(m.A_log.float()) * F.softplus(m.gk_proj(x).view(B, T, H, K).float() + m.dt_bias.float())
    return l2(outs[0]), l2(outs[1]), outs[2], g, beta, new


def test_module_dropins_prefill_then_decode(cuda_dev):
    torch.manual_seed(5)
    fz = pkg().fused
    m = _KdaLike().to(cuda_dev)
    x = torch.randn(2, 33, 96, device=cuda_dev)
    with torch.no_grad():
        got = fz.projections(m, x, conv_cache=None, use_cache=True)
        want = _torch_projections(m, x, None)
        for a, b in zip(got[:5], want[:5]):
            assert rel(a, b) < 1e-5
        for n in "qkv":
            assert torch.equal(got[5][n], want[5][n])
        x1 = torch.randn(2, 1, 96, device=cuda_dev)
        got1 = fz.projections(m, x1, conv_cache=got[5], use_cache=True)
        want1 = _torch_projections(m, x1, want[5])
        for a, b in zip(got1[:5], want1[:5]):
            assert rel(a, b) < 1e-5
        o_core = torch.randn(2, 33, 2, 64, device=cuda_dev)
        out = fz.output(m, o_core, x)
        xf = o_core * torch.rsqrt(o_core.pow(2).mean(-1, keepdim=True) + 1e-6) * m.g_norm.weight
        ref = m.o_proj((xf * torch.sigmoid(m.og_proj(x).view(2, 33, 2, 64))).reshape(2, 33, 128))
        assert rel(out, ref) < 1e-5


def test_decode_chain_in_a_graph_matches_synchronised_calls(cuda_dev):
    """Three decode steps of one KDA layer at the 1.5B layer shape -- fused
    prologue from the conv cache, in-place recurrent step, fused epilogue --
    captured in one CUDA graph, where each kernel is launched as a
    programmatic dependent of the one before it (it may start before that one
    finished and must wait before touching its outputs), against the same
    calls with a device synchronisation after every kernel.  Bit-identical."""
    kb = pkg()
    B, H, K, cs = 4, 16, 128, 4
    D = H * K
    g = torch.Generator(device=cuda_dev).manual_seed(31)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=cuda_dev) * scale).half()

    steps = [dict(x=[rnd(B, 1, D) for _ in range(4)], beta=rnd(B, 1, H), og=rnd(B, 1, D))
             for _ in range(3)]
    w = [(torch.randn(D, 1, cs, generator=g, device=cuda_dev) * 0.4).half().float()
         for _ in range(3)]
    bias = [(torch.randn(D, generator=g, device=cuda_dev) * 0.1).half().float() for _ in range(3)]
    A_log = torch.log(torch.rand(H, K, generator=g, device=cuda_dev) * 15 + 1)
    dt = torch.log(torch.expm1(torch.rand(H, K, generator=g, device=cuda_dev) * 0.099 + 1e-3))
    nw = torch.rand(H, K, generator=g, device=cuda_dev) + 0.5
    hist0 = {n: rnd(B, cs - 1, D) for n in "qkv"}
    S0 = torch.randn(B, H, K, K, generator=g, device=cuda_dev) * 0.02

    def run(S, sync):
        hist, outs = hist0, []
        for st in steps:
            q, k, v, gg, beta, hist = kb.kda_prologue(*st["x"], st["beta"], w, bias, A_log, dt,
                                                      H, K, K, 1e-6, conv_cache=hist,
                                                      want_cache=True)
            if sync:
                torch.cuda.synchronize()
            o, _ = kb.kda_recurrent(q, k, v, gg, beta, state=S, state_dtype=torch.float32,
                                    inplace=True)
            if sync:
                torch.cuda.synchronize()
            outs.append(kb.kda_epilogue(o, st["og"], nw, 1e-6))
            if sync:
                torch.cuda.synchronize()
        return outs

    S_ref = S0.clone()
    ref = run(S_ref, True)

    S_g = S0.clone()
    side = torch.cuda.Stream(cuda_dev)
    side.wait_stream(torch.cuda.current_stream(cuda_dev))
    with torch.cuda.stream(side):
        run(S0.clone(), False)                       # warm-up outside the capture
    torch.cuda.current_stream(cuda_dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = run(S_g, False)
    S_g.copy_(S0)
    graph.replay()
    torch.cuda.synchronize()
    for a, r in zip(outs, ref):
        assert torch.equal(a, r)
    assert torch.equal(S_g, S_ref)
    assert kb.device_error() == 0
