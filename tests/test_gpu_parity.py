"""GPU parity of the CUDA kernels (called through the C ABI via ops.py).

Bars (from the task's north star): fp32 inputs within 1e-5 relative
Frobenius error of the reference; fp16/bf16 q/k/v with an fp32 state within
2e-3.  Three kinds of evidence:

1. the golden vectors of the reference itself (tests/golden);
2. the numpy oracle on fresh seeded inputs at sizes it finishes in seconds;
3. size-independent properties at the BASELINE sizes: chunkwise == recurrent,
   sequence continuation through the state, and linearity in (v, S0).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden, pkg
from oracle import kda_oracle as O

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 2e-3}


def rel(a, b):
    a = a.detach().double().cpu() if isinstance(a, torch.Tensor) else torch.as_tensor(a).double()
    b = b.detach().double().cpu() if isinstance(b, torch.Tensor) else torch.as_tensor(b).double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den else 1.0)


def _golden_tensors(d, dev):
    dt = TORCH_DT[d["dtype_name"]]
    t = lambda a, dtype: torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)  # noqa
    x = dict(q=t(d["q"], dt), k=t(d["k"], dt), v=t(d["v"], dt),
             g=t(d["g"], torch.float32), beta=t(d["beta"], torch.float32))
    x["S0"] = None if d["S0"] is None else t(d["S0"], torch.float32)
    sdt = TORCH_DT[d["state_dtype_name"]] if d["state_dtype_name"] else None
    return x, sdt


@pytest.mark.parametrize("name", golden_cases())
def test_recurrent_vs_reference_golden(name, cuda_dev):
    d = load_golden(name)
    x, sdt = _golden_tensors(d, cuda_dev)
    o, S = pkg().kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], state=x["S0"],
                               state_dtype=sdt)
    assert o.dtype == x["v"].dtype and S.dtype == (sdt or x["v"].dtype)
    tol = TOL[d["dtype_name"]]
    assert rel(o.float(), d["o_rec"]) < tol
    assert rel(S.float(), d["S_rec"]) < tol


@pytest.mark.parametrize("name", [n for n in golden_cases() if not n.startswith("rec_")])
def test_chunkwise_vs_reference_golden(name, cuda_dev):
    d = load_golden(name)
    x, sdt = _golden_tensors(d, cuda_dev)
    o, S = pkg().kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                               initial_state=x["S0"], chunk_size=d["C"], state_dtype=sdt)
    assert o.dtype == x["v"].dtype and S.dtype == (sdt or x["v"].dtype)
    assert o.shape == d["o_chunk"].shape and S.shape == d["S_chunk"].shape
    tol = TOL[d["dtype_name"]]
    assert rel(o.float(), d["o_chunk"]) < tol, rel(o.float(), d["o_chunk"])
    assert rel(S.float(), d["S_chunk"]) < tol, rel(S.float(), d["S_chunk"])


def _oracle_case(B, T, H, K, V, C, dtype, s0, seed, cuda_dev):
    s = pkg().synth
    x = s.make_inputs(B, T, H, K, V, dtype=dtype, seed=seed, s0_std=s0)
    sdt = torch.float32 if dtype != torch.float32 else None
    npy = lambda t: None if t is None else (t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy())  # noqa
    name = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[dtype]
    if dtype == torch.bfloat16:
        # the reference chunkwise runs bf16 values through its fp32 path
        ro, rS = O.kda_chunkwise(npy(x["q"]), npy(x["k"]), npy(x["v"]), npy(x["g"]),
                                 npy(x["beta"]), initial_state=npy(x["S0"]), chunk_size=C,
                                 state_dtype="f32", v_dtype="bf16")
    else:
        ro, rS = O.kda_chunkwise(npy(x["q"]), npy(x["k"]), npy(x["v"]), npy(x["g"]),
                                 npy(x["beta"]), initial_state=npy(x["S0"]), chunk_size=C,
                                 state_dtype="f32" if sdt else None)
    g = {k: (v.to(cuda_dev) if v is not None else None) for k, v in x.items()}
    o, S = pkg().kda_chunkwise(g["q"], g["k"], g["v"], g["g"], g["beta"],
                               initial_state=g["S0"], chunk_size=C, state_dtype=sdt)
    return o, S, ro, rS, TOL[name]


@pytest.mark.parametrize("B,T,H,K,V,C,dtype,s0", [
    (2, 512, 2, 128, 128, 64, torch.float16, None),
    (1, 384, 3, 128, 128, 128, torch.float16, 0.02),
    (1, 256, 2, 128, 128, 64, torch.bfloat16, 0.02),
    (2, 256, 2, 64, 64, 64, torch.float16, 0.02),
    (1, 512, 2, 64, 128, 64, torch.float32, 0.02),
    (1, 96, 1, 16, 48, 32, torch.float32, None),
])
def test_chunkwise_vs_oracle(B, T, H, K, V, C, dtype, s0, cuda_dev):
    o, S, ro, rS, tol = _oracle_case(B, T, H, K, V, C, dtype, s0, seed=1, cuda_dev=cuda_dev)
    assert rel(o.float(), ro.astype(np.float32)) < tol
    assert rel(S.float(), rS) < tol


# --------------------------------------------------------------------------- #
# size-independent properties at the BASELINE sizes
# --------------------------------------------------------------------------- #
def _cfg(cfg_id, dev, **kw):
    return {k: (v.to(dev) if v is not None else None)
            for k, v in pkg().synth.make_config(cfg_id, seed=3, **kw).items()}


@pytest.mark.parametrize("cfg_id", [1, 3])
def test_chunkwise_equals_recurrent_full_size(cfg_id, cuda_dev):
    over = {} if cfg_id == 1 else dict(B=2, T=8192)      # config 3 shapes, 1/4 of B and T
    x = _cfg(cfg_id, cuda_dev, **over)
    kb = pkg()
    oc, Sc = kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"],
                              initial_state=x["S0"], chunk_size=64, state_dtype=torch.float32)
    orr, Sr = kb.kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], state=x["S0"],
                               state_dtype=torch.float32)
    assert rel(oc.float(), orr.float()) < 2e-3
    assert rel(Sc, Sr) < 2e-3


def test_continuation_through_state(cuda_dev):
    """run(T) == run(T1) followed by run(T - T1, initial_state=S1)."""
    x = _cfg(1, cuda_dev)
    kb = pkg()
    T1 = 1536
    o, S = kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"], chunk_size=64,
                            state_dtype=torch.float32)
    sl = lambda t, a, b: t[:, a:b]  # noqa: E731
    o1, S1 = kb.kda_chunkwise(*(sl(x[n], 0, T1) for n in ("q", "k", "v", "g", "beta")),
                              chunk_size=64, state_dtype=torch.float32)
    o2, S2 = kb.kda_chunkwise(*(sl(x[n], T1, None) for n in ("q", "k", "v", "g", "beta")),
                              initial_state=S1, chunk_size=64, state_dtype=torch.float32)
    assert rel(torch.cat([o1, o2], 1).float(), o.float()) < 2e-3
    assert rel(S2, S) < 2e-3


def test_linearity_in_values_and_state(cuda_dev):
    """For fixed q, k, g, beta the core is linear in (v, S0)."""
    x = _cfg(3, cuda_dev, B=1, T=4096)
    kb = pkg()
    gen = torch.Generator(device=cuda_dev).manual_seed(11)
    v2 = torch.randn(x["v"].shape, device=cuda_dev, generator=gen).to(x["v"].dtype)
    S02 = torch.randn(x["S0"].shape, device=cuda_dev, generator=gen) * 0.02
    run = lambda v, s0: kb.kda_chunkwise(x["q"], x["k"], v, x["g"], x["beta"],  # noqa: E731
                                         initial_state=s0, state_dtype=torch.float32)
    oa, Sa = run(x["v"], x["S0"])
    ob, Sb = run(v2, S02)
    vs = (x["v"].float() + v2.float())
    oc, Sc = run(vs.to(x["v"].dtype), x["S0"] + S02)
    # bf16 rounding of v1 + v2 enters once: compare against the fp32-summed inputs' run
    assert rel(oc.float(), oa.float() + ob.float()) < 6e-3
    assert rel(Sc, Sa + Sb) < 6e-3


# --------------------------------------------------------------------------- #
# decode: CUDA-graph capture exactly as GraphedDecoder does it
# --------------------------------------------------------------------------- #
def test_recurrent_graph_capture_matches_eager(cuda_dev):
    """Static state + side-stream warm-up + capture + copy-back
    (kimi_linear/graph_decode.py:241-289), replayed step after step, equals
    one eager call over the whole sequence."""
    kb = pkg()
    B, H, K, V, steps = 8, 4, 128, 128, 48
    x = pkg().synth.make_inputs(B, steps, H, K, V, dtype=torch.float16, seed=5, s0_std=0.02)
    x = {k: v.to(cuda_dev) for k, v in x.items()}
    o_ref, S_ref = kb.kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], state=x["S0"],
                                    state_dtype=torch.float32)
    state = x["S0"].clone()
    tok = {n: x[n][:, :1].clone() for n in ("q", "k", "v", "g", "beta")}
    out = torch.empty(B, 1, H, V, device=cuda_dev, dtype=torch.float16)

    def step():
        o, S = kb.kda_recurrent(tok["q"], tok["k"], tok["v"], tok["g"], tok["beta"],
                                state=state, state_dtype=torch.float32)
        state.copy_(S)
        out.copy_(o)

    snap = state.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(s)
    state.copy_(snap)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    state.copy_(snap)
    outs = []
    for t in range(steps):
        for n in tok:
            tok[n].copy_(x[n][:, t:t + 1])
        graph.replay()
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert rel(torch.cat(outs, 1).float(), o_ref.float()) < 1e-5
    assert rel(state, S_ref) < 1e-5
    del graph


def test_recurrent_decode_config2_vs_oracle(cuda_dev):
    """Config 2 decode state shapes (K = V = 128, fp32 state ~ N(0, 0.02)) for
    64 steps on a 2x2 slice of the batch x heads, against the oracle."""
    s = pkg().synth
    x = s.make_inputs(2, 64, 2, 128, 128, dtype=torch.float16, seed=2, s0_std=0.02)
    ro, rS = O.kda_recurrent(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), x["g"].numpy(),
                             x["beta"].numpy(), state=x["S0"].numpy(), state_dtype="f32")
    g = {k: v.to(cuda_dev) for k, v in x.items()}
    state = g["S0"]
    outs = []
    for t in range(64):
        o, state = pkg().kda_recurrent(*(g[n][:, t:t + 1] for n in ("q", "k", "v", "g", "beta")),
                                       state=state, state_dtype=torch.float32)
        outs.append(o)
    assert rel(torch.cat(outs, 1).float(), ro.astype(np.float32)) < 2e-3
    assert rel(state, rS) < 1e-5


def test_decode_full_config2_batch_one_step(cuda_dev):
    """One decode step at the full config-2 batch (B=64, H=16, K=V=128, fp32
    state): 2048 state tiles, several per persistent CTA, against the oracle;
    then the same step from a state whose rows are not 16-byte aligned (the
    guarded kernel) must agree with it."""
    s = pkg().synth
    x = s.make_inputs(64, 1, 16, 128, 128, dtype=torch.float16, seed=11, s0_std=0.02)
    ro, rS = O.kda_recurrent(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), x["g"].numpy(),
                             x["beta"].numpy(), state=x["S0"].numpy(), state_dtype="f32")
    g = {k: v.to(cuda_dev) for k, v in x.items()}
    o, S = pkg().kda_recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"], state=g["S0"],
                               state_dtype=torch.float32)
    assert rel(o.float(), ro.astype(np.float32)) < 2e-3
    assert rel(S, rS) < 1e-5
    wide = torch.zeros(64, 16, 128, 129, device=cuda_dev)
    wide[..., 1:] = g["S0"]
    o2, S2 = pkg().kda_recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"],
                                 state=wide[..., 1:], state_dtype=torch.float32)
    assert rel(S2, S) < 1e-6 and rel(o2.float(), o.float()) < 1e-3


# --------------------------------------------------------------------------- #
# edge cases
# --------------------------------------------------------------------------- #
def test_noncontiguous_slices_like_the_module(cuda_dev):
    """Body/tail slices as KimiDeltaAttention.forward passes them
    (kda.py:519-520,526-527)."""
    kb = pkg()
    x = pkg().synth.make_inputs(2, 200, 2, 64, 64, dtype=torch.float16, seed=4)
    g = {k: (v.to(cuda_dev) if v is not None else None) for k, v in x.items()}
    body = 192
    ob, Sb = kb.kda_chunkwise(*(g[n][:, :body] for n in ("q", "k", "v", "g", "beta")),
                              chunk_size=64, state_dtype=torch.float32)
    ot, St = kb.kda_recurrent(*(g[n][:, body:] for n in ("q", "k", "v", "g", "beta")),
                              state=Sb, state_dtype=torch.float32)
    ofull, Sfull = kb.kda_recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"],
                                    state_dtype=torch.float32)
    assert rel(torch.cat([ob, ot], 1).float(), ofull.float()) < 2e-3
    assert rel(St, Sfull) < 2e-3
    # transposed layout with a unit innermost stride
    qt = g["q"].transpose(1, 2).contiguous().transpose(1, 2)
    o2, S2 = kb.kda_recurrent(qt, g["k"], g["v"], g["g"], g["beta"], state_dtype=torch.float32)
    assert rel(o2.float(), ofull.float()) < 1e-6


@pytest.mark.parametrize("sdt,s0dt", [(torch.float16, torch.float16),
                                      (torch.bfloat16, torch.float32),
                                      (None, torch.bfloat16)])
def test_state_dtypes(sdt, s0dt, cuda_dev):
    kb = pkg()
    x = pkg().synth.make_inputs(1, 128, 2, 32, 32, dtype=torch.float32, seed=6, s0_std=0.02)
    s0 = x["S0"].to(s0dt)
    npy = lambda t: t.float().numpy()  # noqa: E731
    name = {torch.float16: "f16", torch.bfloat16: "bf16", None: None}[sdt]
    ro, rS = O.kda_chunkwise(npy(x["q"]), npy(x["k"]), npy(x["v"]), npy(x["g"]),
                             npy(x["beta"]), initial_state=npy(s0), chunk_size=32,
                             state_dtype=name)
    g = {k: v.to(cuda_dev) for k, v in x.items()}
    o, S = kb.kda_chunkwise(g["q"], g["k"], g["v"], g["g"], g["beta"],
                            initial_state=s0.to(cuda_dev), chunk_size=32, state_dtype=sdt)
    assert S.dtype == (sdt or torch.float32)
    assert rel(o, ro) < 1e-5
    assert rel(S.float(), rS) < (1e-5 if sdt is None else 4e-3)


def test_empty_and_tiny(cuda_dev):
    kb = pkg()
    x = pkg().synth.make_inputs(2, 1, 3, 32, 16, dtype=torch.float32, seed=7, s0_std=0.02)
    g = {k: v.to(cuda_dev) for k, v in x.items()}
    # T = 1, chunk 1
    o, S = kb.kda_chunkwise(g["q"], g["k"], g["v"], g["g"], g["beta"], initial_state=g["S0"],
                            chunk_size=1)
    ro, rS = O.kda_recurrent(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), x["g"].numpy(),
                             x["beta"].numpy(), state=x["S0"].numpy())
    assert rel(o, ro) < 1e-5 and rel(S, rS) < 1e-5
    # T = 0: the state passes through (kda.py:134-137,185)
    e = {n: g[n][:, :0] for n in ("q", "k", "v", "g", "beta")}
    o0, S0 = kb.kda_chunkwise(e["q"], e["k"], e["v"], e["g"], e["beta"],
                              initial_state=g["S0"], chunk_size=64)
    assert o0.shape == (2, 0, 3, 16) and torch.equal(S0, g["S0"])
    o0, S0 = kb.kda_recurrent(e["q"], e["k"], e["v"], e["g"], e["beta"], state=g["S0"])
    assert torch.equal(S0, g["S0"])
    # B = 0
    z = {n: g[n][:0] for n in ("q", "k", "v", "g", "beta")}
    o0, S0 = kb.kda_chunkwise(z["q"], z["k"], z["v"], z["g"], z["beta"], chunk_size=1)
    assert o0.shape == (0, 1, 3, 16) and S0.shape == (0, 3, 32, 16)


def test_inputs_are_not_modified(cuda_dev):
    kb = pkg()
    x = pkg().synth.make_inputs(1, 128, 2, 128, 128, dtype=torch.float16, seed=8, s0_std=0.02)
    g = {k: v.to(cuda_dev) for k, v in x.items()}
    before = {k: v.clone() for k, v in g.items()}
    kb.kda_chunkwise(g["q"], g["k"], g["v"], g["g"], g["beta"], initial_state=g["S0"],
                     state_dtype=torch.float32)
    kb.kda_recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"], state=g["S0"],
                     state_dtype=torch.float32)
    torch.cuda.synchronize()
    for k in g:
        assert torch.equal(g[k], before[k]), k


def test_bad_arguments_raise_on_gpu(cuda_dev):
    kb = pkg()
    x = pkg().synth.make_inputs(1, 64, 2, 32, 32, dtype=torch.float32, seed=9)
    g = {k: (v.to(cuda_dev) if v is not None else None) for k, v in x.items()}
    with pytest.raises(RuntimeError):
        kb.kda_chunkwise(g["q"], g["k"], g["v"], g["g"], g["beta"], chunk_size=48)
    with pytest.raises(RuntimeError):
        kb.kda_recurrent(g["q"], g["k"][:, :, :1], g["v"], g["g"], g["beta"])
    with pytest.raises(RuntimeError):
        kb.kda_recurrent(g["q"], g["k"], g["v"], g["g"], g["beta"].cpu())
    big = torch.zeros(1, 4, 1, 512, device=cuda_dev)
    with pytest.raises(RuntimeError, match="unsupported shape"):
        kb.kda_recurrent(big, big, big[..., :32], big, torch.zeros(1, 4, 1, device=cuda_dev))


# --------------------------------------------------------------------------- #
# in-place state update (opt-in, not in the reference)
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("which,shape,dtype", [
    ("recurrent", (4, 1, 4, 128, 128), torch.float16),     # decode kernel
    ("recurrent", (2, 5, 2, 64, 32), torch.float32),       # guarded kernel, T > 1
    ("chunkwise", (1, 128, 2, 128, 128), torch.float16),   # tensor-core path
    ("chunkwise", (2, 64, 2, 32, 32), torch.float32),      # CUDA-core path
])
def test_inplace_equals_out_of_place(which, shape, dtype, cuda_dev):
    B, T, H, K, V = shape
    kb = pkg()
    x = kb.synth.make_inputs(B, T, H, K, V, dtype=dtype, seed=31, s0_std=0.02)
    g = {n: t.to(cuda_dev) for n, t in x.items()}
    args = [g[n] for n in ("q", "k", "v", "g", "beta")]
    fn = kb.kda_recurrent if which == "recurrent" else kb.kda_chunkwise
    kw = {} if which == "recurrent" else {"chunk_size": 64 if T % 64 == 0 else T}
    st = g["S0"].clone()
    o_ref, S_ref = fn(*args, st, state_dtype=torch.float32, **kw)
    assert torch.equal(st, g["S0"])                           # default: input untouched
    o_in, S_in = fn(*args, st, state_dtype=torch.float32, inplace=True, **kw)
    assert S_in is st
    assert torch.equal(S_in, S_ref) and torch.equal(o_in, o_ref)


def test_graph_decode_inplace_needs_no_copy_back(cuda_dev):
    """A captured single-token step that updates its static state in place
    (no copy-back), replayed step after step, equals one eager call."""
    kb = pkg()
    B, H, K, V, steps = 8, 4, 128, 128, 24
    x = kb.synth.make_inputs(B, steps, H, K, V, dtype=torch.float16, seed=33, s0_std=0.02)
    x = {k: v.to(cuda_dev) for k, v in x.items()}
    o_ref, S_ref = kb.kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"], state=x["S0"],
                                    state_dtype=torch.float32)
    state = x["S0"].clone()
    tok = {n: x[n][:, :1].clone() for n in ("q", "k", "v", "g", "beta")}
    out = torch.empty(B, 1, H, V, device=cuda_dev, dtype=torch.float16)

    def step():
        o, S = kb.kda_recurrent(tok["q"], tok["k"], tok["v"], tok["g"], tok["beta"],
                                state=state, state_dtype=torch.float32, inplace=True)
        out.copy_(o)

    snap = state.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    state.copy_(snap)
    outs = []
    for t in range(steps):
        for n in tok:
            tok[n].copy_(x[n][:, t:t + 1])
        graph.replay()
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert rel(torch.cat(outs, 1).float(), o_ref.float()) < 1e-5
    assert rel(state, S_ref) < 1e-5
    del graph
