"""GPU parity of the static-buffer MLA decode kernels (``csrc/mla_decode.cu``)
through the C ABI (``mla.mla_decode_core`` / ``mla.decode_step_static``).

Bars (written here): fp16 outputs within 2e-3 relative Frobenius error of the
reference, bf16 within 8e-3 (bf16 keeps 8 mantissa bits; the reference rounds
p and ``mixed`` to the buffer dtype, the kernel rounds p against a per-tile
running maximum first); the buffer row and ``pos`` exact.  Evidence: the
reference module's own outputs (tests/golden/mla_*.npz), the numpy oracle at
the 1.5B layer shapes (16 heads, kv_lora_rank 512, head dims 128), CUDA-graph
replay of consecutive steps, and the module-level drop-in.
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from conftest import load_mla, mla_cases, pkg
from oracle import kda_oracle as ko
from oracle import mla_oracle as mo

pytestmark = pytest.mark.gpu

TD = {"f16": torch.float16, "bf16": torch.bfloat16}
TOL = {"f16": 2e-3, "bf16": 8e-3}


def rel(a, b):
    a = a.detach().double().cpu() if isinstance(a, torch.Tensor) else torch.as_tensor(a).double()
    b = b.detach().double().cpu() if isinstance(b, torch.Tensor) else torch.as_tensor(b).double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den else 1.0)


def _t(a, dev, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)


@pytest.mark.parametrize("name", mla_cases())
def test_mla_vs_reference_module(name, cuda_dev):
    c = load_mla(name)
    dt = TD[c["dtype"]]
    buf = _t(c["kv_buf"], cuda_dev, dt)
    pos = torch.tensor([c["pos"]], dtype=torch.int64, device=cuda_dev)
    out = pkg().mla.mla_decode_core(_t(c["q_nope"], cuda_dev, dt), _t(c["c_kv"], cuda_dev, dt),
                                    buf, pos, _t(c["w"], cuda_dev, dt), c["H"], c["DN"], c["DV"],
                                    c["scale"])
    assert out.dtype == dt and tuple(out.shape) == (c["B"], 1, c["H"] * c["DV"])
    assert int(pos.item()) == c["pos_after"]
    assert torch.equal(buf[:, c["pos"]].float().cpu(), torch.from_numpy(c["kv_buf_after_row"]))
    keep = torch.ones(c["L"], dtype=torch.bool)
    keep[c["pos"]] = False
    assert torch.equal(buf[:, keep].float().cpu(), torch.from_numpy(c["kv_buf"])[:, keep])
    assert rel(out.float(), c["attn_out"]) < TOL[c["dtype"]], rel(out.float(), c["attn_out"])
    assert pkg().device_error() == 0


def _case(B, L, H, KVL, DN, DV, pos, dt, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, 1, H, DN, generator=g) * 0.5).to(dt)
    ck = torch.randn(B, 1, KVL, generator=g).to(dt)
    buf = torch.zeros(B, L, KVL).to(dt)
    buf[:, :pos] = torch.randn(B, pos, KVL, generator=g).to(dt)
    w = (torch.randn(H * (DN + DV), KVL, generator=g) * KVL ** -0.5).to(dt)
    return q, ck, buf, w


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("B,L,pos,dt", [
    (2, 1000, 700, torch.float16),      # 16 tiles, the last ones past pos (not loaded)
    (1, 8448, 8192, torch.bfloat16),    # configs[4]-like buffer: prompt 8192 + 256
    (4, 64, 63, torch.float16),         # one tile, pos at the last slot
    (3, 129, 128, torch.float16),       # ragged last tile (rows past L zero-filled)
])
def test_mla_1p5b_shapes_vs_oracle(B, L, pos, dt, cuda_dev):
    H, KVL, DN, DV = 16, 512, 128, 128
    q, ck, buf, w = _case(B, L, H, KVL, DN, DV, pos, dt, cuda_dev)
    scale = DN ** -0.5
    want, wbuf, _ = mo.mla_decode_static(_np(q), _np(ck), _np(buf), pos, _np(w), H, DN, DV,
                                         scale, "f16" if dt == torch.float16 else "bf16")
    gb = buf.to(cuda_dev)
    gp = torch.tensor([pos], dtype=torch.int64, device=cuda_dev)
    out = pkg().mla.mla_decode_core(q.to(cuda_dev), ck.to(cuda_dev), gb, gp, w.to(cuda_dev),
                                    H, DN, DV, scale)
    tol = 2e-3 if dt == torch.float16 else 8e-3
    assert rel(out.float(), want) < tol, rel(out.float(), want)
    assert int(gp.item()) == pos + 1
    assert torch.equal(gb[:, pos].float().cpu(), torch.from_numpy(wbuf[:, pos]))


def test_mla_graph_replay_advances_pos(cuda_dev):
    """Three captured-graph replays = three decode steps (pos read on the device)."""
    B, L, H, KVL, DN, DV, pos0 = 2, 300, 16, 512, 128, 128, 200
    dt = torch.float16
    q, ck, buf, w = _case(B, L, H, KVL, DN, DV, pos0, dt, cuda_dev, seed=3)
    scale = DN ** -0.5
    kb = pkg()
    gq, gck, gw = q.to(cuda_dev), ck.to(cuda_dev), w.to(cuda_dev)
    gb = buf.to(cuda_dev)
    gp = torch.tensor([pos0], dtype=torch.int64, device=cuda_dev)
    # warm up on a copy so the captured buffer starts from the same state
    side = torch.cuda.Stream(cuda_dev)
    side.wait_stream(torch.cuda.current_stream(cuda_dev))
    with torch.cuda.stream(side):
        kb.mla.mla_decode_core(gq, gck, gb.clone(), gp.clone(), gw, H, DN, DV, scale)
    torch.cuda.current_stream(cuda_dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = kb.mla.mla_decode_core(gq, gck, gb, gp, gw, H, DN, DV, scale)
    nb, npos = _np(buf), pos0
    for step in range(3):
        gq.copy_((torch.randn(B, 1, H, DN) * 0.5).to(dt))
        gck.copy_(torch.randn(B, 1, KVL).to(dt))
        graph.replay()
        torch.cuda.synchronize()
        want, nb, npos = mo.mla_decode_static(_np(gq), _np(gck), nb, npos, _np(gw), H, DN, DV,
                                              scale, "f16")
        assert int(gp.item()) == npos
        assert rel(out.float(), want) < 2e-3, (step, rel(out.float(), want))
    assert torch.equal(gb.float().cpu(), torch.from_numpy(nb))
    del graph


def test_decode_step_static_drop_in(cuda_dev):
    """The module-level drop-in on a stand-in with the reference's attributes."""
    B, L, H, KVL, DN, DV, hidden, pos = 2, 150, 16, 512, 128, 128, 256, 99
    dt = torch.float16
    torch.manual_seed(0)
    m = types.SimpleNamespace(
        num_heads=H, qk_nope_head_dim=DN, qk_rope_head_dim=0, v_head_dim=DV,
        scale=(DN + 0) ** -0.5,
        kv_b_proj=torch.nn.Linear(KVL, H * (DN + DV), bias=False).to(cuda_dev, dt),
        o_proj=torch.nn.Linear(H * DV, hidden, bias=False).to(cuda_dev, dt))
    q, ck, buf, _ = _case(B, L, H, KVL, DN, DV, pos, dt, cuda_dev, seed=5)
    state = {"c_kv_buf": buf.to(cuda_dev),
             "pos": torch.tensor([pos], dtype=torch.int64, device=cuda_dev)}
    x = torch.zeros(B, 1, hidden, device=cuda_dev, dtype=dt)
    with torch.no_grad():
        out, st = pkg().mla.decode_step_static(m, x, q.to(cuda_dev), None, ck.to(cuda_dev),
                                               None, state, True)
        core, _, _ = mo.mla_decode_static(_np(q), _np(ck), _np(buf), pos,
                                          _np(m.kv_b_proj.weight), H, DN, DV, m.scale, "f16")
        want = m.o_proj(torch.from_numpy(core).to(cuda_dev, dt))
    assert st is state and int(state["pos"].item()) == pos + 1
    assert rel(out.float(), want.float()) < 3e-3


def test_pos_outside_buffer_is_reported_not_written(cuda_dev):
    """pos >= L: the kernel's own bounds check skips the write and raises the
    device error word (the reference's index_copy_ would raise)."""
    B, L, H, KVL, DN, DV = 1, 64, 4, 64, 16, 16
    q, ck, buf, w = _case(B, L, H, KVL, DN, DV, L, torch.float16, cuda_dev, seed=7)
    gb = buf.to(cuda_dev)
    before = gb.clone()
    gp = torch.tensor([L], dtype=torch.int64, device=cuda_dev)
    kb = pkg()
    kb.device_error(clear=True)
    kb.mla.mla_decode_core(q.to(cuda_dev), ck.to(cuda_dev), gb, gp, w.to(cuda_dev), H, DN, DV,
                           DN ** -0.5)
    torch.cuda.synchronize()
    assert kb.device_error(clear=True) == 4
    assert torch.equal(gb, before)
