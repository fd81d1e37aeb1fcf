"""Host-side behaviour of the reference-signature shim (no GPU needed):
argument checking, the gradient path, the absence of any CPU path, and
``install()`` patching the reference's module globals."""

from __future__ import annotations

import os
import sys
import types

import pytest
import torch

from conftest import pkg


def _inputs(T=64, dtype=torch.float32):
    s = pkg().synth
    return s.make_inputs(1, T, 2, 32, 32, dtype=dtype, seed=0)


def test_cpu_tensors_raise_no_fallback():
    x = _inputs()
    kb = pkg()
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        kb.kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"], chunk_size=64)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        kb.kda_recurrent(x["q"], x["k"], x["v"], x["g"], x["beta"])


def test_ragged_t_raises_like_reference():
    x = _inputs(T=40)
    with pytest.raises(RuntimeError, match="multiple of chunk_size"):
        pkg().kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"], chunk_size=64)
    with pytest.raises(ZeroDivisionError):
        pkg().kda_chunkwise(x["q"], x["k"], x["v"], x["g"], x["beta"], chunk_size=0)


def test_grad_path_has_no_cpu_fallback():
    """Inputs that require grad take the autograd path; it too needs CUDA."""
    x = _inputs()
    q = x["q"].clone().requires_grad_(True)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        pkg().kda_recurrent(q, x["k"], x["v"], x["g"], x["beta"])
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        pkg().kda_chunkwise(q, x["k"], x["v"], x["g"], x["beta"], chunk_size=64)
    with pytest.raises(RuntimeError, match="cannot record gradients"):
        pkg().kda_recurrent(q, x["k"], x["v"], x["g"], x["beta"], state=x["S0"],
                            inplace=True)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        pkg().ops.kda_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], None,
                               x["v"], None)


def test_fused_kernels_stay_forward_only():
    kb = pkg()
    t = torch.zeros(1, 4, 64, requires_grad=True)
    with pytest.raises(RuntimeError):
        kb.kda_epilogue(t.view(1, 4, 1, 64), t, torch.ones(1, 64), 1e-6)


def test_package_alias_registered():
    import importlib
    kb = pkg()
    assert importlib.import_module("kimi_linear_b200") is kb
    assert sys.modules["kimi_linear_b200.ops"] is kb.ops


def _fake_reference():
    """Module objects shaped like kimi_linear and kimi_linear.kda."""
    pkg_mod = types.ModuleType("fake_kimi_linear")
    kda_mod = types.ModuleType("fake_kimi_linear.kda")

    def ref_chunk(*a, **k):
        return "reference-chunkwise"

    def ref_rec(*a, **k):
        return "reference-recurrent"

    kda_mod.kda_chunkwise, kda_mod.kda_recurrent = ref_chunk, ref_rec
    pkg_mod.kda_chunkwise, pkg_mod.kda_recurrent = ref_chunk, ref_rec
    pkg_mod.kda = kda_mod
    return pkg_mod, kda_mod, ref_chunk, ref_rec


def test_install_patches_module_and_package_reexports():
    kb = pkg()
    pkg_mod, kda_mod, ref_chunk, ref_rec = _fake_reference()
    patched = kb.install(kda_module=kda_mod, package=pkg_mod)
    try:
        assert kda_mod.kda_chunkwise is kb.kda_chunkwise
        assert kda_mod.kda_recurrent is kb.kda_recurrent
        assert pkg_mod.kda_chunkwise is kb.kda_chunkwise
        assert pkg_mod.kda_recurrent is kb.kda_recurrent
        assert len(patched) == 4
    finally:
        kb.uninstall()
    assert kda_mod.kda_chunkwise is ref_chunk and pkg_mod.kda_recurrent is ref_rec


# the reference checkout, when this host has one: set KDA_REFERENCE_PATH to it
REF = os.environ.get("KDA_REFERENCE_PATH", "")


@pytest.mark.skipif(not REF or not os.path.isdir(os.path.join(REF, "kimi_linear")),
                    reason="KDA_REFERENCE_PATH does not name a reference checkout")
def test_reference_module_routes_through_patch():
    """With the reference checkout importable, KimiDeltaAttention.forward
    reaches the patched kernels (it resolves them at call time,
    kda.py:503,519,526): on CPU tensors our entry point raises its
    'needs CUDA tensors' error, which proves the routing."""
    sys.path.insert(0, REF)
    try:
        import kimi_linear
        from kimi_linear.configuration import KimiLinearConfig
        from kimi_linear.kda import KimiDeltaAttention
        kb = pkg()
        cfg = KimiLinearConfig.from_json(os.path.join(REF, "configs", "kimi_linear_tiny_test.json"))
        mod = KimiDeltaAttention(cfg)
        x = torch.randn(1, 32, cfg.hidden_size)
        kb.install()
        try:
            assert kimi_linear.kda_chunkwise is kb.kda_chunkwise
            with torch.no_grad(), pytest.raises(RuntimeError, match="CUDA tensors"):
                mod(x)
            with torch.no_grad(), pytest.raises(RuntimeError, match="CUDA tensors"):
                mod(x[:, :1], use_cache=True)
        finally:
            kb.uninstall()
        with torch.no_grad():
            assert mod(x).shape == x.shape   # the reference path again
    finally:
        sys.path.remove(REF)


def test_install_inplace_state_option():
    kb = pkg()
    pkg_mod, kda_mod, ref_chunk, ref_rec = _fake_reference()
    kb.install(kda_module=kda_mod, package=pkg_mod, inplace_state=True)
    try:
        assert kda_mod.kda_chunkwise is kb.kda_chunkwise_inplace
        assert kda_mod.kda_recurrent is kb.kda_recurrent_inplace
        assert pkg_mod.kda_recurrent is kb.kda_recurrent_inplace
    finally:
        kb.uninstall()
    assert kda_mod.kda_recurrent is ref_rec


def test_install_module_patches_and_restores_methods():
    """install_module routes a KimiDeltaAttention-like class's _projections /
    _output through the fused drop-ins; uninstall_module restores them."""
    kb = pkg()

    class FakeKDA:
        def _projections(self, x, conv_cache=None, use_cache=False):
            return "reference-projections"

        def _output(self, o_core, x):
            return "reference-output"

    orig_p, orig_o = FakeKDA._projections, FakeKDA._output
    kb.fused.install_module(FakeKDA)
    try:
        assert FakeKDA._projections is kb.fused.projections
        assert FakeKDA._output is kb.fused.output
    finally:
        kb.fused.uninstall_module()
    assert FakeKDA._projections is orig_p and FakeKDA._output is orig_o


def test_fused_cpu_tensors_raise():
    kb = pkg()
    x = torch.zeros(1, 4, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        kb.kda_epilogue(torch.zeros(1, 4, 2, 32), x, torch.ones(2, 32), 1e-6)


def test_mla_decode_host_checks():
    """The MLA decode drop-in: no CPU path, NoPE only, single token only."""
    kb = pkg()
    B, L, H, KVL, DN, DV = 1, 64, 4, 64, 16, 16
    q = torch.zeros(B, 1, H, DN, dtype=torch.float16)
    ck = torch.zeros(B, 1, KVL, dtype=torch.float16)
    buf = torch.zeros(B, L, KVL, dtype=torch.float16)
    pos = torch.tensor([3], dtype=torch.int64)
    w = torch.zeros(H * (DN + DV), KVL, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        kb.mla.mla_decode_core(q, ck, buf, pos, w, H, DN, DV, DN ** -0.5)
    m = types.SimpleNamespace(num_heads=H, qk_nope_head_dim=DN, qk_rope_head_dim=8,
                              v_head_dim=DV, scale=0.1)
    state = {"c_kv_buf": buf, "pos": pos}
    with pytest.raises(NotImplementedError, match="NoPE"):
        kb.mla.decode_step_static(m, torch.zeros(B, 1, 8), q, None, ck, None, state, True)
    with pytest.raises(RuntimeError, match="single-token"):
        kb.mla.decode_step_static(m, torch.zeros(B, 2, 8), q, None, ck, None, state, True)


def test_install_mla_patches_and_restores():
    kb = pkg()

    class FakeMLA:
        def _decode_step_static(self, *a):
            return "reference"

    kb.mla.install_mla(FakeMLA)
    assert FakeMLA._decode_step_static is kb.mla.decode_step_static
    kb.mla.uninstall_mla()
    assert FakeMLA()._decode_step_static() == "reference"
