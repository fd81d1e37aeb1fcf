"""Pin the prologue / epilogue oracle to vectors made by the reference module
(``tests/golden/make_golden_fused.py``: the reference's own
``KimiDeltaAttention._projections`` and ``_output`` on CPU).

Tolerances: fp32 cases agree to fp32 rounding (1e-5 relative; the conv sums
run in a different order).  bf16 cases round several intermediates to bf16;
a one-ulp flip of such a rounding moves an element by 2^-8 relative, so the
bar is 2e-3 relative on the whole tensor (the product tolerance).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import fused_cases, load_fused
from oracle import kda_io_oracle as IO
from oracle.kda_oracle import rel_err

TOL = {"f32": 1e-5, "bf16": 2e-3}


def oracle_prologue(d):
    m = d["meta"]
    H, hd = m["H"], m["head_dim"]
    w = {n: d[f"w_{n}"].reshape(d[f"w_{n}"].shape[0], -1) for n in "qkv"}
    b = {n: d[f"b_{n}"] for n in "qkv" if f"b_{n}" in d}
    hist = {n: d[f"hist_{n}"] for n in "qkv"} if "hist_q" in d else None
    return IO.prologue(d["q_in"], d["k_in"], d["v_in"], d["gk"], d["beta_logit"], w, b,
                       d["A_log"], d["dt_bias"], H, hd, hd, m["l2norm_eps"], m["dtype"],
                       hist=hist, want_cache=m["mode"] != "prefill")


@pytest.mark.parametrize("name", fused_cases())
def test_prologue_oracle_matches_reference(name):
    d = load_fused(name)
    tol = TOL[d["meta"]["dtype"]]
    q, k, v, g, beta, cache = oracle_prologue(d)
    for key, got in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        assert got.shape == d[key].shape, key
        assert rel_err(got, d[key]) < tol, (key, rel_err(got, d[key]))
    if d["meta"]["mode"] != "prefill":
        for n in "qkv":
            assert np.array_equal(cache[n], d[f"new_{n}"]), n


@pytest.mark.parametrize("name", fused_cases())
def test_epilogue_oracle_matches_reference(name):
    d = load_fused(name)
    m = d["meta"]
    y = IO.epilogue(d["o_core"], d["og"], d["norm_w"], m["rms_eps"], m["dtype"])
    assert y.shape == d["y"].shape
    assert rel_err(y, d["y"]) < TOL[m["dtype"]], rel_err(y, d["y"])
