"""Pin the numpy oracle to the reference: golden vectors made by running the
reference's own ``kda_chunkwise`` / ``kda_recurrent`` (tests/golden/make_golden.py).

Tolerances: the fp32 oracle restates the fp32 arithmetic and must agree to
fp32 rounding (5e-6 relative; C=128 amplifies it).  The fp16 chunkwise path rounds ~20 transients
to fp16 per chunk (kda.py:159-182); sub-ulp fp32 differences flip some of those
roundings, so the bar is 2e-4 relative, 10x inside the 2e-3 product
tolerance.  Recurrent fp16/bf16 cases only round the output once.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import kda_oracle as O

TOL_CHUNK = {"f32": 5e-6, "f16": 2e-4, "bf16": 1e-4}
TOL_REC = {"f32": 1e-6, "f16": 2e-5, "bf16": 2e-5}


def _as_dtype(d, key):
    a = d[key]
    return a.astype(np.float16) if d["dtype_name"] == "f16" else a.astype(np.float32)


@pytest.mark.parametrize("name", golden_cases())
def test_recurrent_matches_reference(name):
    d = load_golden(name)
    q, k, v = (_as_dtype(d, x) for x in ("q", "k", "v"))
    o, S = O.kda_recurrent(q, k, v, d["g"], d["beta"], state=d["S0"],
                           state_dtype=d["state_dtype_name"], v_dtype=d["dtype_name"])
    assert o.shape == d["o_rec"].shape and S.shape == d["S_rec"].shape
    assert O.rel_err(o, d["o_rec"]) < TOL_REC[d["dtype_name"]]
    assert O.rel_err(S, d["S_rec"]) < 2e-6


@pytest.mark.parametrize("name", [n for n in golden_cases() if not n.startswith("rec_")])
def test_chunkwise_matches_reference(name):
    d = load_golden(name)
    q, k, v = (_as_dtype(d, x) for x in ("q", "k", "v"))
    o, S = O.kda_chunkwise(q, k, v, d["g"], d["beta"], initial_state=d["S0"],
                           chunk_size=d["C"], state_dtype=d["state_dtype_name"],
                           v_dtype=d["dtype_name"])
    tol = TOL_CHUNK[d["dtype_name"]]
    assert O.rel_err(o, d["o_chunk"]) < tol, O.rel_err(o, d["o_chunk"])
    assert O.rel_err(S, d["S_chunk"]) < tol, O.rel_err(S, d["S_chunk"])


def test_chunkwise_rejects_ragged_t():
    d = load_golden("c0_f32")
    with pytest.raises(RuntimeError):
        O.kda_chunkwise(d["q"][:, :100], d["k"][:, :100], d["v"][:, :100], d["g"][:, :100],
                        d["beta"][:, :100], chunk_size=64)


def test_chunkwise_equals_recurrent_config0():
    """The reference's own consistency claim (README.md:160) on config 0."""
    d = load_golden("c0_f32")
    o_c, S_c = O.kda_chunkwise(d["q"], d["k"], d["v"], d["g"], d["beta"], chunk_size=64)
    o_r, S_r = O.kda_recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"])
    assert O.rel_err(o_c, o_r) < 1e-5
    assert O.rel_err(S_c, S_r) < 1e-5


def test_round_bf16_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf, 0.0], dtype=np.float32)
    r = O.round_bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0); 1 + 3*2^-8 -> 1 + 2^-6
    assert r.tolist() == [1.0, 1.0, 1.015625, -2.5, np.inf, 0.0]
