"""Pin the MLA decode oracle (``oracle/mla_oracle.py``) against the reference
module's own ``MLA._decode_step_static`` (``tests/golden/make_golden_mla.py``).
CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_mla, mla_cases
from oracle import kda_oracle as ko
from oracle import mla_oracle as mo

# fp16/bf16 outputs: the oracle reduces in float64 / numpy fp32 order, the
# reference in torch's; both round to the same dtype at the same points
TOL = {"f16": 2e-3, "bf16": 8e-3}


@pytest.mark.parametrize("name", mla_cases())
def test_oracle_matches_reference_module(name):
    c = load_mla(name)
    out, buf, pos1 = mo.mla_decode_static(c["q_nope"], c["c_kv"], c["kv_buf"], c["pos"],
                                          c["w"], c["H"], c["DN"], c["DV"], c["scale"],
                                          c["dtype"])
    assert pos1 == c["pos_after"] == c["pos"] + 1
    np.testing.assert_array_equal(buf[:, c["pos"]], c["kv_buf_after_row"])
    keep = np.ones(c["L"], bool)
    keep[c["pos"]] = False
    np.testing.assert_array_equal(buf[:, keep], c["kv_buf"][:, keep])
    err = ko.rel_err(out, c["attn_out"])
    assert err < TOL[c["dtype"]], (name, err)
