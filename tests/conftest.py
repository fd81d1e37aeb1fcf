"""Shared pytest setup for the KDA B200 tests.

Marker ``gpu``: needs a B200 (sm_100) and the built ``libkda_b200.so``; those
tests are the parity tests proper and call the kernels through the C ABI.
Everything else runs on a CPU-only host.
"""

from __future__ import annotations

import glob
import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def pkg():
    """The package (its directory name is not an identifier)."""
    return importlib.import_module("-kimi-linear-_b200")


def golden_cases():
    """Golden cases of the KDA core (tests/golden/make_golden.py)."""
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if not os.path.basename(p).startswith(("fused_", "grad_", "mla_")))


def mla_cases():
    """Golden static-buffer MLA decode steps (tests/golden/make_golden_mla.py)."""
    return sorted(os.path.basename(p)[:-4]
                  for p in glob.glob(os.path.join(GOLDEN, "mla_*.npz")))


def load_mla(name):
    """Golden MLA case ``name``: arrays plus B, L, H, KVL, DN, DV, hidden, pos,
    pos_after, dtype (string) and scale."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    B, L, H, KVL, DN, DV, hidden, pos, pos_after = (int(x) for x in d["meta"])
    d.update(B=B, L=L, H=H, KVL=KVL, DN=DN, DV=DV, hidden=hidden, pos=pos,
             pos_after=pos_after, dtype=str(d["dtype"]), scale=float(d["scale"]))
    return d


def grad_cases():
    """Golden gradient cases (tests/golden/make_golden_grad.py)."""
    return sorted(os.path.basename(p)[:-4]
                  for p in glob.glob(os.path.join(GOLDEN, "grad_*.npz")))


def load_grad(name):
    """Golden gradient case ``name``: dict of numpy arrays plus ``fn``, ``dtype``,
    ``state_dtype`` (strings) and B, T, H, K, V, C."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    B, T, H, K, V, C = (int(x) for x in d["meta"])
    d.update(B=B, T=T, H=H, K=K, V=V, C=None if C < 0 else C, fn=str(d["fn"]),
             dtype=str(d["dtype"]), state_dtype=str(d["state_dtype"]) or None)
    return d


def fused_cases():
    """Golden cases of the fused prologue / epilogue (make_golden_fused.py)."""
    return sorted(os.path.basename(p)[:-4]
                  for p in glob.glob(os.path.join(GOLDEN, "fused_*.npz")))


def load_fused(name):
    """Fused golden case ``name``: dict of numpy arrays plus ``meta`` (a dict)."""
    import json
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def load_golden(name):
    """Golden case ``name`` as a dict of numpy arrays plus metadata."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    src = str(d.get("inputs_from", ""))
    if src:
        base = np.load(os.path.join(GOLDEN, f"{src}.npz"))
        for key in ("q", "k", "v", "g", "beta"):
            d[key] = base[key]
    B, T, H, K, V, C = (int(x) for x in d["meta"])
    d.update(B=B, T=T, H=H, K=K, V=V, C=None if C < 0 else C,
             dtype_name=str(d["dtype"]), state_dtype_name=str(d["state_dtype"]) or None)
    if "S0" not in d:
        d["S0"] = None
    return d


def gpu_available():
    try:
        import torch
        if not torch.cuda.is_available():
            return False
        major, minor = torch.cuda.get_device_capability(0)
        return (major, minor) == (10, 0)
    except Exception:
        return False


@pytest.fixture(scope="session")
def kb():
    return pkg()


@pytest.fixture(scope="session")
def cuda_dev():
    if not gpu_available():
        pytest.fail("gpu test selected but no sm_100 GPU is visible")
    import torch
    return torch.device("cuda", 0)
