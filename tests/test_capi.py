"""C-ABI checks that need no GPU: the library loads, exports every function
``include/kda_b200.h`` declares, agrees with the ctypes struct layout, and
rejects malformed arguments before touching the device."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import REPO, pkg

HEADER = os.path.join(REPO, "include", "kda_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b((?:kda|mla)_\w+)\s*\(", src,
                                 flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    return pkg()._lib.load()


def test_header_declares_expected_symbols():
    names = _declared_functions()
    assert set(names) == set(pkg()._lib.EXPORTED), names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name


def test_struct_layout_matches(lib):
    L = pkg()._lib
    assert lib.kda_args_size() == ctypes.sizeof(L.KdaArgs)
    assert lib.mla_decode_args_size() == ctypes.sizeof(L.MlaDecodeArgs)
    assert lib.kda_backward_args_size() == ctypes.sizeof(L.KdaBackwardArgs)
    assert lib.kda_abi_version() == L.ABI_VERSION


def test_status_strings(lib):
    L = pkg()._lib
    for code in range(0, 11):
        s = lib.kda_status_string(code).decode()
        assert s and s != "unknown status", code
    assert lib.kda_status_string(999).decode() == "unknown status"
    assert L.status_string(L.KDA_ERR_CHUNK) == "T is not a multiple of chunk_size"


def _args(**kw):
    L = pkg()._lib
    a = L.KdaArgs()
    a.abi_version = L.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V = 1, 64, 1, 32, 32
    a.chunk_size = 64
    a.io_dtype = a.state_out_dtype = a.state_in_dtype = L.DTYPE_F32
    a.scale = 32 ** -0.5
    fake = 1 << 20   # never dereferenced: every case below fails validation first
    for name in ("q", "k", "v", "g", "beta", "o", "state_out"):
        setattr(a, name, fake)
    for name, n in (("q_stride", 4), ("k_stride", 4), ("v_stride", 4), ("g_stride", 4),
                    ("o_stride", 4), ("state_out_stride", 4), ("state_in_stride", 4)):
        setattr(a, name, (ctypes.c_int64 * n)(2048, 32, 32, 1))
    a.beta_stride = (ctypes.c_int64 * 3)(64, 1, 1)
    for key, val in kw.items():
        setattr(a, key, val)
    return a


def test_validation_errors_without_device(lib):
    L = pkg()._lib
    call = lambda a: lib.kda_chunkwise_fwd(ctypes.byref(a), None)  # noqa: E731
    assert lib.kda_chunkwise_fwd(None, None) == L.KDA_ERR_NULL_POINTER
    assert call(_args(abi_version=99)) == L.KDA_ERR_SHAPE
    assert call(_args(T=100)) == L.KDA_ERR_CHUNK                     # kda.py:124
    assert call(_args(chunk_size=0)) == L.KDA_ERR_CHUNK
    assert call(_args(K=512)) == L.KDA_ERR_SHAPE
    assert call(_args(io_dtype=7)) == L.KDA_ERR_DTYPE
    assert call(_args(q=None)) == L.KDA_ERR_NULL_POINTER
    assert call(_args(state_out=None)) == L.KDA_ERR_NULL_POINTER
    bad = _args()
    bad.v_stride = (ctypes.c_int64 * 4)(2048, 32, 32, 2)
    assert call(bad) == L.KDA_ERR_STRIDE
    assert call(_args(io_dtype=L.DTYPE_F16, q=(1 << 20) + 1)) == L.KDA_ERR_ALIGNMENT
    # the recurrent entry point accepts any T
    assert lib.kda_recurrent_fwd(ctypes.byref(_args(T=37, q=None)), None) == L.KDA_ERR_NULL_POINTER
    # B == 0: nothing to do, success without a device
    assert call(_args(B=0)) == L.KDA_OK
    # an in-place state must be exactly the same view as the input state
    alias = _args(state_in=1 << 21, state_out=1 << 21)
    alias.state_in_dtype = L.DTYPE_F16
    assert call(alias) == L.KDA_ERR_DTYPE
    alias = _args(state_in=1 << 21, state_out=1 << 21)
    alias.state_in_dtype = L.DTYPE_F32
    alias.state_in_stride = (ctypes.c_int64 * 4)(4096, 1024, 64, 1)
    assert call(alias) == L.KDA_ERR_STRIDE


def test_path_selection_queries_need_no_device(lib):
    a = _args()
    assert lib.kda_chunkwise_path(ctypes.byref(a)) in (0, 1)
    assert lib.kda_chunkwise_path(ctypes.byref(_args(T=100))) == -pkg()._lib.KDA_ERR_CHUNK


def _mla_args(**kw):
    L = pkg()._lib
    a = L.MlaDecodeArgs()
    a.abi_version = L.ABI_VERSION
    a.B, a.L, a.H, a.KVL, a.DN, a.DV = 2, 128, 16, 512, 128, 128
    a.io_dtype = L.DTYPE_F16
    a.scale = 128 ** -0.5
    fake = 1 << 20                       # aligned non-null addresses; validation only
    a.q_nope = a.c_kv = a.kv_buf = a.w = a.out = a.pos = a.workspace = fake
    a.q_nope_stride = (ctypes.c_int64 * 3)(16 * 128, 128, 1)
    a.c_kv_stride = (ctypes.c_int64 * 2)(512, 1)
    a.kv_buf_stride = (ctypes.c_int64 * 3)(128 * 512, 512, 1)
    a.w_stride = (ctypes.c_int64 * 2)(512, 1)
    a.out_stride = (ctypes.c_int64 * 3)(16 * 128, 128, 1)
    a.workspace_bytes = 0
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_mla_argument_errors_before_any_launch(lib):
    """Argument errors come back as status codes before anything touches the GPU."""
    L = pkg()._lib
    call = lambda a: lib.mla_decode_fwd(ctypes.byref(a), None)  # noqa: E731
    assert call(_mla_args(H=17)) == L.KDA_ERR_SHAPE
    assert call(_mla_args(KVL=96)) == L.KDA_ERR_SHAPE
    assert call(_mla_args(io_dtype=L.DTYPE_F32)) == L.KDA_ERR_DTYPE
    assert call(_mla_args(kv_buf=None)) == L.KDA_ERR_NULL_POINTER
    assert call(_mla_args(kv_buf_stride=(ctypes.c_int64 * 3)(128 * 512, 512, 2))) == \
        L.KDA_ERR_STRIDE
    assert call(_mla_args(kv_buf_stride=(ctypes.c_int64 * 3)(128 * 513, 513, 1))) == \
        L.KDA_ERR_ALIGNMENT
    assert call(_mla_args()) == L.KDA_ERR_WORKSPACE     # workspace_bytes = 0
    assert lib.mla_decode_workspace_bytes(ctypes.byref(_mla_args())) > 0
    assert lib.mla_decode_workspace_bytes(ctypes.byref(_mla_args(KVL=96))) == 0
