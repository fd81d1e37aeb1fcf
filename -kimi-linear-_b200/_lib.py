"""ctypes binding of ``libkda_b200.so`` (the C ABI in ``include/kda_b200.h``).

The library is loaded lazily on first use.  If it is missing or does not load,
:class:`KdaLibraryError` is raised: the KDA entry points have no CPU or
pure-PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkda_b200.so")

ABI_VERSION = 2

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
FLAG_FORCE_SIMT = 1

# kda_status_t
KDA_OK = 0
KDA_ERR_NULL_POINTER = 1
KDA_ERR_SHAPE = 2
KDA_ERR_DTYPE = 3
KDA_ERR_STRIDE = 4
KDA_ERR_ALIGNMENT = 5
KDA_ERR_ARCH = 6
KDA_ERR_LAUNCH = 7
KDA_ERR_CHUNK = 8
KDA_ERR_WORKSPACE = 9
KDA_ERR_CUDA = 10

# every symbol include/kda_b200.h declares
EXPORTED = (
    "kda_chunkwise_fwd",
    "kda_recurrent_fwd",
    "kda_chunkwise_fwd_noalloc",
    "kda_chunkwise_workspace_bytes",
    "kda_chunkwise_path",
    "kda_status_string",
    "kda_device_supported",
    "kda_device_error",
    "kda_prologue_fwd",
    "kda_epilogue_fwd",
    "kda_prologue_args_size",
    "kda_epilogue_args_size",
    "kda_backward",
    "kda_backward_ckpt_floats",
    "kda_backward_args_size",
    "mla_decode_fwd",
    "mla_decode_workspace_bytes",
    "mla_decode_args_size",
    "kda_args_size",
    "kda_abi_version",
)

_I64x4 = ctypes.c_int64 * 4
_I64x3 = ctypes.c_int64 * 3


class KdaArgs(ctypes.Structure):
    """Mirror of ``struct KdaArgs`` (field order and types must match)."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32),
        ("K", ctypes.c_int32), ("V", ctypes.c_int32),
        ("chunk_size", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("state_in_dtype", ctypes.c_int32),
        ("state_out_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("flags", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_stride", _I64x4),
        ("k", ctypes.c_void_p), ("k_stride", _I64x4),
        ("v", ctypes.c_void_p), ("v_stride", _I64x4),
        ("g", ctypes.c_void_p), ("g_stride", _I64x4),
        ("beta", ctypes.c_void_p), ("beta_stride", _I64x3),
        ("state_in", ctypes.c_void_p), ("state_in_stride", _I64x4),
        ("o", ctypes.c_void_p), ("o_stride", _I64x4),
        ("state_out", ctypes.c_void_p), ("state_out_stride", _I64x4),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


_I64x2 = ctypes.c_int64 * 2
_P3 = ctypes.c_void_p * 3


class KdaPrologueArgs(ctypes.Structure):
    """Mirror of ``struct KdaPrologueArgs``."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32),
        ("K", ctypes.c_int32), ("V", ctypes.c_int32),
        ("conv_size", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("gate_dtype", ctypes.c_int32),
        ("l2norm_eps", ctypes.c_float),
        ("q_in", ctypes.c_void_p), ("q_in_stride", _I64x2),
        ("k_in", ctypes.c_void_p), ("k_in_stride", _I64x2),
        ("v_in", ctypes.c_void_p), ("v_in_stride", _I64x2),
        ("conv_w", _P3),
        ("conv_b", _P3),
        ("hist", _P3),
        ("hist_batch_stride", _I64x3),
        ("new_hist", _P3),
        ("gk", ctypes.c_void_p), ("gk_stride", _I64x2),
        ("beta_logit", ctypes.c_void_p), ("beta_logit_stride", _I64x2),
        ("A_log", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("q", ctypes.c_void_p), ("q_stride", _I64x4),
        ("k", ctypes.c_void_p), ("k_stride", _I64x4),
        ("v", ctypes.c_void_p), ("v_stride", _I64x4),
        ("g", ctypes.c_void_p), ("g_stride", _I64x4),
        ("beta", ctypes.c_void_p), ("beta_stride", _I64x3),
    ]


class KdaEpilogueArgs(ctypes.Structure):
    """Mirror of ``struct KdaEpilogueArgs``."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32),
        ("V", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("o", ctypes.c_void_p), ("o_stride", _I64x4),
        ("og", ctypes.c_void_p), ("og_stride", _I64x2),
        ("weight", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("y_stride", _I64x2),
    ]


class KdaBackwardArgs(ctypes.Structure):
    """Mirror of ``struct KdaBackwardArgs``."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32),
        ("K", ctypes.c_int32), ("V", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("state_in_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q", ctypes.c_void_p), ("q_stride", _I64x4),
        ("k", ctypes.c_void_p), ("k_stride", _I64x4),
        ("v", ctypes.c_void_p), ("v_stride", _I64x4),
        ("g", ctypes.c_void_p), ("g_stride", _I64x4),
        ("beta", ctypes.c_void_p), ("beta_stride", _I64x3),
        ("state_in", ctypes.c_void_p), ("state_in_stride", _I64x4),
        ("dout", ctypes.c_void_p), ("dout_stride", _I64x4),
        ("dstate_out", ctypes.c_void_p), ("dstate_out_stride", _I64x4),
        ("dq_part", ctypes.c_void_p),
        ("dk_part", ctypes.c_void_p),
        ("dg_part", ctypes.c_void_p),
        ("dbeta_part", ctypes.c_void_p),
        ("dv", ctypes.c_void_p), ("dv_stride", _I64x4),
        ("dstate_in", ctypes.c_void_p), ("dstate_in_stride", _I64x4),
        ("ckpt", ctypes.c_void_p),
        ("ckpt_floats", ctypes.c_size_t),
        ("dq", ctypes.c_void_p), ("dq_stride", _I64x4),
        ("dk", ctypes.c_void_p), ("dk_stride", _I64x4),
        ("dg", ctypes.c_void_p), ("dg_stride", _I64x4),
        ("dbeta", ctypes.c_void_p), ("dbeta_stride", _I64x3),
    ]


_I64x2 = ctypes.c_int64 * 2


class MlaDecodeArgs(ctypes.Structure):
    """Mirror of ``struct MlaDecodeArgs``."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32), ("L", ctypes.c_int32), ("H", ctypes.c_int32),
        ("KVL", ctypes.c_int32), ("DN", ctypes.c_int32), ("DV", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q_nope", ctypes.c_void_p), ("q_nope_stride", _I64x3),
        ("c_kv", ctypes.c_void_p), ("c_kv_stride", _I64x2),
        ("kv_buf", ctypes.c_void_p), ("kv_buf_stride", _I64x3),
        ("pos", ctypes.c_void_p),
        ("w", ctypes.c_void_p), ("w_stride", _I64x2),
        ("out", ctypes.c_void_p), ("out_stride", _I64x3),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class KdaLibraryError(RuntimeError):
    """The CUDA library is missing or unusable (there is no fallback path)."""


_lock = threading.Lock()
_lib = None


def _declare(lib):
    P = ctypes.POINTER(KdaArgs)
    lib.kda_chunkwise_fwd.argtypes = [P, ctypes.c_void_p]
    lib.kda_chunkwise_fwd.restype = ctypes.c_int
    lib.kda_chunkwise_fwd_noalloc.argtypes = [P, ctypes.c_void_p]
    lib.kda_chunkwise_fwd_noalloc.restype = ctypes.c_int
    lib.kda_recurrent_fwd.argtypes = [P, ctypes.c_void_p]
    lib.kda_recurrent_fwd.restype = ctypes.c_int
    lib.kda_chunkwise_workspace_bytes.argtypes = [P]
    lib.kda_chunkwise_workspace_bytes.restype = ctypes.c_size_t
    lib.kda_chunkwise_path.argtypes = [P]
    lib.kda_chunkwise_path.restype = ctypes.c_int
    lib.kda_status_string.argtypes = [ctypes.c_int]
    lib.kda_status_string.restype = ctypes.c_char_p
    lib.kda_device_supported.argtypes = [ctypes.c_int]
    lib.kda_device_supported.restype = ctypes.c_int
    lib.kda_device_error.argtypes = [ctypes.c_int]
    lib.kda_device_error.restype = ctypes.c_int
    lib.kda_prologue_fwd.argtypes = [ctypes.POINTER(KdaPrologueArgs), ctypes.c_void_p]
    lib.kda_prologue_fwd.restype = ctypes.c_int
    lib.kda_epilogue_fwd.argtypes = [ctypes.POINTER(KdaEpilogueArgs), ctypes.c_void_p]
    lib.kda_epilogue_fwd.restype = ctypes.c_int
    lib.mla_decode_fwd.argtypes = [ctypes.POINTER(MlaDecodeArgs), ctypes.c_void_p]
    lib.mla_decode_fwd.restype = ctypes.c_int
    lib.mla_decode_workspace_bytes.argtypes = [ctypes.POINTER(MlaDecodeArgs)]
    lib.mla_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.mla_decode_args_size.argtypes = []
    lib.mla_decode_args_size.restype = ctypes.c_size_t
    lib.kda_backward.argtypes = [ctypes.POINTER(KdaBackwardArgs), ctypes.c_void_p]
    lib.kda_backward.restype = ctypes.c_int
    lib.kda_backward_ckpt_floats.argtypes = [ctypes.c_int] * 5
    lib.kda_backward_ckpt_floats.restype = ctypes.c_size_t
    lib.kda_backward_args_size.argtypes = []
    lib.kda_backward_args_size.restype = ctypes.c_size_t
    lib.kda_prologue_args_size.argtypes = []
    lib.kda_prologue_args_size.restype = ctypes.c_size_t
    lib.kda_epilogue_args_size.argtypes = []
    lib.kda_epilogue_args_size.restype = ctypes.c_size_t
    lib.kda_args_size.argtypes = []
    lib.kda_args_size.restype = ctypes.c_size_t
    lib.kda_abi_version.argtypes = []
    lib.kda_abi_version.restype = ctypes.c_int


def load(path: str | None = None):
    """Load (once) and return the ctypes library handle."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise KdaLibraryError(
                f"{p} is missing: build it with __graft_entry__.build() or "
                f"'python -m kimi_linear_b200.build' (nvcc, sm_100a)")
        try:
            lib = ctypes.CDLL(p)
        except OSError as exc:  # pragma: no cover - depends on the host
            raise KdaLibraryError(f"cannot load {p}: {exc}") from exc
        missing = [s for s in EXPORTED if not hasattr(lib, s)]
        if missing:
            raise KdaLibraryError(f"{p} lacks symbols {missing}")
        _declare(lib)
        if lib.kda_abi_version() != ABI_VERSION:
            raise KdaLibraryError(f"{p}: ABI version {lib.kda_abi_version()} != {ABI_VERSION}")
        for fn, st in (("kda_prologue_args_size", KdaPrologueArgs),
                       ("kda_epilogue_args_size", KdaEpilogueArgs),
                       ("kda_backward_args_size", KdaBackwardArgs),
                       ("mla_decode_args_size", MlaDecodeArgs)):
            if getattr(lib, fn)() != ctypes.sizeof(st):
                raise KdaLibraryError(f"{p}: {fn}() != ctypes sizeof {ctypes.sizeof(st)}")
        if lib.kda_args_size() != ctypes.sizeof(KdaArgs):
            raise KdaLibraryError(
                f"{p}: sizeof(KdaArgs) {lib.kda_args_size()} != ctypes {ctypes.sizeof(KdaArgs)}")
        if path is None:
            _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().kda_status_string(int(code)).decode()
