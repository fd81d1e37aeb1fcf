"""B200-native (sm_100a) Kimi Delta Attention core.

Drop-in replacement for the two kernels of Lazy-Hakimi/-kimi-linear-:
``kimi_linear.kda.kda_chunkwise`` (``kimi_linear/kda.py:58-185``) and
``kimi_linear.kda.kda_recurrent`` (``kimi_linear/kda.py:188-219``), backed by
hand-written CUDA kernels behind the C ABI of ``include/kda_b200.h``.

The directory name is not a Python identifier, so import it with
``importlib.import_module("-kimi-linear-_b200")``; the package then also
registers itself (and its submodules) as ``kimi_linear_b200``.

To route an existing ``kimi_linear`` model through these kernels::

    import importlib
    kb = importlib.import_module("-kimi-linear-_b200")
    kb.install()            # patches kimi_linear.kda.* and the package re-exports

``KimiDeltaAttention.forward`` looks the two functions up as module globals at
call time (``kda.py:503,519,526``), so prefill, eager decode and
``GraphedDecoder`` all take the new path without further changes.

Also here: the fused prologue / epilogue of the KDA block (``fused``), the
gradient of the core (autograd through both functions) and the static-buffer
MLA decode step of the full-attention layers (``mla.install_mla()``).
"""

from __future__ import annotations

import sys as _sys

from . import _lib, fused, mla, ops, sharding, synth
from ._lib import KdaLibraryError
from .fused import kda_epilogue, kda_prologue
from .ops import KdaError, chunkwise_impl, chunkwise_path, device_error, kda_chunkwise, kda_recurrent

ALIAS = "kimi_linear_b200"
if __name__ != ALIAS:
    _sys.modules.setdefault(ALIAS, _sys.modules[__name__])
    for _sub in ("_lib", "fused", "mla", "ops", "sharding", "synth"):
        _sys.modules.setdefault(f"{ALIAS}.{_sub}", _sys.modules[f"{__name__}.{_sub}"])

__all__ = ["kda_chunkwise", "kda_recurrent", "chunkwise_path", "chunkwise_impl", "device_error",
           "kda_chunkwise_inplace", "kda_recurrent_inplace",
           "kda_prologue", "kda_epilogue",
           "install", "uninstall",
           "KdaError", "KdaLibraryError", "load_library"]


def load_library():
    """Load ``libkda_b200.so`` now (raises :class:`KdaLibraryError` if absent)."""
    return _lib.load()


_saved = []


def kda_chunkwise_inplace(q, k, v, g, beta, initial_state=None, chunk_size=64, tile_size=0,
                          state_dtype=None):
    """``kda_chunkwise`` that updates ``initial_state`` in place (when given)."""
    return kda_chunkwise(q, k, v, g, beta, initial_state, chunk_size, tile_size, state_dtype,
                         inplace=True)


def kda_recurrent_inplace(q, k, v, g, beta, state=None, state_dtype=None):
    """``kda_recurrent`` that updates ``state`` in place (when given)."""
    return kda_recurrent(q, k, v, g, beta, state, state_dtype, inplace=True)


def install(kda_module=None, package=None, inplace_state=False):
    """Point the reference's KDA kernels at this package.

    Replaces ``kda_chunkwise`` / ``kda_recurrent`` in ``kimi_linear.kda`` (or the
    module object ``kda_module``) and in the ``kimi_linear`` package namespace,
    which re-exports them by value (``kimi_linear/__init__.py:9``).  Loads the
    CUDA library first, so a missing build fails here rather than mid-model.
    Returns the list of patched ``(module, name)`` pairs; :func:`uninstall`
    restores the originals.

    ``inplace_state=True`` installs the in-place variants: the recurrent state
    passed in is overwritten with the new one (the reference returns a fresh
    tensor and leaves the old one intact, ``kda.py:137,205``).  The model's
    own cache handling replaces the old state with the returned one, so
    decoding is unchanged, and ``GraphedDecoder``'s copy-back of each KDA
    state (``graph_decode.py:262``) turns into a copy onto itself; only code
    that keeps its own reference to an old state sees the difference.
    """
    import importlib

    _lib.load()
    if kda_module is None:
        kda_module = importlib.import_module("kimi_linear.kda")
    if package is None:
        pkg_name = kda_module.__name__.rpartition(".")[0]
        package = _sys.modules.get(pkg_name) if pkg_name else None
    patched = []
    for mod in (kda_module, package):
        if mod is None:
            continue
        chunk_fn, rec_fn = ((kda_chunkwise_inplace, kda_recurrent_inplace) if inplace_state
                            else (kda_chunkwise, kda_recurrent))
        for name, fn in (("kda_chunkwise", chunk_fn), ("kda_recurrent", rec_fn)):
            if hasattr(mod, name) and getattr(mod, name) is not fn:
                _saved.append((mod, name, getattr(mod, name)))
                setattr(mod, name, fn)
                patched.append((mod.__name__, name))
    return patched


def uninstall():
    """Undo every :func:`install` (most recent first)."""
    while _saved:
        mod, name, fn = _saved.pop()
        setattr(mod, name, fn)
