"""Loader for the compiled sm_100a extension ``zeroq_b200._C``.

The extension is built in-tree by ``__graft_entry__.build()`` (or
``python setup.py build_ext --inplace``).  Policy:

* CPU tensors always take the PyTorch reference path (the numerics oracle).
* CUDA tensors always take the native path.  If the extension is missing on a
  machine that has a GPU, ``ext()`` raises instead of silently falling back, so a
  GPU run can never pass on an eager PyTorch stand-in.
"""

from __future__ import annotations

import importlib
import os

_EXT = None
_EXT_ERR: Exception | None = None


def _load():
    global _EXT, _EXT_ERR
    if _EXT is not None or _EXT_ERR is not None:
        return
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _EXT = importlib.import_module("zeroq_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _EXT_ERR = e


def available() -> bool:
    _load()
    return _EXT is not None


def ext():
    """Return the native module or raise a clear error."""
    _load()
    if _EXT is None:
        raise RuntimeError(
            "zeroq_b200 native extension (zeroq_b200._C) is not built or failed to load: "
            f"{_EXT_ERR!r}. Build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "or `python setup.py build_ext --inplace`."
        )
    return _EXT


def so_path() -> str | None:
    _load()
    if _EXT is None:
        return None
    return os.path.abspath(_EXT.__file__)
