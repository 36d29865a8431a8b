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
_COUNTED = None
_EXT_ERR: Exception | None = None


def _load():
    global _EXT, _EXT_ERR
    if _EXT is not None or _EXT_ERR is not None:
        return
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _EXT = importlib.import_module("zeroq_b200._C")
        global _COUNTED
        _COUNTED = _Counted(_EXT)
    except Exception as e:  # pragma: no cover - depends on the build
        _EXT_ERR = e


def available() -> bool:
    _load()
    return _EXT is not None


# kernels launched per call of each binding (bindings not listed launch one)
_KERNELS_PER_CALL = {"attn_bwd_tc": 3, "gemm_status": 0, "set_gemm_pair_mode": 0,
                     "peer_alloc": 0, "peer_handle": 0, "peer_open": 0, "peer_close": 0,
                     "peer_free": 0, "tensor_from_ptr": 0, "peer_status_read": 0,
                     "peer_flag_words": 0}


class LaunchCounter:
    """Counts this extension's kernel launches while active (``with LaunchCounter() as c``)."""

    active = None

    def __init__(self):
        self.count = 0
        self.by_name = {}

    def __enter__(self):
        LaunchCounter.active = self
        return self

    def __exit__(self, *exc):
        LaunchCounter.active = None
        return False


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        k = _KERNELS_PER_CALL.get(name, 1)

        def call(*args, **kwargs):
            c = LaunchCounter.active
            if c is not None:
                c.count += k
                c.by_name[name] = c.by_name.get(name, 0) + k
            return fn(*args, **kwargs)

        return call


def ext():
    """Return the native module or raise a clear error."""
    _load()
    if _EXT is None:
        raise RuntimeError(
            "zeroq_b200 native extension (zeroq_b200._C) is not built or failed to load: "
            f"{_EXT_ERR!r}. Build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "or `python setup.py build_ext --inplace`."
        )
    return _COUNTED if LaunchCounter.active is not None else _EXT


def so_path() -> str | None:
    _load()
    if _EXT is None:
        return None
    return os.path.abspath(_EXT.__file__)
