"""Loader for the in-tree sm_100a extension ``minispeed_b200._C``.

The extension is built in place by ``python setup.py build_ext --inplace``
(or ``__graft_entry__.build()``).  CUDA tensors always go through it: if it
cannot be imported on a machine with a GPU, :func:`get` raises instead of
silently falling back to PyTorch ops.
"""

from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None


def load():
    global _mod, _err
    if _mod is None and _err is None:
        import torch  # noqa: F401  (loads libc10/libtorch for the extension)

        try:
            _mod = importlib.import_module("minispeed_b200._C")
        except Exception as e:  # pragma: no cover - depends on the build
            _err = e
    if _mod is None:
        raise RuntimeError(
            "minispeed_b200._C is not built or failed to load "
            f"({_err!r}); run `python setup.py build_ext --inplace`") from _err
    return _mod


def get():
    return load()


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def launch_count() -> int:
    """Kernels this library has launched in this process so far."""
    return int(load().launch_count()) if available() else 0
