"""Loader for the in-tree sm_100a extension ``minispeed_b200._C``.

The extension is built in place by ``python setup.py build_ext --inplace``
(or ``__graft_entry__.build()``).  CUDA tensors always go through it: if it
cannot be imported on a machine with a GPU, :func:`get` raises instead of
silently falling back to PyTorch ops.

``MSB_DEBUG_BUILD=1`` loads the bounds-checked variant
``minispeed_b200._C_debug`` instead (built with ``MSB_DEBUG_BUILD=1 python
setup.py build_ext --inplace``): every kernel index the checks cover (token
ids, cross-entropy targets, TMA coordinates, GEMM workspace slots, tile
counters and column-sum partials) is tested on the device; a failure is
recorded and its access skipped, never trapped.  :func:`check_bounds` reads
the records and raises :class:`BoundsError`; the engine calls it after every
step when this build is loaded.
"""

from __future__ import annotations

import importlib
import os

_mod = None
_err: Exception | None = None

# site codes of BoundsSite (csrc/kernels_api.h)
BOUNDS_SITES = {
    1: "embedding token id outside [0, vocab)",
    2: "cross-entropy target outside [0, V)",
    3: "TMA load x coordinate not 16-byte aligned",
    4: "TMA store at a negative or unaligned coordinate",
    5: "GEMM partial beyond the workspace",
    6: "GEMM tile counter beyond the counter array",
    7: "GEMM column-sum partial beyond its buffer",
}


class BoundsError(RuntimeError):
    """A bounds check of the debug build failed on the device."""


def module_name() -> str:
    return "minispeed_b200._C_debug" if os.environ.get("MSB_DEBUG_BUILD") == "1" \
        else "minispeed_b200._C"


def load():
    global _mod, _err
    if _mod is None and _err is None:
        import torch  # noqa: F401  (loads libc10/libtorch for the extension)

        try:
            _mod = importlib.import_module(module_name())
        except Exception as e:  # pragma: no cover - depends on the build
            _err = e
    if _mod is None:
        flag = "MSB_DEBUG_BUILD=1 " if module_name().endswith("_debug") else ""
        raise RuntimeError(
            f"{module_name()} is not built or failed to load "
            f"({_err!r}); run `{flag}python setup.py build_ext --inplace`") from _err
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


def debug_build() -> bool:
    """True when the loaded extension is the bounds-checked build."""
    return available() and bool(load().bounds_check_build())


def bounds_status(reset: bool = True, mod=None) -> list:
    """The device's bounds records after the queued work has finished: one
    dict per translation unit with checks (all counts zero in the release
    build).  ``mod`` reads another loaded build of the extension."""
    import torch

    m = mod if mod is not None else load()
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    return [{"unit": unit, "count": count, "site": site,
             "what": BOUNDS_SITES.get(site, "none"), "index": index, "limit": limit}
            for unit, count, site, index, limit in m.bounds_status(reset)]


def check_bounds(mod=None) -> None:
    """Raise :class:`BoundsError` naming the first failed check of each
    unit, if any failed since the last read (the records are then reset)."""
    bad = [r for r in bounds_status(True, mod) if r["count"]]
    if bad:
        raise BoundsError("; ".join(
            f"{r['unit']}: {r['count']} failed check(s), first: {r['what']} "
            f"(index {r['index']}, limit {r['limit']})" for r in bad))
