"""Run code written for ``minispeed`` on this engine without editing it.

    import minispeed_b200.alias      # before the first ``import minispeed``
    import minispeed as ms           # is now minispeed_b200

Importing this module registers ``minispeed`` and every submodule that user
code or tests of the original package import (``minispeed.precision``,
``minispeed.optim.scheduler``, ``minispeed.flat``, ...; the module list of
``minispeed/__init__.py:23-29`` and the test imports of
``tests/test_precision.py:5-6``, ``tests/test_config.py:3``) as names of
this package's modules.  It refuses when another package named
``minispeed`` is already imported, rather than mixing the two.
"""

from __future__ import annotations

import importlib
import sys

SUBMODULES = (
    "activation_checkpointing", "checkpoint", "comm", "config", "engine", "flat", "optim",
    "optim.adam", "optim.scheduler", "precision", "utils", "zero", "zero.stage_1_and_2",
    "zero.stage_3",
)


def install() -> None:
    """Register ``minispeed`` and its submodules as names of this package."""
    pkg = importlib.import_module("minispeed_b200")
    current = sys.modules.get("minispeed")
    if current is not None and current is not pkg:
        raise RuntimeError(f"another 'minispeed' is already imported ({current!r}); import "
                           "minispeed_b200.alias before it")
    sys.modules["minispeed"] = pkg
    for name in SUBMODULES:
        sys.modules["minispeed." + name] = importlib.import_module("minispeed_b200." + name)


def uninstall() -> None:
    """Drop the aliases (a later ``import minispeed`` finds the real one)."""
    pkg = sys.modules.get("minispeed_b200")
    if sys.modules.get("minispeed") is pkg:
        del sys.modules["minispeed"]
    for name in SUBMODULES:
        mod = sys.modules.get("minispeed." + name)
        if mod is not None and mod is sys.modules.get("minispeed_b200." + name):
            del sys.modules["minispeed." + name]


install()
