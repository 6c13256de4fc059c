"""Stand-in for the name ``minispeed`` when the reference's own test files
run against this engine (``tests/test_gpu_reference_suite.py``).

Put this directory first on ``PYTHONPATH``.  Importing ``minispeed`` then
runs this file, which hands the name (and every submodule name the
reference's tests import) to ``minispeed_b200`` through
``minispeed_b200.alias``; the import statement returns the aliased package.
Child processes started with ``spawn`` inherit ``PYTHONPATH`` and so resolve
``minispeed`` the same way.
"""

import sys

# alias.install() refuses a foreign module under the name; this file's own
# half-initialised module is removed first, and CPython's import machinery
# returns whatever sys.modules holds under the name once this file has run
del sys.modules[__name__]
import minispeed_b200.alias  # noqa: E402,F401
