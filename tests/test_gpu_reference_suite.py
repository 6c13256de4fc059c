"""The reference's own test files, unmodified, run against this engine on
a GPU (``import minispeed`` resolves to ``minispeed_b200`` through
``tests/reference_shim``).

The reference checkout is looked up in ``$MINISPEED_REFERENCE_SRC`` or
``baseline/_ref`` (the offline install of the reference, next to which its
``tests/`` folder is copied at install time); the test skips when neither
holds the reference's ``tests/test_gpu.py``.  ``tests/test_gpu.py`` covers
fp16 training on one GPU, a forced inf that must skip the step, two NCCL
ranks (with two GPUs) and two gloo ranks sharing one GPU at stages 0-3 in
fp32 and fp16 (reference ``tests/test_gpu.py:1-231``); the CPU files run too.
"""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "tests", "reference_shim")


def _reference_src():
    for cand in (os.environ.get("MINISPEED_REFERENCE_SRC"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isfile(os.path.join(cand, "tests", "test_gpu.py")):
            return cand
    return None


@pytest.mark.timeout(900)
def test_reference_suite_through_alias(tmp_path):
    src = _reference_src()
    if src is None:
        pytest.skip("the reference's tests/ folder is not installed next to baseline/_ref")
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MINISPEED_DEVICE",
                        "MINISPEED_BACKEND")}
    env["PYTHONPATH"] = os.pathsep.join([SHIM, src, ROOT])
    code = ("import sys, minispeed, minispeed_b200; "
            "assert minispeed is minispeed_b200, 'alias not in effect'; "
            "import pytest; sys.exit(pytest.main(sys.argv[1:]))")
    r = subprocess.run([sys.executable, "-c", code, "-q", "-p", "no:cacheprovider",
                        "-c", os.devnull, "--rootdir", src, "--import-mode=append",
                        os.path.join(src, "tests")],
                       cwd=str(tmp_path), env=env, capture_output=True, text=True, timeout=850)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    summary = [ln for ln in r.stdout.splitlines() if " passed" in ln]
    assert summary and " failed" not in summary[-1], tail
    print(summary[-1])
