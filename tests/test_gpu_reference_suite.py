"""The reference's own test modules (``tests/test_correctness.py``,
``tests/test_attention.py``, copied unmodified into ``baseline/_ref`` by
``oracle/install_reference.py``) run unchanged against the drop-in on the
GPU: every CUDA test there calls this package's kernels through the
reference's import lines and checks them against the reference's own eager
code.  Skipped when the reference install is absent."""
import os
import subprocess
import sys

import pytest

from conftest import PKG, ROOT

REF = os.path.join(ROOT, "baseline", "_ref")
REF_TESTS = os.path.join(REF, "reference_tests")

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not os.path.isfile(os.path.join(REF_TESTS, "test_attention.py")),
                       reason="reference not installed (python oracle/install_reference.py <checkout>)"),
]


def test_reference_suite_passes_against_dropin_on_gpu():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([PKG, REF])
    out = subprocess.run([sys.executable, "-m", "pytest", "-q", "-rA", "-p", "no:cacheprovider", REF_TESTS],
                         cwd="/", env=env, capture_output=True, text=True, timeout=1200)
    tail = out.stdout[-6000:]
    assert out.returncode == 0, tail + out.stderr[-2000:]
    assert "17 passed" in tail, tail  # 10 CPU + 7 CUDA tests, none skipped
