"""The reference's own test modules run unchanged against the drop-in (CPU
part).

``oracle/install_reference.py`` installs the unmodified reference into
``baseline/_ref`` and copies its ``tests/test_correctness.py`` and
``tests/test_attention.py`` beside it.  With ``iris-kernel_b200`` first on
``sys.path`` and the install after it, ``iris_kernel.fused_*`` must resolve to
this package and ``iris_kernel.torch_eager_*`` to the reference's own files
(the package extends its ``__path__`` with the reference's directory), so the
reference's import lines work as written.  Skipped when the install is
absent.  The GPU half (the reference's CUDA tests against the drop-in's
kernels) is ``test_gpu_reference_suite.py``."""
import ast
import os
import subprocess
import sys

import pytest

from conftest import PKG, ROOT

REF = os.path.join(ROOT, "baseline", "_ref")
REF_TESTS = os.path.join(REF, "reference_tests")

pytestmark = pytest.mark.skipif(not os.path.isfile(os.path.join(REF_TESTS, "test_attention.py")),
                                reason="reference not installed (python oracle/install_reference.py <checkout>)")


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([PKG, REF])
    return env


def _import_lines():
    lines = []
    for name in ("test_correctness.py", "test_attention.py"):
        tree = ast.parse(open(os.path.join(REF_TESTS, name)).read())
        for node in tree.body:
            if isinstance(node, ast.ImportFrom) and node.module and node.module.startswith("iris_kernel"):
                lines.append(ast.unparse(node))
    return lines


def test_reference_test_imports_resolve_to_dropin_and_reference_eager():
    lines = _import_lines()
    assert any("fused_kv" in ln for ln in lines) and any("torch_eager_attention" in ln for ln in lines)
    prog = "\n".join(lines + [
        "import iris_kernel.fused_kv as a, iris_kernel.fused_attention as b",
        "import iris_kernel.torch_eager_kv as c, iris_kernel.torch_eager_attention as d",
        "print(a.__file__); print(b.__file__); print(c.__file__); print(d.__file__)",
    ])
    out = subprocess.run([sys.executable, "-c", prog], cwd="/", env=_env(), capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    files = out.stdout.split()
    assert files[0].startswith(PKG) and files[1].startswith(PKG)  # the drop-in's fused modules
    assert files[2].startswith(REF) and files[3].startswith(REF)  # the reference's eager modules


def test_reference_suite_cpu_tests_pass_against_dropin():
    out = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", REF_TESTS],
                         cwd="/", env=_env(), capture_output=True, text=True, timeout=900)
    tail = out.stdout[-3000:]
    assert out.returncode == 0, tail + out.stderr[-2000:]
    assert " failed" not in tail and "error" not in tail.lower()
    assert "10 passed" in tail  # the CPU tests; the 7 CUDA tests skip without a GPU
