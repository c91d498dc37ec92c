"""Install the unmodified reference (Hunter2030ZeRo/Iris-Kernel) into
``baseline/_ref`` for ``bench.py --impl reference`` and the drop-in tests.

    python oracle/install_reference.py <path to the reference checkout> [--force]

TEST / BASELINE INFRASTRUCTURE ONLY: nothing in the ``iris_kernel`` package
imports what this installs.

The stock command is ``pip install --no-index --no-build-isolation
--find-links /opt/wheelhouse --target baseline/_ref <reference>``.  It cannot
run as is in this image: the reference's ``pyproject.toml`` names the
``uv_build`` build backend, which is not in the offline wheelhouse, and its
dependency pins (``torch>=2.13``, ``tilelang>=0.1.13``) are newer than the
installed torch 2.11 / tilelang 0.1.9.  So the recipe

1. copies the reference to a temporary directory (the checkout is
   read-only),
2. replaces only the ``[build-system]`` table of the copy's
   ``pyproject.toml`` with setuptools (installed here), which packs the same
   ``src/iris_kernel`` modules,
3. runs the pip command above on the copy with ``--no-deps``,
4. checks that every installed ``iris_kernel/*.py`` is byte-identical to the
   reference's ``src/iris_kernel/*.py`` (sha256),
5. copies the reference's two test modules (``tests/test_correctness.py``,
   ``tests/test_attention.py``) to ``baseline/_ref/reference_tests/`` so that
   a GPU box, which has no reference checkout, can run them unchanged
   against the drop-in (``tests/test_gpu_reference_suite.py``).

``baseline/_ref`` is git-ignored (not product source) but travels to the GPU
box with the working tree.
"""
from __future__ import annotations

import hashlib
import os
import re
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TARGET = os.path.join(ROOT, "baseline", "_ref")
TESTS = ("test_correctness.py", "test_attention.py")
STAMP = os.path.join(TARGET, "INSTALLED_FROM.txt")

_SETUPTOOLS_BACKEND = '[build-system]\nrequires = ["setuptools"]\nbuild-backend = "setuptools.build_meta"\n'


def _sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def _modules(src_pkg: str) -> list[str]:
    return sorted(f for f in os.listdir(src_pkg) if f.endswith(".py"))


def installed() -> bool:
    """True when ``baseline/_ref`` holds a verified install."""
    return os.path.exists(STAMP) and os.path.isdir(os.path.join(TARGET, "iris_kernel"))


def install(reference: str, force: bool = False, verbose: bool = True) -> str:
    src_pkg = os.path.join(reference, "src", "iris_kernel")
    if not os.path.isdir(src_pkg):
        raise FileNotFoundError(f"{src_pkg} is not a reference checkout")
    if installed() and not force:
        return TARGET
    if os.path.isdir(TARGET):
        shutil.rmtree(TARGET)
    with tempfile.TemporaryDirectory(prefix="iris_ref_") as tmp:
        copy = os.path.join(tmp, "reference")
        shutil.copytree(reference, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        pyproject = os.path.join(copy, "pyproject.toml")
        os.chmod(copy, 0o755)
        os.chmod(pyproject, 0o644)
        with open(pyproject) as f:
            text = f.read()
        text, n = re.subn(r"\[build-system\][^\[]*", _SETUPTOOLS_BACKEND + "\n", text, flags=re.S)
        if n != 1:
            raise RuntimeError("reference pyproject.toml has no [build-system] table")
        with open(pyproject, "w") as f:
            f.write(text)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", TARGET, copy]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"pip install of the reference failed:\n{res.stdout[-2000:]}\n{res.stderr[-2000:]}")
    dst_pkg = os.path.join(TARGET, "iris_kernel")
    for name in _modules(src_pkg):
        a, b = os.path.join(src_pkg, name), os.path.join(dst_pkg, name)
        if not os.path.exists(b) or _sha(a) != _sha(b):
            raise RuntimeError(f"installed {name} differs from the reference's source")
    tdir = os.path.join(TARGET, "reference_tests")
    os.makedirs(tdir, exist_ok=True)
    for name in TESTS:
        shutil.copyfile(os.path.join(reference, "tests", name), os.path.join(tdir, name))
    with open(STAMP, "w") as f:
        f.write("reference modules (sha256, byte-identical to src/iris_kernel):\n")
        for name in _modules(src_pkg):
            f.write(f"{name} {_sha(os.path.join(dst_pkg, name))}\n")
    if verbose:
        print(f"installed the reference into {TARGET}")
    return TARGET


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        sys.exit("usage: python oracle/install_reference.py <reference checkout> [--force]")
    install(args[0], force="--force" in sys.argv)
