"""B200-native (sm_100a) INT4 paged KV-cache kernels.

Drop-in for Hunter2030ZeRo/Iris-Kernel's two hot paths:

* ``iris_kernel.fused_kv.fused_rope_int4_paged_append``       (write)
* ``iris_kernel.fused_attention.fused_int4_paged_decode_attention`` (read)

Both call hand-written CUDA kernels through the C ABI of
``include/iris_b200.h`` (``libiris_b200.so``, loaded by ctypes).  There is no
CPU fallback: importing the package fails if the library is missing.

The reference's package also holds its eager PyTorch modules
(``iris_kernel.torch_eager_kv``, ``iris_kernel.torch_eager_attention``),
which code written against it imports next to the fused ones.  This package
does not reimplement them.  When the reference's own ``iris_kernel``
directory is importable (a directory on ``sys.path`` holding
``iris_kernel/torch_eager_kv.py``, such as the reference's ``src/`` or an
install of it), that directory is appended to this package's ``__path__``:
``iris_kernel.fused_*`` resolve here first, and module names this package
lacks resolve to the reference's files, unmodified.
"""
import os as _os
import sys as _sys


def _reference_dirs():
    here = _os.path.dirname(_os.path.abspath(__file__))
    seen = set()
    for entry in _sys.path:
        cand = _os.path.abspath(_os.path.join(entry or _os.getcwd(), "iris_kernel"))
        if cand == here or cand in seen:
            continue
        seen.add(cand)
        if _os.path.isfile(_os.path.join(cand, "torch_eager_kv.py")):
            yield cand


for _d in _reference_dirs():
    if _d not in __path__:
        __path__.append(_d)

from . import _lib  # noqa: E402,F401  (fails loudly if the shared library is absent)
from ._runtime import check_errors, set_validation_mode, validation_mode  # noqa: E402,F401

__all__ = ["check_errors", "set_validation_mode", "validation_mode"]
