"""B200-native (sm_100a) INT4 paged KV-cache kernels.

Drop-in for Hunter2030ZeRo/Iris-Kernel's two hot paths:

* ``iris_kernel.fused_kv.fused_rope_int4_paged_append``       (write)
* ``iris_kernel.fused_attention.fused_int4_paged_decode_attention`` (read)

Both call hand-written CUDA kernels through the C ABI of
``include/iris_b200.h`` (``libiris_b200.so``, loaded by ctypes).  There is no
CPU fallback: importing the package fails if the library is missing.
"""
from . import _lib  # noqa: F401  (fails loudly if the shared library is absent)
from ._runtime import check_errors, set_validation_mode, validation_mode  # noqa: F401

__all__ = ["check_errors", "set_validation_mode", "validation_mode"]
