"""The C-ABI library loads without a GPU, exports every entry point that
include/iris_b200.h declares, and rejects bad host-side arguments with its
documented status codes before touching CUDA.  CPU only."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "iris_b200.h")


def _declared():
    src = open(HEADER).read()
    return re.findall(r"IRIS_API\s+[\w\s\*]+?\b(iris_b200_\w+)\s*\(", src)


def test_header_declares_entry_points():
    names = _declared()
    assert "iris_b200_rope_int4_paged_append" in names
    assert "iris_b200_int4_paged_decode" in names
    assert len(names) == len(set(names))


def test_python_constants_match_the_header():
    from iris_kernel import _lib

    src = open(HEADER).read()
    consts = dict(re.findall(r"#define (IRIS_\w+) (0x[0-9a-fA-F]+|\d+)\b", src))
    for name, value in consts.items():
        short = name[len("IRIS_"):]
        if hasattr(_lib, short):
            assert getattr(_lib, short) == int(value, 0), name
    assert _lib.APPEND_INLINE_CHECK_TOKENS == int(consts["IRIS_APPEND_INLINE_CHECK_TOKENS"])
    assert _lib.ERR_DUP_SLOT == int(consts["IRIS_ERR_DUP_SLOT"], 0)


def test_library_exports_every_declared_symbol():
    from iris_kernel import _lib

    so = _lib.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (iris_b200_\w+)", out))
    declared = set(_declared())
    assert declared <= exported, declared - exported
    # the ctypes table covers exactly the declared API
    assert set(_lib.SIGNATURES) == declared


def test_host_side_status_codes_without_gpu():
    from iris_kernel import _lib

    lib = _lib.lib
    assert lib.iris_b200_version() >= 100
    assert lib.iris_b200_status_string(2) == b"unsupported shape"
    # head_dim not a multiple of 64 -> unsupported, before any CUDA call
    p = ctypes.c_void_p(16)
    st = lib.iris_b200_rope_int4_paged_append(p, p, p, p, p, p, p, p, p, p, 4, 2, 96, 8, 4, 16, p, None)
    assert st == 2
    # page size other than 16 -> unsupported
    st = lib.iris_b200_int4_paged_decode(p, p, p, p, p, p, 4, p, p, None, 0, 1, 8, 2, 128, 4, 8, 4, 0.1, p, 1 << 20,
                                         p, None)
    assert st == 2
    # Hq not a multiple of Hkv -> invalid
    st = lib.iris_b200_int4_paged_decode(p, p, p, p, p, p, 4, p, p, None, 0, 1, 7, 2, 128, 4, 16, 4, 0.1, p, 1 << 20,
                                         p, None)
    assert st == 1
    # slot bitmap size: one bit per slot
    assert lib.iris_b200_append_check_workspace_bytes(4, 16) == 8
    assert lib.iris_b200_append_check_workspace_bytes(3, 11) == 8
    assert lib.iris_b200_decode_workspace_bytes(64, 32, 8, 128, 0) > 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-CUDA error path")
def test_wrappers_require_cuda_like_the_reference():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    x = torch.zeros(1, 1, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        fused_rope_int4_paged_append(x, x, torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32),
                                     torch.zeros(1, 32, dtype=torch.float16), torch.zeros(1, 32, dtype=torch.float16),
                                     torch.zeros(1, 16, 1, 32, dtype=torch.uint8),
                                     torch.zeros(1, 16, 1, 32, dtype=torch.uint8),
                                     torch.zeros(1, 16, 1, 2, dtype=torch.float16),
                                     torch.zeros(1, 16, 1, 2, dtype=torch.float16), rotary_dim=64, page_size=16)
    with pytest.raises(RuntimeError):
        fused_int4_paged_decode_attention(x, torch.zeros(1, 16, 1, 32, dtype=torch.uint8),
                                          torch.zeros(1, 16, 1, 32, dtype=torch.uint8),
                                          torch.zeros(1, 16, 1, 2, dtype=torch.float16),
                                          torch.zeros(1, 16, 1, 2, dtype=torch.float16),
                                          torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, dtype=torch.int32))
