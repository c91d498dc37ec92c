"""The allocation-free decode entry point, for callers that may not allocate
device memory themselves (plugins handed their tensors by a framework that
owns all device memory, code in allocator or stream callbacks, serving loops
that forbid allocation after start-up): iris_b200_int4_paged_decode_noalloc
keeps its scratch in a static array inside the library.

Called through the C ABI twice in a row on different inputs (the second call
reuses the scratch the first one left), each output must match the regular
entry point's (which gets a workspace from the caller) and the FP32 oracle
within the decode tolerance of the other tests.  Collected last (file name)
so that a run that stops at the first failure has run every other test
first; it also passes alone in a fresh process."""
import numpy as np
import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _args(t, out, err):
    q, kd, vd, ks, vs, bt, lens = (t[k] for k in cases.DECODE_KEYS)
    B, Hq, D = q.shape
    NP, P, Hkv, _ = kd.shape
    head = [q.data_ptr(), kd.data_ptr(), vd.data_ptr(), ks.data_ptr(), vs.data_ptr(), bt.data_ptr(), bt.stride(0),
            lens.data_ptr(), out.data_ptr(), None, 0, B, Hq, Hkv, D, NP, P, bt.shape[1], D ** -0.5]
    return head, err.data_ptr(), torch.cuda.current_stream().cuda_stream


def _regular(lib, t):
    out = torch.empty_like(t["query"])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    q = t["query"]
    ws_bytes = lib.iris_b200_decode_workspace_bytes(q.shape[0], q.shape[1], t["k_data"].shape[2], q.shape[2], 0)
    ws = torch.full((ws_bytes,), 0xA5, dtype=torch.uint8, device="cuda")  # contents do not matter
    head, errp, stream = _args(t, out, err)
    assert lib.iris_b200_int4_paged_decode(*head, ws.data_ptr(), ws.numel(), errp, stream) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def _noalloc(lib, t):
    out = torch.empty_like(t["query"])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    head, errp, stream = _args(t, out, err)
    assert lib.iris_b200_int4_paged_decode_noalloc(*head, errp, stream) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_noalloc_decode_matches_regular_entry_point_twice():
    from iris_kernel import _lib

    lib = _lib.lib
    # long and short sequences, so split-KV records go through the scratch
    first = cases.decode_random(seed=71, B=4, Hq=16, Hkv=4, D=128, lens=[3000, 17, 900, 5000])
    second = cases.decode_random(seed=72, B=3, Hq=8, Hkv=8, D=64, lens=[2500, 40, 1234])
    for c in (first, second):
        t = to_dev(c, cases.DECODE_KEYS)
        got = _noalloc(lib, t)
        ref = _regular(lib, t)
        assert_decode_close(got, ref)
        assert_decode_close(got, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))
    # and once more on the first input after the second call changed the scratch
    t = to_dev(first, cases.DECODE_KEYS)
    got = _noalloc(lib, t)
    assert_decode_close(got, _regular(lib, t))
    assert_decode_close(got, orc.decode_attention(*[first[k] for k in cases.DECODE_KEYS]))


def test_noalloc_serves_small_mqa_problems():
    """The scratch a call needs is sized by its problem (its page count caps
    the split-KV ranges), so a short MQA decode at D=128, whose SM-derived
    worst case exceeds the array, still runs."""
    from iris_kernel import _lib

    lib = _lib.lib
    assert lib.iris_b200_decode_workspace_bytes(1, 16, 1, 128, 0) > _lib.DECODE_NOALLOC_SCRATCH_BYTES
    c = cases.decode_random(seed=74, B=1, Hq=16, Hkv=1, D=128, lens=[64])
    t = to_dev(c, cases.DECODE_KEYS)
    got = _noalloc(lib, t)
    assert_decode_close(got, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))


def test_noalloc_rejects_problems_larger_than_its_scratch():
    from iris_kernel import _lib

    lib = _lib.lib
    # MQA with 16 query heads at D=128 over a block table of 8404 columns may
    # use ~2100 split-KV ranges of 16 KB of records each: more than the array
    c = cases.decode_random(seed=73, B=1, Hq=16, Hkv=1, D=128, lens=[64], extra_cols=8400)
    t = to_dev(c, cases.DECODE_KEYS)
    out = torch.full_like(t["query"], float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    head, errp, stream = _args(t, out, err)
    assert lib.iris_b200_int4_paged_decode_noalloc(*head, errp, stream) == 5  # IRIS_EWORKSPACE
    torch.cuda.synchronize()
    assert bool(torch.isnan(out).all())  # nothing was launched
