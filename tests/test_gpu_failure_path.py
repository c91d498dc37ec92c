"""Failure detection without a GPU fault: a kernel's bounded wait on a
barrier phase that nothing completes gives up after a short limit, records
IRIS_ERR_PIPELINE_TIMEOUT in the caller's error word and returns; the wrapper
maps it to the documented exception, and the context stays usable."""
import time

import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_records_the_bit_and_leaves_the_context_usable():
    import iris_kernel
    from iris_kernel import _lib, _runtime
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    assert _lib.lib.iris_b200_selftest_bounded_wait(err.data_ptr(), 20_000_000, stream) == 0  # 20 ms
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(err.item()) == _lib.ERR_PIPELINE_TIMEOUT
    assert 0.015 < elapsed < 5.0  # it waited for its limit, then returned
    with pytest.raises(RuntimeError, match="timed out"):
        _runtime.raise_for_bits(int(err.item()))
    # invalid limits are refused before any launch
    assert _lib.lib.iris_b200_selftest_bounded_wait(err.data_ptr(), 0, stream) == 1  # IRIS_EINVAL
    assert _lib.lib.iris_b200_selftest_bounded_wait(err.data_ptr(), 3_000_000_000, stream) == 1
    # the device and the library still work
    c = cases.decode_random(seed=5, B=2, Hq=8, Hkv=2, D=128, lens=[700, 33])
    t = to_dev(c, cases.DECODE_KEYS)
    out = fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS])
    torch.cuda.synchronize()
    assert_decode_close(out, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))
    iris_kernel.check_errors()
