"""The write path's division-free quantiser against the reference's IEEE
arithmetic over its whole finite domain (GPU).

The append computes scale = fp16(max(amax / 7, 2^-14)) and q = rint(x /
scale) without a divide instruction (a Markstein-corrected reciprocal and a
round-half-even magic add).  The reference divides (torch_eager_kv.py:77-86).
``iris_b200_selftest_quantizer_sweep`` runs both forms for every
non-negative finite fp16 absmax (31,744 values) and, for each, every fp16 x
with |x| <= absmax (both signs), about 1.0e9 (x, scale) pairs; every packed
word and every scale must agree."""
import pytest
import torch

pytestmark = pytest.mark.gpu

FINITE = 0x7C00  # non-negative finite fp16 bit patterns: 0x0000 .. 0x7BFF


def _sweep(lo, hi):
    from iris_kernel import _lib

    counts = torch.zeros(3, dtype=torch.int64, device="cuda")
    status = _lib.lib.iris_b200_selftest_quantizer_sweep(lo, hi, counts.data_ptr(),
                                                         torch.cuda.current_stream().cuda_stream)
    assert status == 0
    torch.cuda.synchronize()
    return [int(x) for x in counts.cpu()]


def _words(lo, hi):
    # 8 magnitudes per word, magnitudes 0..amax, two signs
    return sum(2 * (a // 8 + 1) for a in range(lo, hi))


def test_quantizer_matches_ieee_on_every_finite_scale_and_value():
    bad_words, bad_scales, words = _sweep(0, FINITE)
    assert words == _words(0, FINITE)  # every pair was visited
    assert bad_scales == 0
    assert bad_words == 0


def test_partial_range_visits_exactly_its_pairs():
    """A sub-range of absmax values visits exactly its own pairs (the launch
    shape covers every magnitude up to each absmax, nothing past it)."""
    bad_words, bad_scales, words = _sweep(1000, 1010)
    assert words == _words(1000, 1010)
    assert bad_words == 0 and bad_scales == 0
    bad_words, bad_scales, words = _sweep(0x7BF0, FINITE)
    assert words == _words(0x7BF0, FINITE)
    assert bad_words == 0 and bad_scales == 0
