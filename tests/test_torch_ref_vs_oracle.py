"""The PyTorch FP32 decode reference used for the large GPU parity cases
agrees with the numpy oracle (itself pinned to the reference).  CPU only."""
import numpy as np
import pytest
import torch

import cases
from _refs import to_dev, torch_decode_fp32
from oracle import iris_oracle as orc


@pytest.mark.parametrize("name", sorted(cases.DECODE_SPECS))
def test_torch_reference_matches_oracle(name):
    c = cases.decode_random(**cases.DECODE_SPECS[name])
    ref = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    t = to_dev(c, cases.DECODE_KEYS, device="cpu")
    got = torch_decode_fp32(*[t[k] for k in cases.DECODE_KEYS]).numpy()
    np.testing.assert_allclose(got, ref, atol=2e-5, rtol=1e-5)
