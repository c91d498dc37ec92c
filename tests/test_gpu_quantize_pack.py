"""fused_quantize_pack_int4 (the standalone quantise + pack drop-in) on the
GPU: bit-exact packed bytes and scales against the oracle restatement of the
reference's quantize_int4_groupwise + pack_int4, for the reference test's
head dims (tests/test_correctness.py:461-589 uses 64, 128, 256), on normal
data with outliers, the golden quantiser edge rows (exact .5 ties, zeros,
subnormals, fp16 max) and every finite fp16 amax; plus its argument errors."""
import numpy as np
import pytest
import torch

import cases
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _run(x_np):
    from iris_kernel.fused_kv import fused_quantize_pack_int4

    x = torch.from_numpy(np.ascontiguousarray(x_np)).cuda()
    T, H, D = x.shape
    packed = torch.full((T, H, D // 2), 0xAB, dtype=torch.uint8, device="cuda")
    scales = torch.full((T, H, D // 32), float("nan"), dtype=torch.float16, device="cuda")
    fused_quantize_pack_int4(x, packed, scales)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy()


def _oracle(x_np):
    q, s = orc.quantize_int4_groupwise(x_np, 32)
    return orc.pack_int4(q), s


@pytest.mark.parametrize("head_dim", [64, 128, 256, 512])
def test_random_with_outliers_bit_exact(head_dim):
    rng = np.random.default_rng(3407 + head_dim)
    x = rng.standard_normal((37, 4, head_dim)).astype(np.float16)
    x[rng.random(x.shape) < 0.01] *= np.float16(20)
    p, s = _run(x)
    pr, sr = _oracle(x)
    assert np.array_equal(p, pr)
    assert np.array_equal(s.view(np.uint16), sr.view(np.uint16))


def test_reference_case_shape():
    """The reference test's own shape: 7 tokens x 4 heads."""
    for head_dim in (64, 128, 256):
        x = np.random.default_rng(3407).standard_normal((7, 4, head_dim)).astype(np.float16)
        p, s = _run(x)
        pr, sr = _oracle(x)
        assert np.array_equal(p, pr) and np.array_equal(s.view(np.uint16), sr.view(np.uint16))


def test_golden_edge_groups(golden):
    x = cases.quant_edge_groups()  # [rows, 32]: ties, zeros, subnormals, fp16 max
    rows = x.shape[0] - x.shape[0] % 2
    x3 = x[:rows].reshape(rows // 2, 1, 64)
    p, s = _run(x3)
    assert np.array_equal(p.reshape(rows, 16), golden["quant_edge.out.packed"][:rows].reshape(rows, 16))
    assert np.array_equal(s.reshape(rows).view(np.uint16),
                          golden["quant_edge.out.scale"][:rows].reshape(rows).view(np.uint16))


def test_every_finite_amax(golden):
    tab = cases.fp16_amax_table_input()[:0x7C00]  # one group per finite non-negative fp16 amax
    n = tab.shape[0] - tab.shape[0] % 2
    p, s = _run(tab[:n].reshape(n // 2, 1, 64))
    assert np.array_equal(s.reshape(n).view(np.uint16), golden["amax_table.out.scale"][:n].view(np.uint16))
    assert np.array_equal(p.reshape(n, 16)[:, 0], golden["amax_table.out.byte0"][:n])


def test_argument_errors():
    from iris_kernel.fused_kv import fused_quantize_pack_int4

    x = torch.zeros(2, 2, 64, dtype=torch.float16, device="cuda")
    p = torch.empty(2, 2, 32, dtype=torch.uint8, device="cuda")
    s = torch.empty(2, 2, 2, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        fused_quantize_pack_int4(x.cpu(), p, s)
    with pytest.raises(TypeError):
        fused_quantize_pack_int4(x.float(), p, s)
    with pytest.raises(NotImplementedError):
        fused_quantize_pack_int4(torch.zeros(2, 2, 96, dtype=torch.float16, device="cuda"),
                                 torch.empty(2, 2, 48, dtype=torch.uint8, device="cuda"),
                                 torch.empty(2, 2, 3, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        fused_quantize_pack_int4(x, p[:, :, :16], s)
    with pytest.raises(TypeError):
        fused_quantize_pack_int4(x, p.to(torch.int8), s)
