"""The matched FP16 paged decode (fused_fp16_paged_decode_attention) on the
GPU against the FP32 oracle restatement of the reference's eager FP16 decode
(tolerance max-abs 2e-3 / relative 1e-2, as for the INT4 decode) and the
reference's own fp16 outputs; GQA ratios 1-16, D 64/128, ragged lengths with
NaN/Inf in the slots past each sequence's end, long sequences that straddle
split-KV ranges, argument and data errors."""
import numpy as np
import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _fused(c, **kw):
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

    t = to_dev(c, cases.FP16_DECODE_KEYS)
    out = fused_fp16_paged_decode_attention(*[t[k] for k in cases.FP16_DECODE_KEYS], **kw)
    torch.cuda.synchronize()
    return out


def _oracle(c, **kw):
    return orc.decode_attention_fp16(*[c[k] for k in cases.FP16_DECODE_KEYS], **kw)


@pytest.mark.parametrize("name", sorted(cases.FP16_DECODE_SPECS))
def test_specs_match_oracle_and_reference(golden, name):
    c = cases.decode_random_fp16(**cases.FP16_DECODE_SPECS[name])
    out = _fused(c)
    assert out.dtype == torch.float16
    assert_decode_close(out, _oracle(c))
    assert_decode_close(out, golden[f"fp16_decode.{name}.out.output"].astype(np.float32), atol=3e-3, rtol=1e-2)


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (16, 16, 64), (64, 8, 128), (32, 2, 128), (8, 1, 64)])
def test_geometries_and_long_sequences(hq, hkv, d):
    lens = [5000, 1, 16, 333, 2100]
    c = cases.decode_random_fp16(seed=hq * 7 + hkv + d, B=len(lens), Hq=hq, Hkv=hkv, D=d, lens=lens)
    assert_decode_close(_fused(c), _oracle(c))


def test_softmax_scale_and_output_buffer():
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

    c = cases.decode_random_fp16(seed=5, B=2, Hq=8, Hkv=2, D=128, lens=[100, 40])
    t = to_dev(c, cases.FP16_DECODE_KEYS)
    out = torch.full_like(t["query"], float("nan"))
    ret = fused_fp16_paged_decode_attention(*[t[k] for k in cases.FP16_DECODE_KEYS], out, softmax_scale=0.05)
    torch.cuda.synchronize()
    assert ret is out
    assert_decode_close(out, _oracle(c, softmax_scale=0.05))


def test_errors():
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

    c = cases.decode_random_fp16(seed=6, B=2, Hq=8, Hkv=2, D=64, lens=[20, 40])
    t = to_dev(c, cases.FP16_DECODE_KEYS)
    args = [t[k] for k in cases.FP16_DECODE_KEYS]
    with pytest.raises(TypeError):
        fused_fp16_paged_decode_attention(args[0], args[1].float(), args[2].float(), *args[3:])
    with pytest.raises(ValueError):
        fused_fp16_paged_decode_attention(args[0], args[1], args[2][:, :, :1], *args[3:])
    bad = t["block_table"].clone()
    bad[1, 0] = 10_000
    with pytest.raises(IndexError):
        fused_fp16_paged_decode_attention(*args[:3], bad, args[4])
    lens = t["seq_lens"].clone()
    lens[0] = 0
    with pytest.raises(ValueError):
        fused_fp16_paged_decode_attention(*args[:4], lens)
    # the call after an error works
    assert_decode_close(fused_fp16_paged_decode_attention(*args), _oracle(c))
