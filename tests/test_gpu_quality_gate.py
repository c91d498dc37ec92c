"""The reference's INT4 quality gate on the fused kernels (GPU).

Reference: tests/test_attention.py:199-232 requires the INT4 decode to track
the matched FP16 decode over the same keys and values: mean cosine
similarity > 0.97 and RMSE < 0.20.  Here both sides are this package's fused
kernels: the same K/V is written once by the fused RoPE+INT4 append and once
by the fused FP16 append, and the fused INT4 and FP16 decodes read them.
Cases: the reference fixture's shape and BASELINE config 1."""
import numpy as np
import pytest
import torch

import cases
from _refs import to_dev

pytestmark = pytest.mark.gpu


def _gate(int4_out, fp16_out):
    a = int4_out.float().flatten(0, 1)
    b = fp16_out.float().flatten(0, 1)
    cosine = float(torch.nn.functional.cosine_similarity(a, b, dim=-1).mean())
    rmse = float(torch.mean((a - b) ** 2).sqrt())
    return cosine, rmse


@pytest.mark.parametrize("make", [cases.attention_ref_case, cases.config1], ids=["reference_fixture", "config1"])
def test_fused_int4_decode_tracks_fused_fp16_decode(make):
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention, fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_fp16_append, fused_rope_int4_paged_append

    c = make()
    t = to_dev(c, cases.APPEND_KEYS + ("query", "block_table", "seq_lens"))
    D = t["query"].shape[2]
    NP, P, Hkv, _ = t["k_data"].shape
    fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=D, page_size=P)
    kc = torch.zeros(NP, P, Hkv, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    fused_rope_fp16_append(t["key"], t["value"], t["positions"], t["slot_mapping"], t["cos_cache"], t["sin_cache"],
                           kc, vc, rotary_dim=D, page_size=P)
    out4 = fused_int4_paged_decode_attention(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"],
                                             t["block_table"], t["seq_lens"])
    out16 = fused_fp16_paged_decode_attention(t["query"], kc, vc, t["block_table"], t["seq_lens"])
    torch.cuda.synchronize()
    assert torch.isfinite(out4).all() and torch.isfinite(out16).all()
    cosine, rmse = _gate(out4, out16)
    assert cosine > 0.97, cosine
    assert rmse < 0.20, rmse
