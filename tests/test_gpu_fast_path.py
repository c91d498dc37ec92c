"""The wrappers' repeat-call fast path (GPU).

A call whose tensors and keyword arguments have the signature of an earlier
call that passed every host check reuses that call's prepared C-ABI
arguments.  It must give the same results, keep raising the device-detected
errors (bad slots, bad page ids) in sync mode, and never let a changed
argument skip its host checks."""
import numpy as np
import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def test_repeat_decode_calls_match_the_oracle_and_each_other():
    from iris_kernel import _runtime
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = cases.decode_random(seed=91, B=3, Hq=16, Hkv=4, D=128, lens=[300, 5, 1200])
    t = to_dev(c, cases.DECODE_KEYS)
    args = [t[k] for k in cases.DECODE_KEYS]
    ref = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    first = fused_int4_paged_decode_attention(*args)
    out = torch.empty_like(first)
    for _ in range(3):  # output given: the fast path after the first call
        fused_int4_paged_decode_attention(*args, out)
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    assert any(k[0] == "int4_decode" for k in _runtime._fast)
    assert_decode_close(first, ref)
    # a changed keyword argument is a new signature (checked, then cached)
    other = fused_int4_paged_decode_attention(*args, softmax_scale=0.2)
    assert_decode_close(other, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS], softmax_scale=0.2))
    # a changed argument that fails a host check still raises
    with pytest.raises(NotImplementedError):
        fused_int4_paged_decode_attention(*args, group_size=16)
    with pytest.raises(ValueError):  # the cache's page size no longer matches
        fused_int4_paged_decode_attention(*args, page_size=32)


def test_fast_path_decode_still_raises_device_detected_errors():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = cases.decode_random(seed=92, B=2, Hq=8, Hkv=2, D=64, lens=[40, 70])
    t = to_dev(c, cases.DECODE_KEYS)
    out = torch.empty_like(t["query"])
    fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS], out)  # cached
    good = t["block_table"][1, 0].item()
    t["block_table"][1, 0] = t["k_data"].shape[0] + 7  # same tensor, bad content
    with pytest.raises(IndexError):
        fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS], out)
    t["block_table"][1, 0] = good
    fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS], out)
    torch.cuda.synchronize()
    assert_decode_close(out, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))


def test_repeat_append_calls_are_bit_exact_and_still_validate():
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = cases.append_hot()
    t = to_dev(c, cases.APPEND_KEYS)
    oc = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}
    for _ in range(2):  # the second call takes the fast path and rewrites the same bytes
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=c["rotary_dim"],
                                     page_size=c["page_size"])
    orc.append(**{k: oc[k] for k in cases.APPEND_KEYS}, rotary_dim=c["rotary_dim"], group_size=32,
               page_size=c["page_size"])
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        assert t[k].cpu().numpy().tobytes() == oc[k].tobytes(), k
    before = {k: t[k].clone() for k in ("k_data", "v_data", "k_scale", "v_scale")}
    live = np.flatnonzero(c["slot_mapping"] >= 0)
    t["slot_mapping"][int(live[1])] = t["slot_mapping"][int(live[0])]  # same tensor, duplicate slots
    with pytest.raises(ValueError):
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=c["rotary_dim"],
                                     page_size=c["page_size"])
    for k, v in before.items():
        assert torch.equal(t[k], v)  # a rejected batch writes nothing


def test_repeat_fp16_decode_calls_match_the_oracle_and_raise_device_errors():
    from iris_kernel import _runtime
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

    c = cases.decode_random_fp16(seed=93, B=3, Hq=16, Hkv=4, D=128, lens=[300, 5, 1200])
    t = to_dev(c, cases.FP16_DECODE_KEYS)
    args = [t[k] for k in cases.FP16_DECODE_KEYS]
    ref = orc.decode_attention_fp16(*[c[k] for k in cases.FP16_DECODE_KEYS])
    first = fused_fp16_paged_decode_attention(*args)
    torch.cuda.synchronize()
    assert_decode_close(first, ref)
    out = torch.empty_like(first)
    for _ in range(3):  # output given: the fast path after the first call
        fused_fp16_paged_decode_attention(*args, out)
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    assert any(k[0] == "fp16_decode" for k in _runtime._fast)
    assert torch.equal(fused_fp16_paged_decode_attention(*args), first)  # output allocated per call
    with pytest.raises(ValueError):  # the cache's page size no longer matches
        fused_fp16_paged_decode_attention(*args, page_size=32)
    bt = t["block_table"]
    good = bt[1, 0].item()
    bt[1, 0] = t["k_cache"].shape[0] + 7  # same tensor, bad content: still caught on the device
    with pytest.raises(IndexError):
        fused_fp16_paged_decode_attention(*args, out)
    bt[1, 0] = good
    fused_fp16_paged_decode_attention(*args, out)
    torch.cuda.synchronize()
    assert torch.equal(out, first)
