"""DecodeStep (append + decode captured in one CUDA graph) equals the same
two calls made eagerly (identical cache bytes and output) and the CPU
oracle (cache bytes bit-exact, output within the decode tolerance), over
several steps that append one token per sequence and extend the lengths; a
rejected append inside the graph is reported by check=True and writes
nothing."""
import numpy as np
import pytest
import torch

import math

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _setup(seed):
    """Config 1 with room to grow: every sequence's table gets 4 more columns
    of unused pages and the RoPE tables cover 64 more positions."""
    c = cases.config1(seed=seed)
    bt, lens = c["block_table"], c["seq_lens"]
    npg = [int(math.ceil(int(L) / 16)) for L in lens]
    used = {int(bt[b, j]) for b in range(len(lens)) for j in range(npg[b])}
    free = [p for p in range(c["k_data"].shape[0]) if p not in used]
    grown = np.zeros((len(lens), bt.shape[1] + 4), np.int32)
    for b in range(len(lens)):
        grown[b, :npg[b]] = bt[b, :npg[b]]
        for j in range(npg[b], grown.shape[1]):
            grown[b, j] = free.pop()
    c["block_table"] = grown
    c["cos_cache"], c["sin_cache"] = orc.rope_cache(int(lens.max()) + 64, 128)
    keys = cases.APPEND_KEYS + ("query", "block_table", "seq_lens")
    return c, to_dev(c, keys)


def test_graph_step_equals_eager_calls():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append
    from iris_kernel.step import DecodeStep

    c, ta = _setup(0)
    _, tb = _setup(0)
    B, Hq, D = ta["query"].shape
    Hkv = ta["k_data"].shape[2]
    for t in (ta, tb):  # the prefill, written the same way on both
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=D, page_size=16)
    oc = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}  # the oracle's copy
    orc.append(**{k: oc[k] for k in cases.APPEND_KEYS}, rotary_dim=D, group_size=32, page_size=16)
    step = DecodeStep(ta["k_data"], ta["v_data"], ta["k_scale"], ta["v_scale"], ta["block_table"], ta["seq_lens"],
                      ta["cos_cache"], ta["sin_cache"], num_q_heads=Hq, new_tokens=B, rotary_dim=D)
    g = torch.Generator(device="cuda").manual_seed(7)
    for _ in range(3):
        pos = tb["seq_lens"].clone()
        page = tb["block_table"].gather(1, (pos // 16).long().unsqueeze(1)).squeeze(1)
        slots = (page * 16 + pos % 16).int()
        k = torch.randn(B, Hkv, D, generator=g, device="cuda").half()
        v = torch.randn(B, Hkv, D, generator=g, device="cuda").half()
        q = torch.randn(B, Hq, D, generator=g, device="cuda").half()
        for t in (ta, tb):
            t["seq_lens"].add_(1)
        out_graph = step(q, k, v, pos, slots, check=True).clone()
        fused_rope_int4_paged_append(k, v, pos, slots, tb["cos_cache"], tb["sin_cache"], tb["k_data"], tb["v_data"],
                                     tb["k_scale"], tb["v_scale"], rotary_dim=D, page_size=16)
        out_eager = fused_int4_paged_decode_attention(q, tb["k_data"], tb["v_data"], tb["k_scale"], tb["v_scale"],
                                                      tb["block_table"], tb["seq_lens"])
        torch.cuda.synchronize()
        assert torch.equal(out_graph, out_eager)
        for k_ in ("k_data", "v_data", "k_scale", "v_scale"):
            assert torch.equal(ta[k_], tb[k_])
        # the oracle, on the same step inputs
        oc["seq_lens"] = oc["seq_lens"] + 1
        orc.append(k.cpu().numpy(), v.cpu().numpy(), pos.cpu().numpy(), slots.cpu().numpy(), oc["cos_cache"],
                   oc["sin_cache"], oc["k_data"], oc["v_data"], oc["k_scale"], oc["v_scale"], rotary_dim=D,
                   group_size=32, page_size=16)
        for k_ in ("k_data", "v_data", "k_scale", "v_scale"):
            assert ta[k_].cpu().numpy().tobytes() == oc[k_].tobytes(), k_
        ref = orc.decode_attention(q.cpu().numpy(), oc["k_data"], oc["v_data"], oc["k_scale"], oc["v_scale"],
                                   oc["block_table"], oc["seq_lens"])
        assert_decode_close(out_graph, ref)


def test_graph_step_reports_a_rejected_append():
    from iris_kernel.fused_kv import fused_rope_int4_paged_append
    from iris_kernel.step import DecodeStep

    c, t = _setup(1)
    B, Hq, D = t["query"].shape
    Hkv = t["k_data"].shape[2]
    fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=D, page_size=16)
    step = DecodeStep(t["k_data"], t["v_data"], t["k_scale"], t["v_scale"], t["block_table"], t["seq_lens"],
                      t["cos_cache"], t["sin_cache"], num_q_heads=Hq, new_tokens=B, rotary_dim=D)
    before = {k: t[k].clone() for k in ("k_data", "v_data", "k_scale", "v_scale")}
    slots = torch.full((B,), 5, dtype=torch.int32, device="cuda")  # one slot for every token: duplicates
    k = torch.zeros(B, Hkv, D, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        step(t["query"], k, k, torch.zeros(B, dtype=torch.int32, device="cuda"), slots, check=True)
    for name, v in before.items():
        assert torch.equal(t[name], v)
