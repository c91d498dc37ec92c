"""BASELINE config 4 at its shape (GPU): Hq 64, Hkv 8, D 128 (the
decode_kernel path: 8 query heads per KV head), 131,072-token contexts,
K/V ~ N(0, 0.5) with K RoPE'd (base 500000) at positions 0..131,071, the
cache written by the fused append over randomly permuted pages.

Two sequences (the config has 16; the shape per sequence is what matters):

* the whole-sequence decode, and
* the split-context decode with 8,192-token splits over 8 emulated ranks,
  both split assignments: each rank's log-sum-exp partial from the CUDA
  decode over its own splits, the packed buffers concatenated as the
  all-gather lays them out, merged by the CUDA merge,

against the PyTorch FP32 reference (``tests/_refs.py``, itself checked
against the oracle) within max-abs 2e-3 / relative 1e-2."""
import numpy as np
import pytest
import torch

from _refs import assert_decode_close, torch_decode_fp32

pytestmark = pytest.mark.gpu

B, L, HQ, HKV, D, P, G = 2, 131072, 64, 8, 128, 16, 32
SPLIT = 8192


def _rope_tables(max_pos, dim, base, dev):
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32, device=dev) / dim))
    f = torch.arange(max_pos, dtype=torch.float32, device=dev)[:, None] * inv[None, :]
    return f.cos().half(), f.sin().half()


@pytest.fixture(scope="module")
def c4():
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(404)
    npg = L // P
    pool = B * npg + 5
    bt = torch.randperm(pool, generator=g, device=dev)[:B * npg].view(B, npg).int().contiguous()
    kd = torch.zeros(pool, P, HKV, D // 2, dtype=torch.uint8, device=dev)
    vd = torch.zeros_like(kd)
    ks = torch.zeros(pool, P, HKV, D // G, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    cos, sin = _rope_tables(L, D, 500000.0, dev)
    pos_all = torch.arange(L, dtype=torch.int32, device=dev)
    chunk = 32768
    for b in range(B):
        for t0 in range(0, L, chunk):
            pos = pos_all[t0:t0 + chunk]
            slots = (bt[b, (pos // P).long()] * P + pos % P).int().contiguous()
            k = (torch.randn(chunk, HKV, D, generator=g, device=dev) * 0.5).half()
            v = (torch.randn(chunk, HKV, D, generator=g, device=dev) * 0.5).half()
            fused_rope_int4_paged_append(k, v, pos.contiguous(), slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                         page_size=P)
    q = torch.randn(B, HQ, D, generator=g, device=dev).half()
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    ref = torch_decode_fp32(q, kd, vd, ks, vs, bt, lens)
    return dict(q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt, lens=lens, ref=ref)


def test_config4_whole_sequence_decode(c4):
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    out = fused_int4_paged_decode_attention(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"], c4["bt"], c4["lens"])
    torch.cuda.synchronize()
    assert_decode_close(out, c4["ref"])


@pytest.mark.parametrize("mode", ["strided", "contiguous"])
def test_config4_split_context_eight_emulated_ranks(c4, mode):
    from iris_kernel import parallel as Pl
    from iris_kernel.fused_attention import decode_partial, merge_lse_packed

    world = 8
    lens_host = np.full(B, L, np.int64)
    sends = []
    for rank in range(world):
        plan = Pl.plan_split_context(lens_host, world, rank, split_tokens=SPLIT, mode=mode)
        assert plan.covers_every_sequence  # 16 splits per sequence over 8 ranks
        o, lse = decode_partial(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"],
                                Pl.local_block_table(plan, c4["bt"]),
                                torch.from_numpy(plan.lens.astype(np.int32)).cuda())
        sends.append(Pl.pack_partials(o, lse, plan.seqs, B))
    out = merge_lse_packed(torch.cat(sends), world, B, HQ, D)
    torch.cuda.synchronize()
    assert_decode_close(out, c4["ref"])
