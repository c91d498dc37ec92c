"""GPU parity of the INT4 paged decode against the FP32 oracle (tolerance
max-abs 2e-3 / relative 1e-2), edge cases, errors, and full-size configs
checked through the PyTorch FP32 reference on sampled sequences."""
import math

import numpy as np
import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev, torch_decode_fp32
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _fused(c, **kw):
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    t = to_dev(c, cases.DECODE_KEYS)
    out = fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS], **kw)
    torch.cuda.synchronize()
    return out


def _oracle(c, **kw):
    return orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS], **kw)


def test_attention_ref_case_matches_golden_and_oracle(golden):
    c = cases.attention_ref_case()
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        c[k] = golden[f"attn_ref.out.{k}"].copy()
    out = _fused(c)
    assert out.dtype == torch.float16 and out.shape == (2, 8, 128)
    assert_decode_close(out, _oracle(c))
    # the reference test's own bound against its fp16 eager output (tests/test_attention.py:196)
    assert_decode_close(out, golden["attn_ref.out.output"].astype(np.float32), atol=5e-2, rtol=5e-2)


@pytest.mark.parametrize("name", sorted(cases.DECODE_SPECS))
def test_decode_specs_match_oracle(golden, name):
    c = cases.decode_random(**cases.DECODE_SPECS[name])
    out = _fused(c)
    assert_decode_close(out, _oracle(c))
    assert_decode_close(out, golden[f"decode.{name}.out.output"].astype(np.float32), atol=3e-3, rtol=1e-2)


def test_config1_write_then_decode(golden):
    """BASELINE config 1 end to end on the GPU: fused append writes the cache
    (bit-exact with the oracle), fused decode reads it."""
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = cases.config1()
    t = to_dev(c, cases.APPEND_KEYS + ("query", "block_table", "seq_lens"))
    fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
    out = fused_int4_paged_decode_attention(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"],
                                            t["block_table"], t["seq_lens"])
    torch.cuda.synchronize()
    oc = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}
    orc.append(**{k: oc[k] for k in cases.APPEND_KEYS}, rotary_dim=128, group_size=32, page_size=16)
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        assert t[k].cpu().numpy().tobytes() == oc[k].tobytes(), k
    assert_decode_close(out, _oracle(oc))
    assert_decode_close(out, golden["config1.out.output"].astype(np.float32), atol=3e-3, rtol=1e-2)


GEOMS = [  # (Hq, Hkv, D)
    (8, 8, 64), (16, 16, 64), (32, 8, 128), (16, 2, 128), (32, 2, 128), (8, 1, 128), (16, 1, 64),
    (12, 3, 128), (64, 8, 128), (24, 6, 64), (32, 32, 128),
]


@pytest.mark.parametrize("Hq,Hkv,D", GEOMS)
def test_head_geometries(Hq, Hkv, D):
    c = cases.decode_random(seed=Hq * 100 + Hkv * 10 + D, B=3, Hq=Hq, Hkv=Hkv, D=D, lens=[1, 16, 77])
    assert_decode_close(_fused(c), _oracle(c))


@pytest.mark.parametrize("lens", [[1], [15], [16], [17], [31, 32, 33], [1, 1, 1, 1, 1, 1, 1, 1], [4096]])
def test_lengths(lens):
    c = cases.decode_random(seed=sum(lens), B=len(lens), Hq=32, Hkv=8, D=128, lens=lens)
    assert_decode_close(_fused(c), _oracle(c))


def test_many_short_and_one_long_sequence():
    """Ranges that hold several whole sequences, and a sequence split over
    many ranges (exercises the split-KV records and the combine)."""
    rng = np.random.default_rng(8)
    lens = list(rng.integers(1, 60, 300)) + [20000] + list(rng.integers(1, 40, 50))
    c = cases.decode_random(seed=8, B=len(lens), Hq=8, Hkv=2, D=128, lens=lens)
    assert_decode_close(_fused(c), _oracle(c))


def test_split_records_across_batch_shapes_on_one_workspace():
    """Split-KV records live in the cached workspace, whose layout moves with
    the batch shape: batches with different shapes and split patterns,
    alternated on one stream and one workspace, keep giving the first
    results."""
    a = cases.decode_random(seed=81, B=3, Hq=32, Hkv=8, D=128, lens=[9000, 40, 5000])
    b = cases.decode_random(seed=82, B=5, Hq=32, Hkv=8, D=128, lens=[700, 12000, 3, 3000, 2500])
    first_a, first_b = _fused(a), _fused(b)
    assert_decode_close(first_a, _oracle(a))
    assert_decode_close(first_b, _oracle(b))
    for _ in range(3):
        assert torch.equal(_fused(a), first_a)
        assert torch.equal(_fused(b), first_b)


def test_softmax_scale_and_output_argument():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = cases.decode_random(seed=31, B=2, Hq=16, Hkv=4, D=128, lens=[100, 300])
    t = to_dev(c, cases.DECODE_KEYS)
    out = torch.full_like(t["query"], float("nan"))
    ret = fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS], out, softmax_scale=0.3)
    assert ret.data_ptr() == out.data_ptr()
    assert_decode_close(out, _oracle(c, softmax_scale=0.3))


def test_block_table_column_view():
    """A block table that is a column slice of a wider table (row stride >
    width) reads the right pages."""
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = cases.decode_random(seed=41, B=3, Hq=8, Hkv=2, D=64, lens=[40, 10, 33])
    t = to_dev(c, cases.DECODE_KEYS)
    wide = torch.full((3, t["block_table"].shape[1] + 7), -5, dtype=torch.int32, device="cuda")
    wide[:, :t["block_table"].shape[1]] = t["block_table"]
    view = wide[:, :t["block_table"].shape[1]]
    assert not view.is_contiguous()
    out = fused_int4_paged_decode_attention(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"], view,
                                            t["seq_lens"])
    assert_decode_close(out, _oracle(c))


@pytest.mark.parametrize("bad,exc", [("len0", ValueError), ("short", ValueError), ("page", IndexError),
                                     ("page_neg", IndexError)])
def test_errors(bad, exc):
    c = cases.decode_random(seed=51, B=2, Hq=8, Hkv=2, D=128, lens=[40, 20])
    if bad == "len0":
        c["seq_lens"] = np.array([40, 0], np.int32)
    elif bad == "short":
        c["seq_lens"] = np.array([40, 100], np.int32)
    elif bad == "page":
        c["block_table"] = c["block_table"].copy()
        c["block_table"][1, 1] = c["k_data"].shape[0]
    else:
        c["block_table"] = c["block_table"].copy()
        c["block_table"][0, 2] = -1
    with pytest.raises(exc):
        _fused(c)
    import iris_kernel

    iris_kernel.check_errors()  # sync mode already consumed the error word


def test_unsupported_shapes_raise():
    c = cases.decode_random(seed=52, B=1, Hq=8, Hkv=2, D=128, lens=[20])
    with pytest.raises(NotImplementedError):
        _fused(c, group_size=16)
    c2 = cases.decode_random(seed=53, B=1, Hq=34, Hkv=2, D=128, lens=[20])
    with pytest.raises(NotImplementedError):
        _fused(c2)


def test_decode_partial_and_merge_equal_full():
    """Split-context building blocks: page-aligned token ranges decoded in
    LSE form and merged equal the full decode."""
    from iris_kernel.fused_attention import decode_partial, merge_lse_partials

    c = cases.decode_random(seed=61, B=4, Hq=16, Hkv=4, D=128, lens=[640, 1000, 333, 700], garbage_tail=False)
    t = to_dev(c, cases.DECODE_KEYS)
    bt, L = t["block_table"], t["seq_lens"]
    cuts = [0, 160, 320, 1024]  # tokens (multiples of 16)
    parts_o, parts_l = [], []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        sub_len = torch.clamp(L - lo, min=0).clamp(max=hi - lo)
        assert bool((sub_len > 0).all())
        o, lse = decode_partial(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"],
                                bt[:, lo // 16:], sub_len.int().contiguous())
        parts_o.append(o)
        parts_l.append(lse)
    out = merge_lse_partials(torch.stack(parts_o), torch.stack(parts_l))
    assert_decode_close(out, _oracle(c))
    # the LSE agrees with the oracle's natural-log LSE (converted to log2 units of scaled logits)
    o_full, lse_full = decode_partial(*[t[k] for k in cases.DECODE_KEYS])
    _, lse_ref = orc.decode_attention_lse(*[c[k] for k in cases.DECODE_KEYS])
    np.testing.assert_allclose(lse_full.cpu().numpy(), lse_ref / math.log(2), atol=2e-3, rtol=1e-4)
    assert_decode_close(o_full, _oracle(c), atol=1e-3, rtol=5e-3)


# ------------------------------------------------------------ full sizes

def _full_cache(B, L_list, Hq, Hkv, D, seed, k_outlier_channels=(), kstd=1.0, pool_pages=None):
    """Cache written by the fused append (bit-exact write path) from
    N(0,1) fp16 K/V with RoPE base 10000, pages scattered by a permutation."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    g = torch.Generator(device="cuda").manual_seed(seed)
    P = 16
    npg = [math.ceil(L / P) for L in L_list]
    NP = pool_pages or sum(npg)
    perm = torch.randperm(NP, generator=g, device="cuda").int()
    maxp = max(npg)
    bt = torch.zeros(B, maxp, dtype=torch.int32, device="cuda")
    o = 0
    for b in range(B):
        bt[b, :npg[b]] = perm[o:o + npg[b]]
        o += npg[b]
    kd = torch.zeros(NP, P, Hkv, D // 2, dtype=torch.uint8, device="cuda")
    vd, ks, vs = torch.zeros_like(kd), torch.zeros(NP, P, Hkv, D // 32, dtype=torch.float16, device="cuda"), None
    vs = torch.zeros_like(ks)
    maxL = max(L_list)
    cos_np, sin_np = orc.rope_cache(maxL, D)
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    for b in range(B):  # one sequence per append call keeps peak memory small
        L = L_list[b]
        k = torch.randn(L, Hkv, D, generator=g, device="cuda") * kstd
        for ch in k_outlier_channels:
            k[..., ch] *= 8
        v = torch.randn(L, Hkv, D, generator=g, device="cuda") * kstd
        pos = torch.arange(L, device="cuda", dtype=torch.int32)
        slots = (bt[b, pos // P] * P + pos % P).int()
        fused_rope_int4_paged_append(k.half(), v.half(), pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                     page_size=P)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").half()
    return q, kd, vd, ks, vs, bt, torch.tensor(L_list, dtype=torch.int32, device="cuda")


def test_config2_llama8b_shape_sampled():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    B, L = 64, 4096
    q, kd, vd, ks, vs, bt, lens = _full_cache(B, [L] * B, 32, 8, 128, seed=2, k_outlier_channels=(3, 40, 77, 121))
    out = fused_int4_paged_decode_attention(q, kd, vd, ks, vs, bt, lens)
    seqs = [0, 17, 63]
    ref = torch_decode_fp32(q, kd, vd, ks, vs, bt, lens, seqs=seqs)
    assert_decode_close(out[seqs], ref)


def test_config3_mha_varlen_sampled():
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    rng = np.random.default_rng(1)
    lens = [int(x) for x in rng.integers(1, 16385, 128)]
    q, kd, vd, ks, vs, bt, L = _full_cache(128, lens, 16, 16, 64, seed=3)
    out = fused_int4_paged_decode_attention(q, kd, vd, ks, vs, bt, L)
    seqs = [int(np.argmin(lens)), int(np.argmax(lens)), 5, 77]
    ref = torch_decode_fp32(q, kd, vd, ks, vs, bt, L, seqs=seqs)
    assert_decode_close(out[seqs], ref)


@pytest.mark.parametrize("hq,hkv,d,lens", [(32, 8, 128, [300, 1200]), (16, 16, 64, [1, 17, 64]),
                                           (64, 8, 128, [4096])])
def test_grid_sized_by_the_block_table_width_gives_identical_results(hq, hkv, d, lens):
    """The decode grid is capped by batch * block-table width / 4 ranges; the
    ranges themselves depend only on the lengths, so a wide block table (the
    full grid) and an exact one (a few CTAs) give bit-identical outputs."""
    narrow = cases.decode_random(seed=hq + hkv + d + len(lens), B=len(lens), Hq=hq, Hkv=hkv, D=d, lens=lens)
    wide = dict(narrow)
    bt = narrow["block_table"]
    wide["block_table"] = np.concatenate([bt, np.full((bt.shape[0], 3000), -1, np.int32)], axis=1)
    a, b = _fused(narrow), _fused(wide)
    assert torch.equal(a, b)
    assert_decode_close(a, _oracle(narrow))
