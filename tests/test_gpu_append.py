"""GPU parity of the fused write path against the oracle / reference golden
fixtures: packed bytes and fp16 scales must be bit-identical."""
import hashlib

import numpy as np
import pytest
import torch

import cases
from _refs import to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu

CACHE = ("k_data", "v_data", "k_scale", "v_scale")


def _fused(c):
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    t = to_dev(c, cases.APPEND_KEYS)
    fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=c["rotary_dim"],
                                 group_size=c["group_size"], page_size=c["page_size"])
    torch.cuda.synchronize()
    return {k: t[k].cpu().numpy() for k in CACHE}


def _oracle(c):
    c = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}
    orc.append(**{k: c[k] for k in cases.APPEND_KEYS}, rotary_dim=c["rotary_dim"], group_size=c["group_size"],
               page_size=c["page_size"])
    return {k: c[k] for k in CACHE}


def _assert_bytes_equal(got, ref):
    for k in CACHE:
        assert got[k].tobytes() == ref[k].tobytes(), k


@pytest.mark.parametrize("name", ["append_hot", "append_outliers"])
def test_matches_reference_golden(golden, name):
    got = _fused(getattr(cases, name)())
    for k in CACHE:
        assert got[k].tobytes() == golden[f"{name}.out.{k}"].tobytes(), k


def test_config1_matches_reference_digests(golden):
    got = _fused(cases.config1())
    for k in CACHE:
        assert hashlib.sha256(got[k].tobytes()).hexdigest() == str(golden[f"config1.sha.{k}"]), k


def test_reference_hot_path_case_all_four_tensors_bit_exact():
    # tests/test_correctness.py:592-748 (the reference only checks k_scale to 2e-3)
    c = cases.append_hot(seed=7)
    _assert_bytes_equal(_fused(c), _oracle(c))


@pytest.mark.parametrize("D", [64, 128, 192, 256, 512])
@pytest.mark.parametrize("H", [1, 3, 8])
def test_head_dims_and_heads(D, H):
    rng = np.random.default_rng(D * 10 + H)
    T, P, NP = 37, 16, 8
    c = cases.append_outliers(seed=D + H, T=T, H=H, D=D, P=P, NP=NP, max_pos=64)
    c["key"] = (rng.standard_normal((T, H, D)) * 3).astype(np.float16)
    _assert_bytes_equal(_fused(c), _oracle(c))


def test_exhaustive_amax_to_scale_and_quantiser_sweep():
    """Every finite non-negative fp16 amax value, each group filled with
    random fp16 values |x| <= amax (random bit patterns), through both the
    K path (identity RoPE) and the V path."""
    rng = np.random.default_rng(99)
    amax = np.arange(0x7C00, dtype=np.uint16).view(np.float16)  # 31744 groups
    bits = rng.integers(0, 0x7C00, (amax.size, 31), dtype=np.uint16)
    x = bits.view(np.float16).astype(np.float32)
    x = np.minimum(x, amax.astype(np.float32)[:, None])  # |x| <= amax
    sign = rng.random(x.shape) < 0.5
    x = np.where(sign, -x, x).astype(np.float16)
    grp = np.concatenate([amax[:, None], x], axis=1)
    # shuffle the position of the amax element inside each group
    perm = rng.permuted(np.tile(np.arange(32), (amax.size, 1)), axis=1)
    grp = np.take_along_axis(grp, perm, axis=1)
    T, H, D = amax.size // 4, 1, 128
    val = grp.reshape(T, H, D)
    c = dict(key=val, value=val[::-1].copy(), positions=np.zeros(T, np.int32),
             slot_mapping=np.arange(T, dtype=np.int32), cos_cache=np.ones((1, 64), np.float16),
             sin_cache=np.zeros((1, 64), np.float16), k_data=np.zeros((T // 16, 16, H, 64), np.uint8),
             v_data=np.zeros((T // 16, 16, H, 64), np.uint8), k_scale=np.zeros((T // 16, 16, H, 4), np.float16),
             v_scale=np.zeros((T // 16, 16, H, 4), np.float16), rotary_dim=D, group_size=32, page_size=16)
    _assert_bytes_equal(_fused(c), _oracle(c))


def test_config5a_decode_style_append_full():
    """BASELINE config 5a: 2048 sequences x 1 token, Hkv=1, D=128, random
    positions in [0, 32768), RoPE base 500000, 1% x20 outliers."""
    rng = np.random.default_rng(51)
    T, H, D, P = 2048, 1, 128, 16
    x = rng.standard_normal((2, T, H, D), dtype=np.float32)
    x[rng.random(x.shape) < 0.01] *= 20
    cos, sin = orc.rope_cache(32768, D, 500000.0)
    NP = 2048 * 2
    slots = (rng.permutation(NP)[:T] * P + rng.integers(0, P, T)).astype(np.int32)
    c = dict(key=x[0].astype(np.float16), value=x[1].astype(np.float16),
             positions=rng.integers(0, 32768, T).astype(np.int32), slot_mapping=slots, cos_cache=cos, sin_cache=sin,
             k_data=np.zeros((NP, P, H, D // 2), np.uint8), v_data=np.zeros((NP, P, H, D // 2), np.uint8),
             k_scale=np.zeros((NP, P, H, D // 32), np.float16), v_scale=np.zeros((NP, P, H, D // 32), np.float16),
             rotary_dim=D, group_size=32, page_size=P)
    _assert_bytes_equal(_fused(c), _oracle(c))


@pytest.mark.parametrize("H,D", [(3, 128), (1, 256), (8, 64), (5, 192), (2, 512)])
def test_large_batches_all_rows_bit_exact(H, D):
    """Batches of more than one resident wave of CTAs, so the L2 prefetch of
    later CTAs' rows is active and runs past the end: odd head counts, a
    ragged end, padding slots and random positions, every row compared with
    the oracle."""
    rng = np.random.default_rng(H * 1000 + D)
    P = 16
    T = -(-16500 // H) + 5  # rows >= 16384, not a multiple of the tile
    NP = -(-T // P) + 8
    x = rng.standard_normal((2, T, H, D), dtype=np.float32) * 2
    x[rng.random(x.shape) < 0.01] *= 20
    cos, sin = orc.rope_cache(4096, D, 10000.0)
    slots = (rng.permutation(NP * P)[:T]).astype(np.int32)
    slots[rng.random(T) < 0.03] = -1
    c = dict(key=x[0].astype(np.float16), value=x[1].astype(np.float16),
             positions=rng.integers(0, 4096, T).astype(np.int32), slot_mapping=slots, cos_cache=cos, sin_cache=sin,
             k_data=np.full((NP, P, H, D // 2), 0x5A, np.uint8), v_data=np.full((NP, P, H, D // 2), 0x5A, np.uint8),
             k_scale=np.full((NP, P, H, D // 32), 2.0, np.float16),
             v_scale=np.full((NP, P, H, D // 32), 2.0, np.float16), rotary_dim=D, group_size=32, page_size=P)
    _assert_bytes_equal(_fused(c), _oracle(c))


@pytest.mark.parametrize("T,D", [(300, 128), (100, 128), (37, 64)])
def test_sixteen_byte_aligned_inputs_take_the_narrow_loads(T, D):
    """K / V / cos / sin bases that are 16- but not 32-byte aligned use the
    16-byte load form of either kernel (large batches, and batches of at most
    128 tokens); the result is the same bytes."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = cases.append_outliers(seed=5 + T, T=T, H=8, D=D, P=16, NP=32, max_pos=512)
    ref = _oracle(c)
    t = to_dev(c, cases.APPEND_KEYS)

    def shifted(x):  # same values, base address 16 bytes past a 32-byte boundary
        buf = torch.empty(x.numel() + 8, dtype=x.dtype, device=x.device)
        y = buf[8:].view(x.shape)
        y.copy_(x)
        assert y.data_ptr() % 32 == 16
        return y

    for k in ("key", "value", "cos_cache", "sin_cache"):
        t[k] = shifted(t[k])
    fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=c["rotary_dim"],
                                 group_size=c["group_size"], page_size=c["page_size"])
    torch.cuda.synchronize()
    _assert_bytes_equal({k: t[k].cpu().numpy() for k in CACHE}, ref)


def test_config5b_prefill_append_full_size_sampled():
    """BASELINE config 5b at full size (8 x 8192 tokens, Hkv=8, D=128, fresh
    permuted pages): every written row must equal the oracle's; rows are
    compared in full for a 4096-token sample and the whole cache through a
    size-independent round trip (each dequantised value within half a scale
    step of the rotated input) plus the untouched-pages check."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    g = torch.Generator(device="cuda").manual_seed(52)
    S, L, H, D, P = 8, 8192, 8, 128, 16
    T = S * L
    NP = T // P + 64
    dev = "cuda"
    k = torch.randn(T, H, D, generator=g, device=dev)
    v = torch.randn(T, H, D, generator=g, device=dev)
    k[torch.rand(k.shape, generator=g, device=dev) < 0.01] *= 20
    v[torch.rand(v.shape, generator=g, device=dev) < 0.01] *= 20
    k, v = k.half(), v.half()
    cos_np, sin_np = orc.rope_cache(L, D, 500000.0)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    pages = torch.randperm(NP, generator=g, device=dev)[: T // P].view(S, L // P)
    pos = torch.arange(L, device=dev, dtype=torch.int32).repeat(S)
    slots = (pages.repeat_interleave(P, dim=1) * P + torch.arange(L, device=dev) % P).view(-1).int()
    kd = torch.full((NP, P, H, D // 2), 0xAB, dtype=torch.uint8, device=dev)
    vd = kd.clone()
    ks = torch.full((NP, P, H, D // 32), 3.0, dtype=torch.float16, device=dev)
    vs = ks.clone()
    fused_rope_int4_paged_append(k, v, pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D, page_size=P)
    torch.cuda.synchronize()
    # sampled bit-exact rows against the oracle
    idx = torch.randperm(T, generator=g, device=dev)[:4096]
    si = slots[idx].long()
    sub = dict(key=k[idx].cpu().numpy(), value=v[idx].cpu().numpy(), positions=pos[idx].cpu().numpy(),
               slot_mapping=np.arange(4096, dtype=np.int32), cos_cache=cos_np, sin_cache=sin_np,
               k_data=np.zeros((256, P, H, D // 2), np.uint8), v_data=np.zeros((256, P, H, D // 2), np.uint8),
               k_scale=np.zeros((256, P, H, D // 32), np.float16), v_scale=np.zeros((256, P, H, D // 32), np.float16),
               rotary_dim=D, group_size=32, page_size=P)
    ref = _oracle(sub)
    for name, t in (("k_data", kd), ("v_data", vd), ("k_scale", ks), ("v_scale", vs)):
        got = t.view(NP * P, H, -1)[si].cpu().numpy()
        assert got.tobytes() == ref[name].reshape(4096, H, -1).tobytes(), name
    # untouched pages keep their fill
    used = torch.zeros(NP, dtype=torch.bool, device=dev)
    used[pages.view(-1)] = True
    assert bool((kd[~used] == 0xAB).all()) and bool((vs[~used] == 3.0).all())
    # round trip over every written row: |dequant(v) - v| <= scale / 2 (values inside the clamp)
    from _refs import unpack_dequant_torch

    vrow = vd.view(NP * P, H, D // 2)[slots.long()]
    srow = vs.view(NP * P, H, D // 32)[slots.long()]
    deq = unpack_dequant_torch(vrow, srow)
    err = (deq - v.float()).abs()
    bound = srow.float().repeat_interleave(32, dim=-1) * 0.5 * (1 + 1e-3)
    assert bool((err <= bound).all())


def _small_case():
    return cases.append_hot(seed=3)


def test_negative_slot_is_ignored():
    c = _small_case()
    c["slot_mapping"] = np.full(7, -1, np.int32)
    got = _fused(c)
    for k in CACHE:
        assert got[k].tobytes() == c[k].tobytes()


def test_unwritten_regions_unchanged():
    c = _small_case()
    got = _fused(c)
    mask = np.zeros(c["k_data"].shape[:2], bool)
    s = c["slot_mapping"][c["slot_mapping"] >= 0]
    mask[s // 16, s % 16] = True
    for k in CACHE:
        assert got[k][~mask].tobytes() == c[k][~mask].tobytes()


@pytest.mark.parametrize("bad,exc", [("dup", ValueError), ("slot", IndexError), ("pos_neg", IndexError),
                                     ("pos_big", IndexError)])
def test_errors_raise_reference_types_and_leave_cache_untouched(bad, exc):
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = _small_case()
    if bad == "dup":
        c["slot_mapping"] = np.array([17, 2, -1, 31, 17, 47, 63], np.int32)
    elif bad == "slot":
        c["slot_mapping"] = np.array([17, 2, -1, 31, 64, 47, 63], np.int32)
    elif bad == "pos_neg":
        c["positions"] = np.array([0, 1, 2, -3, 4, 5, 6], np.int32)
    else:
        c["positions"] = np.array([0, 1, 2, 3, 4, 5, 7], np.int32)
    t = to_dev(c, cases.APPEND_KEYS)
    before = {k: t[k].clone() for k in CACHE}
    with pytest.raises(exc):
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
    for k in CACHE:
        assert torch.equal(t[k], before[k])


@pytest.mark.parametrize("T", [128, 129, 300])
@pytest.mark.parametrize("bad,exc", [("dup", ValueError), ("slot", IndexError), ("pos_big", IndexError)])
def test_errors_on_both_validation_paths(T, bad, exc):
    """Batches of at most 128 tokens are validated inside the append kernel,
    larger ones by the check kernel before it: the same errors either way,
    with the offending tokens at the ends of the batch."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    NP = -(-T // 16) + 4
    c = cases.append_outliers(seed=T, T=T, H=2, D=128, P=16, NP=NP, max_pos=512)
    sm = c["slot_mapping"]
    live = np.flatnonzero(sm >= 0)
    first, last = int(live[0]), int(live[-1])
    if bad == "dup":
        sm[last] = sm[first]
    elif bad == "slot":
        sm[last] = NP * 16
    else:
        c["positions"][first] = 512
    t = to_dev(c, cases.APPEND_KEYS)
    before = {k: t[k].clone() for k in CACHE}
    with pytest.raises(exc):
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
    for k in CACHE:
        assert torch.equal(t[k], before[k])


def test_c_abi_check_then_append_on_a_small_batch():
    """A C-ABI caller that runs iris_b200_append_check before a small batch
    (which the append also validates itself) gets the same bytes and the
    same rejection."""
    from iris_kernel import _lib

    lib = _lib.lib
    for dup in (False, True):
        c = _small_case()
        if dup:
            c["slot_mapping"] = np.array([17, 2, -1, 31, 17, 47, 63], np.int32)
        t = to_dev(c, cases.APPEND_KEYS)
        before = {k: t[k].clone() for k in CACHE}
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        NP, P = t["k_data"].shape[0], t["k_data"].shape[1]
        T, H, D = t["key"].shape
        ws = torch.zeros(max(lib.iris_b200_append_check_workspace_bytes(NP, P), 4), dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        pos, sl = t["positions"], t["slot_mapping"]
        assert lib.iris_b200_append_check(pos.data_ptr(), sl.data_ptr(), T, t["cos_cache"].shape[0], NP, P,
                                          ws.data_ptr(), ws.numel(), err.data_ptr(), stream) == 0
        assert lib.iris_b200_rope_int4_paged_append(
            t["key"].data_ptr(), t["value"].data_ptr(), pos.data_ptr(), sl.data_ptr(), t["cos_cache"].data_ptr(),
            t["sin_cache"].data_ptr(), t["k_data"].data_ptr(), t["v_data"].data_ptr(), t["k_scale"].data_ptr(),
            t["v_scale"].data_ptr(), T, H, D, t["cos_cache"].shape[0], NP, P, err.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        if dup:
            assert int(err.item()) == _lib.ERR_DUP_SLOT
            for k in CACHE:
                assert torch.equal(t[k], before[k])
        else:
            assert int(err.item()) == 0
            ref = _oracle(c)
            for k in CACHE:
                assert t[k].cpu().numpy().tobytes() == ref[k].tobytes(), k


def test_deferred_validation_records_and_rejects_the_batch():
    """Deferred mode: no host sync in the call; the bad batch is recorded and,
    as in the reference (which raises before writing), nothing of it is
    written.  Until check_errors() clears the record, later appends on the
    device are refused too; after it, they write normally."""
    import iris_kernel
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = _small_case()
    good = to_dev(c, cases.APPEND_KEYS)
    bad_c = dict(c)
    bad_c["slot_mapping"] = np.array([17, 2, -1, 31, 99, 47, 63], np.int32)  # one slot out of range
    t = to_dev(bad_c, cases.APPEND_KEYS)
    before = {k: t[k].clone() for k in CACHE}
    good_before = {k: good[k].clone() for k in CACHE}
    iris_kernel.set_validation_mode("deferred")
    try:
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
        fused_rope_int4_paged_append(*[good[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
        torch.cuda.synchronize()
        for k in CACHE:
            assert torch.equal(t[k], before[k])  # rejected batch: untouched
            assert torch.equal(good[k], good_before[k])  # refused while the error is pending
        with pytest.raises(IndexError):
            iris_kernel.check_errors()
        iris_kernel.check_errors()  # cleared
        fused_rope_int4_paged_append(*[good[k] for k in cases.APPEND_KEYS], rotary_dim=128, page_size=16)
        iris_kernel.check_errors()
    finally:
        iris_kernel.set_validation_mode("sync")
    ref = _oracle(c)
    for k in CACHE:
        assert good[k].cpu().numpy().tobytes() == ref[k].tobytes()


def test_unsupported_shapes_raise():
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    c = cases.append_small()  # D=8, G=4: outside the fused path, as in the reference
    t = to_dev(c, cases.APPEND_KEYS)
    with pytest.raises(NotImplementedError):
        fused_rope_int4_paged_append(*[t[k] for k in cases.APPEND_KEYS], rotary_dim=8, group_size=4, page_size=2)
    c = _small_case()
    t = to_dev(c, cases.APPEND_KEYS)
    with pytest.raises(TypeError):
        fused_rope_int4_paged_append(t["key"], t["value"], t["positions"].long(), t["slot_mapping"], t["cos_cache"],
                                     t["sin_cache"], *[t[k] for k in CACHE], rotary_dim=128, page_size=16)


def _quant_case(groups):
    """Wrap [N, 32] fp16 groups as a V-only append (identity RoPE on K too)."""
    n = groups.shape[0]
    pad = (-n) % 64
    if pad:
        groups = np.concatenate([groups, np.zeros((pad, 32), np.float16)])
    T = groups.shape[0] // 4
    val = groups.reshape(T, 1, 128)
    NPg = T // 16
    return dict(key=val[::-1].copy(), value=val, positions=np.zeros(T, np.int32),
                slot_mapping=np.arange(T, dtype=np.int32), cos_cache=np.ones((1, 64), np.float16),
                sin_cache=np.zeros((1, 64), np.float16), k_data=np.zeros((NPg, 16, 1, 64), np.uint8),
                v_data=np.zeros((NPg, 16, 1, 64), np.uint8), k_scale=np.zeros((NPg, 16, 1, 4), np.float16),
                v_scale=np.zeros((NPg, 16, 1, 4), np.float16), rotary_dim=128, group_size=32, page_size=16)


def test_quantiser_every_exact_tie():
    """Every (amax, k) with x = (k + 1/2) * scale representable in fp16 and
    |x| <= amax: the quotient is exactly a half-integer and must round to
    even, as the reference's IEEE division + torch.round do."""
    amax = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16)
    a32 = amax.astype(np.float32)
    s = np.maximum(a32 / np.float32(7.0), np.float32(2.0 ** -14)).astype(np.float16).astype(np.float32)
    rows = []
    for k in range(-8, 8):
        x = ((k + 0.5) * s).astype(np.float32)
        ok = (x.astype(np.float16).astype(np.float32) == x) & (np.abs(x) <= a32)
        rows.append(np.stack([a32[ok], x[ok]], 1))
    pairs = np.concatenate(rows)
    assert len(pairs) > 50000
    g = np.zeros((len(pairs), 32), np.float32)
    g[:, 0] = pairs[:, 0]
    g[:, 1:] = pairs[:, 1:2]  # the tie value in 31 slots
    g[:, 2] = -pairs[:, 1]
    c = _quant_case(g.astype(np.float16))
    _assert_bytes_equal(_fused(c), _oracle(c))


def test_quantiser_dense_sweep():
    """For 600 amax values spread over the fp16 range, every fp16 x with
    |x| <= amax (both signs), against the oracle's IEEE division."""
    rng = np.random.default_rng(2024)
    pick = np.unique(np.concatenate([rng.integers(1, 0x7C00, 560), np.arange(0x3C00 - 20, 0x3C00 + 20)]))
    allx = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    groups = []
    for bits in pick:
        a = np.array([bits], np.uint16).view(np.float16).astype(np.float32)[0]
        xs = allx[allx <= a]
        xs = np.concatenate([xs, -xs])
        n = (len(xs) + 30) // 31
        body = np.zeros(n * 31, np.float32)
        body[:len(xs)] = xs
        grp = np.concatenate([np.full((n, 1), a, np.float32), body.reshape(n, 31)], 1)
        groups.append(grp)
    g = np.concatenate(groups).astype(np.float16)
    assert g.shape[0] > 100000
    c = _quant_case(g)
    _assert_bytes_equal(_fused(c), _oracle(c))
