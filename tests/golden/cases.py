"""Deterministic (numpy PCG64) input generators for the golden fixtures and
the parity tests.  Shapes follow the reference's own test fixtures
(tests/test_correctness.py:104-183, :592-748; tests/test_attention.py:16-162)
and BASELINE config 1.  Everything here is plain numpy so the same inputs are
rebuilt bit-identically on any host with the same numpy.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(os.path.dirname(_HERE))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle import iris_oracle as orc  # noqa: E402  (test infrastructure)


def _randn16(rng, shape, std=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float16)


def _cache(rng, num_pages, page_size, hkv, d, group, fill="random"):
    dshape = (num_pages, page_size, hkv, d // 2)
    sshape = (num_pages, page_size, hkv, d // group)
    if fill == "zeros":
        return (np.zeros(dshape, np.uint8), np.zeros(dshape, np.uint8),
                np.zeros(sshape, np.float16), np.zeros(sshape, np.float16))
    return (rng.integers(0, 256, dshape, dtype=np.uint8), rng.integers(0, 256, dshape, dtype=np.uint8),
            _randn16(rng, sshape), _randn16(rng, sshape))


def append_small(seed=3407):
    """Shape of the reference's ``_make_append_case`` (T=4, Hkv=2, D=8,
    page 2, G=4, slots [3,0,-1,6], identity RoPE, random prefilled cache)."""
    rng = np.random.default_rng(seed)
    T, H, D, P, NP, G = 4, 2, 8, 2, 4, 4
    key = _randn16(rng, (T, H, D))
    value = rng.random((T, H, D), dtype=np.float32).astype(np.float16)
    kd, vd, ks, vs = _cache(rng, NP, P, H, D, G)
    return dict(key=key, value=value, positions=np.arange(4, dtype=np.int32),
                slot_mapping=np.array([3, 0, -1, 6], np.int32),
                cos_cache=np.ones((4, D // 2), np.float16), sin_cache=np.zeros((4, D // 2), np.float16),
                k_data=kd, v_data=vd, k_scale=ks, v_scale=vs, rotary_dim=D, group_size=G, page_size=P)


def append_hot(seed=3407):
    """Shape of the reference's hot-path append test: T=7, Hkv=4, D=128,
    page 16, 4 pages, slots [17,2,-1,31,32,47,63], base-10000 RoPE."""
    rng = np.random.default_rng(seed)
    T, H, D, P, NP, G = 7, 4, 128, 16, 4, 32
    key = _randn16(rng, (T, H, D))
    value = _randn16(rng, (T, H, D))
    cos, sin = orc.rope_cache(7, D)
    kd, vd, ks, vs = _cache(rng, NP, P, H, D, G)
    return dict(key=key, value=value, positions=np.arange(7, dtype=np.int32),
                slot_mapping=np.array([17, 2, -1, 31, 32, 47, 63], np.int32),
                cos_cache=cos, sin_cache=sin, k_data=kd, v_data=vd, k_scale=ks, v_scale=vs,
                rotary_dim=D, group_size=G, page_size=P)


def append_outliers(seed=11, T=96, H=2, D=128, P=16, NP=16, base=500000.0, max_pos=512):
    """Config-5-style distribution at CPU size: N(0,1) with 1% of entries x20,
    random positions, scattered unique slots, RoPE base 500000."""
    rng = np.random.default_rng(seed)
    G = 32
    def draw():
        x = rng.standard_normal((T, H, D), dtype=np.float32)
        mask = rng.random((T, H, D)) < 0.01
        x[mask] *= 20.0
        return x.astype(np.float16)
    key, value = draw(), draw()
    cos, sin = orc.rope_cache(max_pos, D, base)
    slots = rng.permutation(NP * P)[:T].astype(np.int32)
    slots[rng.random(T) < 0.1] = -1
    pos = rng.integers(0, max_pos, T).astype(np.int32)
    kd, vd, ks, vs = _cache(rng, NP, P, H, D, G)
    return dict(key=key, value=value, positions=pos, slot_mapping=slots, cos_cache=cos, sin_cache=sin,
                k_data=kd, v_data=vd, k_scale=ks, v_scale=vs, rotary_dim=D, group_size=G, page_size=P)


def quant_edge_groups():
    """Hand-built [N, 1, 32*k] fp16 rows that stress the quantiser: exact
    .5 ties, all-zero groups, subnormals, fp16 max, a single spike, signed
    zeros and values straddling the clamp."""
    rows = []
    g = np.zeros(32, np.float32)
    rows.append(g.copy())                                   # all zero
    t = np.zeros(32, np.float32); t[0] = 7.0; t[1:15] = np.arange(14) * 0.5 - 3.25
    rows.append(t)                                          # scale 1, many .25/.75
    t = np.zeros(32, np.float32); t[0] = 7.0; t[1:16] = np.arange(-7.5, 7.5, 1.0)
    rows.append(t)                                          # exact ties k+0.5
    t = np.full(32, 2.0 ** -24, np.float32); t[3] = -2.0 ** -20
    rows.append(t)                                          # subnormals -> 2^-14 clamp
    t = np.zeros(32, np.float32); t[5] = 65504.0; t[6] = -65504.0; t[7] = 4680.0
    rows.append(t)                                          # fp16 max
    t = np.linspace(-1, 1, 32, dtype=np.float32); t[-1] = 100.0
    rows.append(t)                                          # spike
    t = -np.zeros(32, np.float32); t[9] = 1e-3
    rows.append(t)                                          # -0.0 and a small value
    rng = np.random.default_rng(5)
    for s in (1.0, 0.37, 1e-3, 3e3):
        rows.append((rng.standard_normal(32) * s).astype(np.float32))
    # ties generated from random fp16 scales: x = (k + 0.5) * s exactly
    for _ in range(8):
        s = np.float16(rng.uniform(0.01, 10))
        k = rng.integers(-7, 7, 32)
        x = ((k + 0.5) * np.float32(s)).astype(np.float32)
        x[0] = 7 * np.float32(s)
        rows.append(x)
    arr = np.stack(rows).astype(np.float16)
    return arr.reshape(arr.shape[0], 1, 32)


def fp16_amax_table_input():
    """One group of 32 per non-negative fp16 bit pattern 0x0000..0x7FFF
    (finite, inf and NaN): element 0 holds the pattern, the rest are 0, so the
    group amax is that value.  Pins the amax -> fp16 scale map exhaustively."""
    bits = np.arange(0x8000, dtype=np.uint16)
    x = np.zeros((0x8000, 1, 32), np.float16)
    x[:, 0, 0] = bits.view(np.float16)
    return x


def config1(seed=0):
    """batch 4, Hkv=8, Hq=32, D=128, page 16, group 32,
    160 pages, lens [37,128,255,512], per-sequence page tables are disjoint
    slices of a permutation of 160 page ids (seed 0), K/V ~N(0,1) fp16, RoPE
    base 10000 at positions 0..len-1, one fp16 ~N(0,1) query per sequence."""
    rng = np.random.default_rng(seed)
    B, Hq, Hkv, D, P, G, NP = 4, 32, 8, 128, 16, 32, 160
    lens = np.array([37, 128, 255, 512], np.int32)
    perm = rng.permutation(NP).astype(np.int32)
    maxp = int(math.ceil(lens.max() / P))
    bt = np.zeros((B, maxp), np.int32)
    o = 0
    for b in range(B):
        n = int(math.ceil(lens[b] / P))
        bt[b, :n] = perm[o:o + n]
        o += n
    keys, vals, poss, slots = [], [], [], []
    for b in range(B):
        L = int(lens[b])
        keys.append(_randn16(rng, (L, Hkv, D)))
        vals.append(_randn16(rng, (L, Hkv, D)))
        p = np.arange(L, dtype=np.int32)
        poss.append(p)
        slots.append((bt[b, p // P] * P + p % P).astype(np.int32))
    cos, sin = orc.rope_cache(int(lens.max()), D)
    kd, vd, ks, vs = _cache(rng, NP, P, Hkv, D, G, fill="zeros")
    query = _randn16(rng, (B, Hq, D))
    return dict(key=np.concatenate(keys), value=np.concatenate(vals), positions=np.concatenate(poss),
                slot_mapping=np.concatenate(slots), cos_cache=cos, sin_cache=sin,
                k_data=kd, v_data=vd, k_scale=ks, v_scale=vs, rotary_dim=D, group_size=G, page_size=P,
                query=query, block_table=bt, seq_lens=lens)


def decode_random(seed, B, Hq, Hkv, D, lens, *, spare_pages=3, extra_cols=0, scale_lo=0.01, scale_hi=1.0,
                  garbage_tail=True):
    """Random packed cache (any byte) + random positive fp16 scales, a random
    page permutation and ragged lengths.  Slots past each sequence's length in
    its last page hold garbage, including NaN/Inf scales when
    ``garbage_tail`` (the reference benchmark allocates with torch.empty)."""
    rng = np.random.default_rng(seed)
    P, G = 16, 32
    lens = np.asarray(lens, np.int32)
    npg = [int(math.ceil(int(L) / P)) for L in lens]
    NP = sum(npg) + spare_pages
    perm = rng.permutation(NP).astype(np.int32)
    maxp = max(npg) + extra_cols
    bt = np.full((B, maxp), -1, np.int32)
    o = 0
    for b in range(B):
        bt[b, :npg[b]] = perm[o:o + npg[b]]
        o += npg[b]
    kd = rng.integers(0, 256, (NP, P, Hkv, D // 2), dtype=np.uint8)
    vd = rng.integers(0, 256, (NP, P, Hkv, D // 2), dtype=np.uint8)
    ks = rng.uniform(scale_lo, scale_hi, (NP, P, Hkv, D // G)).astype(np.float16)
    vs = rng.uniform(scale_lo, scale_hi, (NP, P, Hkv, D // G)).astype(np.float16)
    if garbage_tail:
        for b in range(B):
            L = int(lens[b])
            if L % P:
                last = bt[b, npg[b] - 1]
                ks[last, L % P:] = np.float16(np.nan)
                vs[last, L % P:] = np.float16(np.inf)
    q = _randn16(rng, (B, Hq, D))
    return dict(query=q, k_data=kd, v_data=vd, k_scale=ks, v_scale=vs, block_table=bt, seq_lens=lens,
                page_size=P, group_size=G)


def attention_ref_case(seed=3407):
    """Shape of the reference's ``_make_attention_case``: B=2, Hq=8, Hkv=2,
    D=128, lens [23, 31], randperm pages with 3 spare, cache written by the
    append path, query RoPE'd at position L-1."""
    rng = np.random.default_rng(seed)
    B, Hq, Hkv, D, P, G = 2, 8, 2, 128, 16, 32
    lens = np.array([23, 31], np.int32)
    maxp = 2
    NP = B * maxp + 3
    bt = rng.permutation(NP)[:B * maxp].reshape(B, maxp).astype(np.int32)
    cos, sin = orc.rope_cache(int(lens.max()), D)
    keys, vals, poss, slots = [], [], [], []
    for b in range(B):
        L = int(lens[b])
        keys.append(_randn16(rng, (L, Hkv, D)))
        vals.append(_randn16(rng, (L, Hkv, D)))
        p = np.arange(L, dtype=np.int32)
        poss.append(p)
        slots.append((bt[b, p // P] * P + p % P).astype(np.int32))
    kd, vd, ks, vs = _cache(rng, NP, P, Hkv, D, G, fill="zeros")
    qu = _randn16(rng, (B, Hq, D))
    qpos = lens - 1
    query = orc.apply_rope(qu, cos[qpos][:, None, :], sin[qpos][:, None, :], D)
    return dict(key=np.concatenate(keys), value=np.concatenate(vals), positions=np.concatenate(poss),
                slot_mapping=np.concatenate(slots), cos_cache=cos, sin_cache=sin,
                k_data=kd, v_data=vd, k_scale=ks, v_scale=vs, rotary_dim=D, group_size=G, page_size=P,
                query=query, block_table=bt, seq_lens=lens)


APPEND_KEYS = ("key", "value", "positions", "slot_mapping", "cos_cache", "sin_cache",
               "k_data", "v_data", "k_scale", "v_scale")
DECODE_KEYS = ("query", "k_data", "v_data", "k_scale", "v_scale", "block_table", "seq_lens")

# decode cases exercised against the reference's eager decode
def decode_random_fp16(seed, B, Hq, Hkv, D, lens, *, spare_pages=3, garbage_tail=True):
    """FP16 paged cache ~N(0,1) with a random page permutation and ragged
    lengths; slots past a sequence's end in its last page hold NaN / Inf
    when ``garbage_tail``."""
    rng = np.random.default_rng(seed)
    P = 16
    lens = np.asarray(lens, np.int32)
    npg = [int(math.ceil(int(L) / P)) for L in lens]
    NP = sum(npg) + spare_pages
    perm = rng.permutation(NP).astype(np.int32)
    bt = np.full((B, max(npg)), -1, np.int32)
    o = 0
    for b in range(B):
        bt[b, :npg[b]] = perm[o:o + npg[b]]
        o += npg[b]
    kc = _randn16(rng, (NP, P, Hkv, D))
    vc = _randn16(rng, (NP, P, Hkv, D))
    if garbage_tail:
        for b in range(B):
            L = int(lens[b])
            if L % P:
                last = bt[b, npg[b] - 1]
                kc[last, L % P:] = np.float16(np.nan)
                vc[last, L % P:] = np.float16(np.inf)
    q = _randn16(rng, (B, Hq, D))
    return dict(query=q, k_cache=kc, v_cache=vc, block_table=bt, seq_lens=lens, page_size=P)


FP16_DECODE_KEYS = ("query", "k_cache", "v_cache", "block_table", "seq_lens")

FP16_APPEND_KEYS = ("key", "value", "positions", "slot_mapping", "cos_cache", "sin_cache", "k_cache", "v_cache")


def fp16_append_case(seed, T=7, H=4, D=128, rotary_dim=128, P=16, NP=4, base=10000.0, slots=None):
    """The reference test's FP16 append case shape (tests/test_correctness.py:
    327-458): random K/V and caches, scattered / negative slots."""
    rng = np.random.default_rng(seed)
    key = _randn16(rng, (T, H, D))
    value = _randn16(rng, (T, H, D))
    if slots is None:
        slots = rng.permutation(NP * P)[:T].astype(np.int32)
        slots[T // 3] = -1
    positions = rng.integers(0, 64, T).astype(np.int32)
    half = rotary_dim // 2
    inv = 1.0 / (base ** (np.arange(0, rotary_dim, 2, dtype=np.float32) / rotary_dim))
    freqs = np.arange(64, dtype=np.float32)[:, None] * inv[None, :]
    return dict(key=key, value=value, positions=positions, slot_mapping=np.asarray(slots, np.int32),
                cos_cache=np.cos(freqs).astype(np.float16), sin_cache=np.sin(freqs).astype(np.float16),
                k_cache=_randn16(rng, (NP, P, H, D)), v_cache=_randn16(rng, (NP, P, H, D)),
                rotary_dim=rotary_dim, page_size=P)


FP16_APPEND_SPECS = {
    "ref_shape": dict(seed=41),
    "partial_rotary": dict(seed=42, D=128, rotary_dim=64),
    "d64_many": dict(seed=43, T=40, H=2, D=64, rotary_dim=64, NP=8),
    "odd_rotary": dict(seed=44, T=9, H=3, D=96, rotary_dim=36, NP=2),
}

FP16_DECODE_SPECS = {
    "gqa4_d128": dict(seed=31, B=3, Hq=32, Hkv=8, D=128, lens=[1, 17, 700]),
    "mha_d64": dict(seed=32, B=4, Hq=8, Hkv=8, D=64, lens=[16, 15, 33, 300]),
    "gqa16_d128": dict(seed=33, B=2, Hq=32, Hkv=2, D=128, lens=[64, 129]),
}

DECODE_SPECS = {
    "gqa4_d128": dict(seed=21, B=3, Hq=16, Hkv=4, D=128, lens=[1, 17, 200]),
    "mha_d64": dict(seed=22, B=4, Hq=4, Hkv=4, D=64, lens=[16, 15, 33, 300]),
    "gqa16_d128": dict(seed=23, B=2, Hq=32, Hkv=2, D=128, lens=[64, 129]),
    "mqa_d64": dict(seed=24, B=2, Hq=8, Hkv=1, D=64, lens=[5, 1000]),
    "gqa8_d128_extra_cols": dict(seed=25, B=2, Hq=16, Hkv=2, D=128, lens=[48, 7], extra_cols=5),
}
