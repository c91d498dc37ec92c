"""Pins the CPU oracle against the reference: known-answer vectors from the
reference's own tests, and golden fixtures produced by running the
reference's eager code (tests/golden/make_golden.py).  CPU only."""
import hashlib

import numpy as np
import pytest

import cases
from oracle import iris_oracle as orc


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --- known answers copied from the reference's tests ----------------------

def test_rope_pos_zero_is_identity():
    # tests/test_correctness.py:18-31
    x = np.random.default_rng(0).standard_normal((2, 3, 8)).astype(np.float16)
    out = orc.apply_rope(x, np.ones((2, 1, 4), np.float16), np.zeros((2, 1, 4), np.float16), 8)
    assert np.array_equal(out, x)


def test_rope_known_quarter_turn():
    # tests/test_correctness.py:34-49: [1,2,3,4] -> [-3,-4,1,2] (NeoX half split)
    x = np.array([[[1.0, 2.0, 3.0, 4.0]]], np.float16)
    out = orc.apply_rope(x, np.zeros((1, 1, 2), np.float16), np.ones((1, 1, 2), np.float16), 4)
    assert out.tolist() == [[[-3.0, -4.0, 1.0, 2.0]]]


def test_rope_preserves_passthrough_dims():
    # tests/test_correctness.py:307-324
    x = np.random.default_rng(1).standard_normal((2, 3, 8)).astype(np.float16)
    out = orc.apply_rope(x, np.zeros((2, 1, 2), np.float16), np.ones((2, 1, 2), np.float16), 4)
    assert np.array_equal(out[..., 4:], x[..., 4:])


def test_quantize_int4_known_values():
    # tests/test_correctness.py:52-72
    q, s = orc.quantize_int4_groupwise(np.array([[[-7.0, -3.0, 0.0, 7.0]]], np.float16), 4)
    assert q.tolist() == [[[-7, -3, 0, 7]]] and q.dtype == np.int8
    assert s.tolist() == [[[1.0]]]


def test_quantize_int4_zero_group_is_finite():
    # tests/test_correctness.py:75-82
    q, s = orc.quantize_int4_groupwise(np.zeros((2, 3, 8), np.float16), 4)
    assert np.all(q == 0) and np.all(np.isfinite(s)) and np.all(s > 0)


def test_pack_int4_known_values():
    # tests/test_correctness.py:85-101: low nibble first, two's complement
    packed = orc.pack_int4(np.array([[-7, -1, 0, 1, 6, 7]], np.int8))
    assert packed.tolist() == [[0xF9, 0x10, 0x76]]


def test_unpack_inverts_pack():
    q = np.arange(-7, 8, dtype=np.int8)
    q = np.concatenate([q, q[::-1][:1]])
    assert np.array_equal(orc.unpack_int4(orc.pack_int4(q)), q)


def test_duplicate_slots_rejected():
    # tests/test_correctness.py:295-304
    c = cases.append_small()
    c["slot_mapping"] = np.array([3, 0, 3, 6], np.int32)
    with pytest.raises(ValueError):
        orc.append(**{k: c[k] for k in cases.APPEND_KEYS}, rotary_dim=c["rotary_dim"],
                   group_size=c["group_size"], page_size=c["page_size"])


@pytest.mark.parametrize("bad,exc", [("pos_neg", IndexError), ("pos_big", IndexError), ("slot_big", IndexError)])
def test_range_errors(bad, exc):
    c = cases.append_small()
    if bad == "pos_neg":
        c["positions"] = np.array([0, -1, 2, 3], np.int32)
    elif bad == "pos_big":
        c["positions"] = np.array([0, 1, 2, 4], np.int32)
    else:
        c["slot_mapping"] = np.array([3, 0, -1, 8], np.int32)
    with pytest.raises(exc):
        orc.append(**{k: c[k] for k in cases.APPEND_KEYS}, rotary_dim=c["rotary_dim"],
                   group_size=c["group_size"], page_size=c["page_size"])


# --- golden fixtures from the reference's eager code ------------------------

def _run_append(c):
    c = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}
    orc.append(**{k: c[k] for k in cases.APPEND_KEYS}, rotary_dim=c["rotary_dim"],
               group_size=c["group_size"], page_size=c["page_size"])
    return c


@pytest.mark.parametrize("name", ["append_small", "append_hot", "append_outliers"])
def test_append_matches_reference_bit_exact(golden, name):
    c = getattr(cases, name)()
    for k in cases.APPEND_KEYS:  # the generator is the one the fixture was made from
        assert np.array_equal(golden[f"{name}.in.{k}"], c[k], equal_nan=True), k
    r = _run_append(c)
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        assert r[k].tobytes() == golden[f"{name}.out.{k}"].tobytes(), k


def test_quant_edge_rows_match_reference(golden):
    x = cases.quant_edge_groups()
    assert np.array_equal(golden["quant_edge.in.x"], x)
    q, s = orc.quantize_int4_groupwise(x, 32)
    assert np.array_equal(q, golden["quant_edge.out.q"])
    assert s.tobytes() == golden["quant_edge.out.scale"].tobytes()
    assert np.array_equal(orc.pack_int4(q), golden["quant_edge.out.packed"])


def test_amax_to_scale_table_exhaustive(golden):
    x = cases.fp16_amax_table_input()[:0x7C00]
    q, s = orc.quantize_int4_groupwise(x, 32)
    assert s.reshape(-1).tobytes() == golden["amax_table.out.scale"].tobytes()
    assert np.array_equal(orc.pack_int4(q)[:, 0, 0], golden["amax_table.out.byte0"])


def test_config1_append_digests(golden):
    r = _run_append(cases.config1())
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        assert _sha(r[k]) == str(golden[f"config1.sha.{k}"]), k


def _decode16(c, **kw):
    return orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS], page_size=c["page_size"],
                                group_size=c["group_size"], **kw).astype(np.float16)


def _assert_fp16_close(got, ref):
    """The oracle runs the same FP32 math in a different summation order, so
    its fp16-cast output may differ from the reference's by one fp16 ulp, or
    by FP32 summation noise (1e-5 absolute) for outputs near zero."""
    g = got.astype(np.float32)
    r = ref.astype(np.float32)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    err = np.abs(g - r)
    assert np.all(err <= ulp + 1e-5), float(np.max(err - ulp))
    assert np.mean(g == r) > 0.99


def test_config1_decode_matches_reference(golden):
    c = _run_append(cases.config1())
    _assert_fp16_close(_decode16(c), golden["config1.out.output"])


def test_attention_ref_case_matches_reference(golden):
    c = _run_append(cases.attention_ref_case())
    for k in ("k_data", "v_data", "k_scale", "v_scale"):
        assert c[k].tobytes() == golden[f"attn_ref.out.{k}"].tobytes()
    _assert_fp16_close(_decode16(c), golden["attn_ref.out.output"])


@pytest.mark.parametrize("name", sorted(cases.DECODE_SPECS))
def test_decode_cases_match_reference(golden, name):
    c = cases.decode_random(**cases.DECODE_SPECS[name])
    _assert_fp16_close(_decode16(c), golden[f"decode.{name}.out.output"])


@pytest.mark.parametrize("name", sorted(cases.FP16_DECODE_SPECS))
def test_fp16_decode_cases_match_reference(golden, name):
    """The matched FP16 decode oracle against the reference's eager FP16
    decode (torch_eager_attention.py:243-294), NaN/Inf tail slots included."""
    c = cases.decode_random_fp16(**cases.FP16_DECODE_SPECS[name])
    got = orc.decode_attention_fp16(*[c[k] for k in cases.FP16_DECODE_KEYS]).astype(np.float16)
    _assert_fp16_close(got, golden[f"fp16_decode.{name}.out.output"])


@pytest.mark.parametrize("name", sorted(cases.FP16_APPEND_SPECS))
def test_fp16_append_matches_reference(golden, name):
    """The FP16 append oracle against the reference test's own expectation
    (its apply_rope, then the scatter), byte for byte."""
    c = cases.fp16_append_case(**cases.FP16_APPEND_SPECS[name])
    orc.append_fp16(*[c[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=c["rotary_dim"], page_size=c["page_size"])
    for k in ("k_cache", "v_cache"):
        assert c[k].tobytes() == golden[f"fp16_append.{name}.out.{k}"].tobytes()


def test_merge_of_split_partials_equals_full():
    c = cases.decode_random(**cases.DECODE_SPECS["gqa4_d128"])
    full, _ = orc.decode_attention_lse(*[c[k] for k in cases.DECODE_KEYS])
    # split sequence 2 (200 tokens) into page-aligned pieces and merge
    b = 2
    parts_o, parts_l = [], []
    for lo, hi in ((0, 64), (64, 176), (176, 200)):
        cc = dict(c)
        cc["block_table"] = c["block_table"][b:b + 1, lo // 16:]
        cc["seq_lens"] = np.array([hi - lo], np.int32)
        cc["query"] = c["query"][b:b + 1]
        o, l = orc.decode_attention_lse(*[cc[k] for k in cases.DECODE_KEYS])
        parts_o.append(o)
        parts_l.append(l)
    merged = orc.merge_partials(np.stack(parts_o), np.stack(parts_l))
    np.testing.assert_allclose(merged[0], full[b], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("make", [cases.attention_ref_case, cases.config1], ids=["reference_fixture", "config1"])
def test_int4_oracle_tracks_fp16_oracle(make):
    """The reference's quality gate (tests/test_attention.py:199-232: mean
    cosine > 0.97 and RMSE < 0.20 between the INT4 and the matched FP16
    decode over the same keys and values) holds for the oracle's INT4 and FP16
    restatements: the same K/V appended once quantised, once in fp16."""
    c = _run_append(make())
    NP, P, Hkv, _ = c["k_data"].shape
    D = c["query"].shape[2]
    kc = np.zeros((NP, P, Hkv, D), np.float16)
    vc = np.zeros_like(kc)
    orc.append_fp16(c["key"], c["value"], c["positions"], c["slot_mapping"], c["cos_cache"], c["sin_cache"], kc, vc,
                    rotary_dim=D, page_size=P)
    a = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]).astype(np.float16).astype(np.float64)
    b = orc.decode_attention_fp16(c["query"], kc, vc, c["block_table"], c["seq_lens"]).astype(np.float16)
    a, b = a.reshape(-1, D), b.astype(np.float64).reshape(-1, D)
    cosine = np.mean(np.sum(a * b, -1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1)))
    rmse = np.sqrt(np.mean((a - b) ** 2))
    assert cosine > 0.97 and rmse < 0.20, (cosine, rmse)
