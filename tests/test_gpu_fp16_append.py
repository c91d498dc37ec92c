"""The FP16 paged append (fused_rope_fp16_append) on the GPU: byte-exact
against the reference test's expectation (golden fixtures) and the oracle,
for full and partial rotary dims (vector and per-element kernels), a large
batch, negative slots, and the reference's errors with the cache untouched."""
import numpy as np
import pytest
import torch

import cases
from _refs import to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _fused(c):
    from iris_kernel.fused_kv import fused_rope_fp16_append

    t = to_dev(c, cases.FP16_APPEND_KEYS)
    fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=c["rotary_dim"],
                           page_size=c["page_size"])
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("name", sorted(cases.FP16_APPEND_SPECS))
def test_matches_reference_bytes(golden, name):
    c = cases.fp16_append_case(**cases.FP16_APPEND_SPECS[name])
    t = _fused(c)
    for k in ("k_cache", "v_cache"):
        assert t[k].cpu().numpy().tobytes() == golden[f"fp16_append.{name}.out.{k}"].tobytes()


def test_large_batch_matches_oracle():
    c = cases.fp16_append_case(seed=45, T=4096, H=8, D=128, rotary_dim=128, NP=300)
    t = _fused(c)
    ref = {k: c[k].copy() for k in ("k_cache", "v_cache")}
    orc.append_fp16(*[c[k] if k not in ref else ref[k] for k in cases.FP16_APPEND_KEYS],
                    rotary_dim=c["rotary_dim"], page_size=c["page_size"])
    for k in ("k_cache", "v_cache"):
        assert t[k].cpu().numpy().tobytes() == ref[k].tobytes()


@pytest.mark.parametrize("rotary_dim,shift", [(48, False), (128, True), (128, False), (96, False)])
def test_every_load_width_matches_oracle(rotary_dim, shift):
    """The kernel's three forms: 16 dims a thread with 32-byte loads (rotary a
    multiple of 32, 32-byte aligned bases), 8 dims with 16-byte loads (rotary
    48, or bases 16 bytes past a 32-byte boundary), byte for byte."""
    from iris_kernel.fused_kv import fused_rope_fp16_append

    c = cases.fp16_append_case(seed=46 + rotary_dim, T=300, H=4, D=128, rotary_dim=rotary_dim, NP=40)
    ref = {k: c[k].copy() for k in ("k_cache", "v_cache")}
    orc.append_fp16(*[c[k] if k not in ref else ref[k] for k in cases.FP16_APPEND_KEYS],
                    rotary_dim=c["rotary_dim"], page_size=c["page_size"])
    t = to_dev(c, cases.FP16_APPEND_KEYS)
    if shift:  # same values, base addresses 16 bytes past a 32-byte boundary
        for k in ("key", "value", "cos_cache", "sin_cache"):
            buf = torch.empty(t[k].numel() + 8, dtype=t[k].dtype, device="cuda")
            y = buf[8:].view(t[k].shape)
            y.copy_(t[k])
            assert y.data_ptr() % 32 == 16
            t[k] = y
    fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=c["rotary_dim"],
                           page_size=c["page_size"])
    torch.cuda.synchronize()
    for k in ("k_cache", "v_cache"):
        assert t[k].cpu().numpy().tobytes() == ref[k].tobytes()


def test_errors_leave_the_cache_untouched():
    from iris_kernel.fused_kv import fused_rope_fp16_append

    c = cases.fp16_append_case(seed=46)
    for slots, exc in (([1, 2, 3, 3, -1, 5, 6], ValueError), ([1, 2, 3, 4, 5, 6, 64], IndexError)):
        c2 = dict(c, slot_mapping=np.asarray(slots, np.int32))
        t = to_dev(c2, cases.FP16_APPEND_KEYS)
        before = {k: t[k].clone() for k in ("k_cache", "v_cache")}
        with pytest.raises(exc):
            fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=128, page_size=16)
        for k in before:
            assert torch.equal(t[k], before[k])
    t = to_dev(c, cases.FP16_APPEND_KEYS)
    with pytest.raises(ValueError):
        fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=130, page_size=16)
    with pytest.raises(TypeError):
        fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS[:6]], t["k_cache"].float(),
                               t["v_cache"].float(), rotary_dim=128, page_size=16)


@pytest.mark.parametrize("T", [64, 128, 129, 300])
@pytest.mark.parametrize("bad,exc", [("dup", ValueError), ("slot", IndexError), ("pos", IndexError)])
def test_errors_on_both_validation_paths(T, bad, exc):
    """Batches of at most 128 tokens are validated inside the FP16 append,
    larger ones by the check kernel before it: the same errors either way,
    with the offending tokens at the ends of the batch."""
    from iris_kernel.fused_kv import fused_rope_fp16_append

    NP = -(-T // 16) + 4
    c = cases.fp16_append_case(seed=T, T=T, H=2, D=128, rotary_dim=128, NP=NP)
    sm = c["slot_mapping"]
    live = np.flatnonzero(sm >= 0)
    first, last = int(live[0]), int(live[-1])
    if bad == "dup":
        sm[last] = sm[first]
    elif bad == "slot":
        sm[last] = NP * 16
    else:
        c["positions"][first] = c["cos_cache"].shape[0]
    t = to_dev(c, cases.FP16_APPEND_KEYS)
    before = {k: t[k].clone() for k in ("k_cache", "v_cache")}
    with pytest.raises(exc):
        fused_rope_fp16_append(*[t[k] for k in cases.FP16_APPEND_KEYS], rotary_dim=128, page_size=16)
    for k in before:
        assert torch.equal(t[k], before[k])
