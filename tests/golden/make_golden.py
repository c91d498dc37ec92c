"""Generate the golden fixtures by running the REFERENCE's own eager code.

Run in a container where the reference checkout is mounted (read-only)::

    python tests/golden/make_golden.py /path/to/Iris-Kernel

It imports ``iris_kernel.torch_eager_kv`` and
``iris_kernel.torch_eager_attention`` from ``<ref>/src`` (CPU PyTorch; the
TileLang modules are never imported), feeds them the deterministic numpy
inputs of ``cases.py`` and writes ``golden.npz``.  Small cases store full
inputs and outputs; config 1 stores SHA-256 digests of the written cache plus
the full decode output (its inputs are rebuilt from ``cases.config1``).
The GPU box never reads the reference: only the committed ``golden.npz``.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, _HERE)
import cases  # noqa: E402


def _t(a):
    return torch.from_numpy(np.array(a, copy=True))


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from iris_kernel.torch_eager_attention import (torch_eager_fp16_paged_decode_attention,
                                                   torch_eager_int4_paged_decode_attention)
    from iris_kernel.torch_eager_kv import apply_rope, pack_int4, quantize_int4_groupwise, torch_eager_append

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out: dict[str, np.ndarray] = {}

    def run_append(prefix, c, store_inputs=True):
        t = {k: _t(c[k]) for k in cases.APPEND_KEYS}
        t["positions"] = t["positions"].to(torch.int64)
        t["slot_mapping"] = t["slot_mapping"].to(torch.int64)
        torch_eager_append(**t, rotary_dim=c["rotary_dim"], group_size=c["group_size"], page_size=c["page_size"])
        for k in ("k_data", "v_data", "k_scale", "v_scale"):
            arr = t[k].numpy()
            if store_inputs:
                out[f"{prefix}.out.{k}"] = arr
            out[f"{prefix}.sha.{k}"] = np.array(_sha(arr))
        if store_inputs:
            for k in cases.APPEND_KEYS:
                out[f"{prefix}.in.{k}"] = c[k]
        return {k: t[k].numpy() for k in ("k_data", "v_data", "k_scale", "v_scale")}

    def run_decode(prefix, c, cache=None):
        t = {k: _t(c[k]) for k in cases.DECODE_KEYS}
        if cache is not None:
            for k, v in cache.items():
                t[k] = _t(v)
        o = torch_eager_int4_paged_decode_attention(
            t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"], t["block_table"], t["seq_lens"],
            page_size=c["page_size"], group_size=c["group_size"])
        out[f"{prefix}.out.output"] = o.numpy()

    run_append("append_small", cases.append_small())
    run_append("append_hot", cases.append_hot())
    run_append("append_outliers", cases.append_outliers())

    # quantiser edge rows and the exhaustive amax -> scale table
    x = cases.quant_edge_groups()
    q, s = quantize_int4_groupwise(_t(x), group_size=32)
    out["quant_edge.in.x"] = x
    out["quant_edge.out.q"] = q.numpy()
    out["quant_edge.out.scale"] = s.numpy()
    out["quant_edge.out.packed"] = pack_int4(q).numpy()
    tab = cases.fp16_amax_table_input()[:0x7C00]  # finite non-negative amax values
    q, s = quantize_int4_groupwise(_t(tab), group_size=32)
    out["amax_table.out.scale"] = s.numpy().reshape(-1)
    out["amax_table.out.byte0"] = pack_int4(q).numpy()[:, 0, 0]

    # config 1: write through the eager append, then eager decode
    c1 = cases.config1()
    cache = run_append("config1", c1, store_inputs=False)
    run_decode("config1", c1, cache)

    # the reference attention test's case shape (cache written by eager append)
    ac = cases.attention_ref_case()
    cache = run_append("attn_ref", ac, store_inputs=False)
    for k, v in cache.items():
        out[f"attn_ref.out.{k}"] = v
    run_decode("attn_ref", ac, cache)

    for name, spec in cases.DECODE_SPECS.items():
        dc = cases.decode_random(**spec)
        run_decode(f"decode.{name}", dc)

    # the matched FP16 decode (its eager reference casts the result to fp16)
    for name, spec in cases.FP16_DECODE_SPECS.items():
        fc = cases.decode_random_fp16(**spec)
        t = {k: _t(fc[k]) for k in cases.FP16_DECODE_KEYS}
        o = torch_eager_fp16_paged_decode_attention(t["query"], t["k_cache"], t["v_cache"], t["block_table"],
                                                    t["seq_lens"], page_size=fc["page_size"])
        out[f"fp16_decode.{name}.out.output"] = o.numpy()

    # FP16 append: the reference test's expectation (apply_rope, then scatter)
    for name, spec in cases.FP16_APPEND_SPECS.items():
        c = cases.fp16_append_case(**spec)
        t = {k: _t(c[k]) for k in cases.FP16_APPEND_KEYS}
        valid = t["slot_mapping"] >= 0
        slots = t["slot_mapping"][valid].long()
        pos = t["positions"][valid].long()
        half = c["rotary_dim"] // 2
        rk = apply_rope(t["key"][valid], t["cos_cache"][pos][:, None, :half], t["sin_cache"][pos][:, None, :half],
                        rotary_dim=c["rotary_dim"])
        t["k_cache"][slots // c["page_size"], slots % c["page_size"]] = rk
        t["v_cache"][slots // c["page_size"], slots % c["page_size"]] = t["value"][valid]
        out[f"fp16_append.{name}.out.k_cache"] = t["k_cache"].numpy()
        out[f"fp16_append.{name}.out.v_cache"] = t["v_cache"].numpy()

    path = os.path.join(_HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
