"""Helpers for the parity tests: moving oracle cases to the GPU, the stated
decode tolerance, and a PyTorch FP32 decode reference for sizes the numpy
oracle cannot hold in memory (it is checked against the oracle on small
cases in test_torch_ref_vs_oracle)."""
from __future__ import annotations

import math

import numpy as np
import torch

# decode within max-abs 2e-3 / relative 1e-2 of the
# eager INT4 dequantise-then-attend reference computed in FP32.
DECODE_ATOL = 2e-3
DECODE_RTOL = 1e-2


def assert_decode_close(got, ref, atol=DECODE_ATOL, rtol=DECODE_RTOL):
    g = got.detach().float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got, np.float32)
    r = ref.detach().float().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, np.float32)
    assert g.shape == r.shape
    assert np.all(np.isfinite(g)), "non-finite output"
    err = np.abs(g - r)
    tol = atol + rtol * np.abs(r)
    bad = err > tol
    assert not bad.any(), (
        f"{int(bad.sum())} / {bad.size} outside atol={atol} rtol={rtol}; max abs err {float(err.max()):.3e}, "
        f"worst excess {float((err - tol).max()):.3e}")


def to_dev(case: dict, keys, device="cuda") -> dict:
    out = {}
    for k in keys:
        v = case[k]
        out[k] = torch.from_numpy(np.ascontiguousarray(v)).to(device)
    return out


def unpack_dequant_torch(packed: torch.Tensor, scales: torch.Tensor, group: int = 32) -> torch.Tensor:
    lo = (packed & 0x0F).to(torch.int16)
    hi = (packed >> 4).to(torch.int16)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    q = torch.stack((lo, hi), dim=-1).flatten(-2).float()
    return q * scales.float().repeat_interleave(group, dim=-1)


@torch.no_grad()
def torch_decode_fp32(query, k_data, v_data, k_scale, v_scale, block_table, seq_lens, *, seqs=None,
                      softmax_scale=None, page_size=16, group=32):
    """FP32 decode for the listed sequences, one KV head at a time (no
    repeat_interleave blow-up).  Returns [len(seqs), Hq, D] fp32."""
    B, Hq, D = query.shape
    Hkv = k_data.shape[2]
    rep = Hq // Hkv
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    seqs = range(B) if seqs is None else seqs
    outs = []
    for b in seqs:
        L = int(seq_lens[b])
        npg = math.ceil(L / page_size)
        ids = block_table[b, :npg].long()
        o = torch.empty(Hq, D, dtype=torch.float32, device=query.device)
        for h in range(Hkv):
            k = unpack_dequant_torch(k_data[ids, :, h].reshape(-1, D // 2)[:L], k_scale[ids, :, h].reshape(-1, D // group)[:L], group)
            v = unpack_dequant_torch(v_data[ids, :, h].reshape(-1, D // 2)[:L], v_scale[ids, :, h].reshape(-1, D // group)[:L], group)
            q = query[b, h * rep:(h + 1) * rep].float()
            logits = (q @ k.T) * scale
            p = torch.softmax(logits, dim=-1)
            o[h * rep:(h + 1) * rep] = p @ v
        outs.append(o)
    return torch.stack(outs)
