"""Multi-GPU decode (iris_kernel.parallel) on the GPU.

* Split-context on one GPU with the ranks emulated in turn (each rank's LSE
  partial from the CUDA decode over its own splits, the packed buffers
  concatenated as an all-gather would, merged by the CUDA merge) equals the
  FP32 oracle within the decode tolerance, for 2, 3 and 8 ranks and both
  split assignments.
* The packed merge ignores parts whose lse is -inf (their O may be garbage).
* Sequence sharding: per-shard decodes reassembled equal the oracle.
* With two or more GPUs: split-context between two processes, each GPU's
  cache holding only its own splits' pages (every other page poisoned with
  NaN scales), over NCCL and over NVLink peer memory (eager and replayed
  from a CUDA graph), equals the oracle on both ranks."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu


def _case():
    # ragged lengths: one-token and one-page sequences, partial last pages
    return cases.decode_random(seed=123, B=6, Hq=32, Hkv=8, D=128, lens=[1000, 1, 333, 16, 2049, 700])


def _emulated(c, world, mode, split_tokens):
    from iris_kernel import parallel as P
    from iris_kernel.fused_attention import decode_partial, merge_lse_packed

    t = to_dev(c, cases.DECODE_KEYS)
    B, Hq, D = t["query"].shape
    sends = []
    for rank in range(world):
        plan = P.plan_split_context(c["seq_lens"], world, rank, split_tokens=split_tokens, mode=mode)
        if len(plan.seqs) == 0:
            sends.append(P.pack_partials(torch.zeros(0, Hq, D, device="cuda"), torch.zeros(0, Hq, device="cuda"),
                                         plan.seqs, B))
            continue
        idx = torch.from_numpy(plan.seqs).cuda()
        o, lse = decode_partial(t["query"].index_select(0, idx).contiguous(), t["k_data"], t["v_data"],
                                t["k_scale"], t["v_scale"], P.local_block_table(plan, t["block_table"]),
                                torch.from_numpy(plan.lens.astype(np.int32)).cuda())
        sends.append(P.pack_partials(o, lse, plan.seqs, B))
    out = merge_lse_packed(torch.cat(sends), world, B, Hq, D)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("mode", ["strided", "contiguous"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_split_context_emulated_ranks_match_oracle(world, mode):
    c = _case()
    out = _emulated(c, world, mode, split_tokens=256)
    assert_decode_close(out, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))


def test_merge_packed_ignores_minus_inf_parts():
    from iris_kernel import parallel as P
    from iris_kernel.fused_attention import merge_lse_packed

    B, Hq, D = 3, 4, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    bufs = [torch.randn(P.packed_size(B, Hq, D), generator=g, device="cuda") for _ in range(3)]
    o2, lse2 = P.packed_views(bufs[2], B, Hq, D)
    o2[1].fill_(float("nan"))
    lse2[1].fill_(float("-inf"))
    out = merge_lse_packed(torch.cat(bufs), 3, B, Hq, D).float()
    torch.cuda.synchronize()
    parts = [P.packed_views(b, B, Hq, D) for b in bufs]
    o = np.stack([p[0].cpu().numpy() for p in parts])
    lse = np.stack([p[1].cpu().numpy() for p in parts]) * np.log(2.0)  # kernel lse is base 2
    ref = np.empty((B, Hq, D), np.float32)
    for b in range(B):
        use = [0, 1] if b == 1 else [0, 1, 2]
        ref[b] = orc.merge_partials(o[use, b], lse[use, b])
    assert torch.isfinite(out).all()
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=2e-3, rtol=1e-2)


def test_sequence_sharding_reassembles_to_oracle():
    from iris_kernel import parallel as P
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = _case()
    t = to_dev(c, cases.DECODE_KEYS)
    out = torch.empty_like(t["query"])
    for shard in P.balance_sequences(c["seq_lens"], 4):
        if not shard:
            continue
        idx = torch.tensor(shard, device="cuda")
        out[idx] = fused_int4_paged_decode_attention(
            t["query"][idx].contiguous(), t["k_data"], t["v_data"], t["k_scale"], t["v_scale"],
            t["block_table"][idx].contiguous(), t["seq_lens"][idx].contiguous())
    torch.cuda.synchronize()
    assert_decode_close(out, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))


def test_split_context_decoder_replays_in_a_cuda_graph():
    """The prepared one-GPU decoder (world of one: no collective) captured in a
    CUDA graph and replayed gives the oracle's output."""
    import iris_kernel
    from iris_kernel import parallel as P

    c = _case()
    t = to_dev(c, cases.DECODE_KEYS)
    plan = P.plan_split_context(c["seq_lens"], 1, 0, split_tokens=256)
    dec = P.SplitContextDecoder(plan, t["block_table"], 32, 128)
    args = [t[k] for k in ("query", "k_data", "v_data", "k_scale", "v_scale")]
    iris_kernel.set_validation_mode("deferred")
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            dec(*args)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = dec(*args)
        dec.output.zero_()
        g.replay()
        torch.cuda.synchronize()
        iris_kernel.check_errors()
    finally:
        iris_kernel.set_validation_mode("sync")
    assert_decode_close(out, orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, c, expected):
    from iris_kernel import parallel as P

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        t = to_dev(c, cases.DECODE_KEYS, device=f"cuda:{rank}")
        plan = P.plan_split_context(c["seq_lens"], world, rank, split_tokens=256, mode="strided")
        # this GPU's cache keeps only the pages of its own splits
        mine = torch.zeros(t["k_data"].shape[0], dtype=torch.bool, device=t["k_data"].device)
        local_bt = P.local_block_table(plan, t["block_table"])
        for i in range(len(plan.seqs)):
            npg = -(-int(plan.lens[i]) // 16)
            mine[local_bt[i, :npg].long()] = True
        for k in ("k_scale", "v_scale"):
            t[k][~mine] = float("nan")
        for k in ("k_data", "v_data"):
            t[k][~mine] = 0x77
        out = P.split_context_decode(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"],
                                     t["block_table"], plan)
        torch.cuda.synchronize()
        assert_decode_close(out, expected)
        dec = P.SplitContextDecoder(plan, t["block_table"], t["query"].shape[1], t["query"].shape[2])
        out2 = dec(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"])
        torch.cuda.synchronize()
        assert torch.equal(out2, out)
        # the same over NVLink peer memory (CUDA IPC exchange buffers, no NCCL in the step):
        # eager calls, then a CUDA graph replayed twice (each step's merge waits for the
        # other GPU's partial, and for its read of this GPU's, before the next decode)
        p2p = P.SplitContextDecoder(plan, t["block_table"], t["query"].shape[1], t["query"].shape[2],
                                    transport="p2p")
        try:
            out3 = p2p(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"]).clone()
            torch.cuda.synchronize()
            assert_decode_close(out3, expected)
            import iris_kernel

            iris_kernel.set_validation_mode("deferred")
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                p2p(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                out4 = p2p(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"])
            for _ in range(2):
                out4.zero_()
                g.replay()
                torch.cuda.synchronize()
                iris_kernel.check_errors()
                assert_decode_close(out4, expected)
            iris_kernel.set_validation_mode("sync")
            del g
        finally:
            p2p.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_split_context_two_gpus_nccl():
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    c = _case()
    expected = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    mp.spawn(_nccl_worker, args=(2, _free_port(), c, expected), nprocs=2, join=True)
