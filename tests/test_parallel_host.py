"""Host-side logic of multi-GPU decode (iris_kernel.parallel), on the CPU.

Sequence sharding must give every sequence to exactly one GPU with balanced
token counts; split-context plans must give every page of every sequence to
exactly one GPU, keep a sequence's partly filled final page last, and their
packed partials, all-gathered over a 2-rank gloo group and merged, must equal
the single-device decode.  The per-GPU partial decode is the numpy oracle
here (the CUDA decode is exercised by tests/test_gpu_parallel.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from oracle import iris_oracle as orc


def _parallel():
    from iris_kernel import parallel

    return parallel


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_balance_sequences_covers_and_balances(world):
    P = _parallel()
    rng = np.random.default_rng(world)
    lens = rng.integers(1, 16385, size=128)
    owned = P.balance_sequences(lens, world)
    flat = sorted(b for o in owned for b in o)
    assert flat == list(range(len(lens)))
    loads = [int(lens[o].sum()) for o in owned]
    # longest-processing-time bound: no GPU exceeds the mean by more than the longest sequence
    assert max(loads) <= lens.sum() / world + lens.max()
    for o in owned:
        assert o == sorted(o)


def test_balance_sequences_more_gpus_than_sequences():
    P = _parallel()
    owned = P.balance_sequences([5, 3], 4)
    assert sorted(b for o in owned for b in o) == [0, 1]
    assert sum(1 for o in owned if not o) == 2


@pytest.mark.parametrize("mode", ["strided", "contiguous"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_split_plans_partition_every_page(mode, world):
    P = _parallel()
    rng = np.random.default_rng(7 + world)
    lens = np.concatenate([rng.integers(1, 2000, size=20), [1, 16, 17, 64, 65, 8192, 8193]])
    split, page = 64, 16
    seen = {b: [] for b in range(len(lens))}
    tokens = np.zeros(len(lens), dtype=np.int64)
    for rank in range(world):
        plan = P.plan_split_context(lens, world, rank, split_tokens=split, page_size=page, mode=mode)
        assert list(plan.seqs) == sorted(plan.seqs)
        for i, b in enumerate(plan.seqs):
            npg = -(-int(plan.lens[i]) // page)
            cols = plan.cols[i, :npg].tolist()
            seen[b] += cols
            tokens[b] += plan.lens[i]
            last_page = -(-int(lens[b]) // page) - 1
            if last_page in cols:  # the final (maybe partial) page closes the virtual sequence
                assert cols[-1] == last_page
    for b, L in enumerate(lens):
        assert sorted(seen[b]) == list(range(-(-int(L) // page))), b
    assert (tokens == lens).all()


def test_split_plan_config4_shape():
    """Config 4: 16 x 131,072 tokens in 8192-token splits over 8 GPUs: every
    GPU holds 2 splits of every sequence."""
    P = _parallel()
    for rank in range(8):
        plan = P.plan_split_context([131072] * 16, 8, rank)
        assert plan.covers_every_sequence
        assert (plan.lens == 2 * 8192).all()
        assert plan.cols.shape == (16, 1024)


def test_split_plan_rejects_bad_arguments():
    P = _parallel()
    with pytest.raises(ValueError):
        P.plan_split_context([10], 2, 2)
    with pytest.raises(ValueError):
        P.plan_split_context([10], 2, 0, split_tokens=100)
    with pytest.raises(ValueError):
        P.plan_split_context([0], 1, 0)
    with pytest.raises(ValueError):
        P.plan_split_context([10], 2, 0, mode="diagonal")


def test_local_block_table_and_pack_on_cpu():
    P = _parallel()
    bt = torch.arange(40, dtype=torch.int32).view(4, 10) + 100
    plan = P.plan_split_context([160, 20, 33, 1], 2, 1, split_tokens=32)
    local = P.local_block_table(plan, bt)
    for i, b in enumerate(plan.seqs):
        npg = -(-int(plan.lens[i]) // 16)
        assert local[i, :npg].tolist() == (bt[b, plan.cols[i, :npg]]).tolist()
    o = torch.randn(len(plan.seqs), 3, 8)
    lse = torch.randn(len(plan.seqs), 3)
    buf = P.pack_partials(o, lse, plan.seqs, 4)
    assert buf.numel() == P.packed_size(4, 3, 8)
    po, pl = P.packed_views(buf, 4, 3, 8)
    missing = [b for b in range(4) if b not in set(plan.seqs.tolist())]
    assert torch.equal(po[torch.as_tensor(plan.seqs)], o)
    assert torch.isneginf(pl[missing]).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _split_worker(rank, world, port, mode, case, expected):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        P = _parallel()
        q, kd, vd, ks, vs, bt, lens = (case[k] for k in cases.DECODE_KEYS)
        B, Hq, D = q.shape
        plan = P.plan_split_context(lens, world, rank, split_tokens=48, page_size=16, mode=mode)
        if len(plan.seqs):
            local_bt = P.local_block_table(plan, torch.from_numpy(bt)).numpy()
            o, lse = orc.decode_attention_lse(q[plan.seqs], kd, vd, ks, vs, local_bt, plan.lens)
            send = P.pack_partials(torch.from_numpy(o), torch.from_numpy(lse.astype(np.float32)), plan.seqs, B)
        else:
            send = P.pack_partials(torch.zeros(0, Hq, D), torch.zeros(0, Hq), plan.seqs, B)
        parts = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(parts, send)
        views = [P.packed_views(p, B, Hq, D) for p in parts]
        merged = orc.merge_partials(np.stack([v[0].numpy() for v in views]), np.stack([v[1].numpy() for v in views]))
        np.testing.assert_allclose(merged, expected, atol=2e-5, rtol=1e-4)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["strided", "contiguous"])
def test_split_context_two_gloo_ranks_equal_single_decode(mode):
    c = cases.decode_random(seed=91, B=5, Hq=8, Hkv=2, D=64, lens=[200, 17, 96, 1, 150])
    expected = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    mp.spawn(_split_worker, args=(2, _free_port(), mode, c, expected), nprocs=2, join=True)
