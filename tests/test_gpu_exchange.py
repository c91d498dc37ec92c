"""Split-context merge over peer memory (``iris_b200_xchg_*``) on one GPU,
the ranks emulated with one exchange buffer each.

On one GPU the emulated ranks' merges cannot wait for one another (nothing
guarantees that separate launches run at the same time), so before each
step the host does what the other ranks' merges would have done by then:
it writes every rank's partial into that rank's slot of the step and raises
every rank's flag.  The merges then run one after another and none of them
waits.  The real cross-GPU handshake runs in the two-GPU worker of
test_gpu_parallel.py.

* Every emulated rank's merge publishes its own partial and merges all of
  them; the output equals the FP32 oracle within the decode tolerance, over
  two steps with different queries (both slots), and the header is left as
  the protocol says (flag and step counter at the step, arrivals reset).
* A merge whose peer never publishes gives up after its time limit, records
  the pipeline-timeout bit and writes nothing (a flag that nothing sets,
  bounded at 20 ms); the context stays usable.
* With one process and no process group the decoder's exchange runs its own
  protocol for real (its only flag is its own), eager and graph-replayed."""
import ctypes

import numpy as np
import pytest
import torch

import cases
from _refs import assert_decode_close, to_dev
from oracle import iris_oracle as orc

pytestmark = pytest.mark.gpu

FLAG, EPOCH, COUNT = 0, 8, 16  # header words (int64) of one exchange buffer


def _slot_floats(rows, d):
    return (rows * (d + 1) * 4 + 255) // 256 * 64


def _alloc(n, rows, d):
    from iris_kernel import _lib
    from iris_kernel.parallel import _device_floats

    nbytes = _lib.lib.iris_b200_xchg_buffer_bytes(rows, d)
    assert nbytes == _lib.XCHG_HEADER_BYTES + 2 * _slot_floats(rows, d) * 4
    bufs, slots, heads = [], [], []
    for _ in range(n):
        p = ctypes.c_void_p()
        assert _lib.lib.iris_b200_xchg_alloc(nbytes, ctypes.byref(p)) == 0
        bufs.append(p.value)
        whole = _device_floats(p.value + _lib.XCHG_HEADER_BYTES, 2 * _slot_floats(rows, d), torch.device("cuda"))
        slots.append([whole[k * _slot_floats(rows, d):k * _slot_floats(rows, d) + rows * (d + 1)] for k in (0, 1)])
        heads.append(_device_floats(p.value, _lib.XCHG_HEADER_BYTES // 4, torch.device("cuda")).view(torch.int64))
    return bufs, slots, heads


def _free(bufs):
    from iris_kernel import _lib

    torch.cuda.synchronize()
    for b in bufs:
        assert _lib.lib.iris_b200_xchg_free(b) == 0


def _partial(c, t, world, rank, query):
    """Rank ``rank``'s packed partial (O [B*Hq, D] then lse [B*Hq])."""
    from iris_kernel import parallel as P
    from iris_kernel.fused_attention import decode_partial

    B, Hq, D = query.shape
    plan = P.plan_split_context(c["seq_lens"], world, rank, split_tokens=256)
    if len(plan.seqs):
        idx = torch.from_numpy(plan.seqs).cuda()
        o, lse = decode_partial(query.index_select(0, idx).contiguous(), t["k_data"], t["v_data"], t["k_scale"],
                                t["v_scale"], P.local_block_table(plan, t["block_table"]),
                                torch.from_numpy(plan.lens.astype(np.int32)).cuda())
    else:
        o, lse = torch.zeros(0, Hq, D, device="cuda"), torch.zeros(0, Hq, device="cuda")
    return P.pack_partials(o, lse, plan.seqs, B)


def _merge(bufs, rank, rows, d, part, out, err, limit_ns):
    from iris_kernel import _lib

    arr = (ctypes.c_void_p * len(bufs))(*bufs)
    n = rows * d
    return _lib.lib.iris_b200_xchg_merge(arr, len(bufs), rank, rows, d, part[:n].data_ptr(), part[n:].data_ptr(),
                                         out.data_ptr(), err.data_ptr(), limit_ns,
                                         torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_merge_matches_oracle_two_steps(world):
    c = cases.decode_random(seed=400 + world, B=6, Hq=32, Hkv=8, D=128, lens=[1000, 1, 333, 16, 2049, 700])
    t = to_dev(c, cases.DECODE_KEYS)
    B, Hq, D = t["query"].shape
    rows = B * Hq
    bufs, slots, heads = _alloc(world, rows, D)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        for e in (1, 2):
            q = t["query"] if e == 1 else (t["query"].float() * -0.7).half()
            parts = [_partial(c, t, world, r, q) for r in range(world)]
            cc = dict(c)
            cc["query"] = q.cpu().numpy()
            ref = orc.decode_attention(*[cc[k] for k in cases.DECODE_KEYS])
            torch.cuda.synchronize()
            for r in range(world):  # what every rank's merge publishes at step e
                slots[r][e & 1].copy_(parts[r])
                heads[r][FLAG] = e
            for r in range(world):
                out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device="cuda")
                assert _merge(bufs, r, rows, D, parts[r], out, err, 2_000_000_000) == 0
                torch.cuda.synchronize()
                assert int(err.item()) == 0
                assert_decode_close(out, ref)
                assert int(heads[r][EPOCH]) == e and int(heads[r][FLAG]) == e
                assert int(heads[r][COUNT]) & 0xFFFFFFFF == 0  # arrivals reset for the next step
                assert torch.equal(slots[r][e & 1], parts[r])  # the merge published this rank's partial
    finally:
        del slots, heads
        _free(bufs)


def test_exchange_merge_times_out_when_a_peer_never_arrives():
    from iris_kernel import _lib
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    c = cases.decode_random(seed=410, B=2, Hq=8, Hkv=2, D=64, lens=[100, 40])
    t = to_dev(c, cases.DECODE_KEYS)
    B, Hq, D = t["query"].shape
    bufs, slots, heads = _alloc(2, B * Hq, D)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    try:
        part = _partial(c, t, 2, 0, t["query"])
        torch.cuda.synchronize()
        # rank 1 never publishes: rank 0 publishes, then gives up before merging
        out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device="cuda")
        assert _merge(bufs, 0, B * Hq, D, part, out, err, 20_000_000) == 0  # 20 ms limit
        torch.cuda.synchronize()
        assert int(err.item()) & _lib.ERR_PIPELINE_TIMEOUT
        assert bool(torch.isnan(out).all())  # nothing written
        assert int(heads[0][FLAG]) == 1 and int(heads[1][FLAG]) == 0
        # the context is still usable: a regular decode right after is correct
        got = fused_int4_paged_decode_attention(*[t[k] for k in cases.DECODE_KEYS])
        torch.cuda.synchronize()
        assert_decode_close(got, ref)
    finally:
        del slots, heads
        _free(bufs)


def test_single_gpu_decoder_over_the_exchange_eager_and_graph():
    """One process, no process group: the exchange's own protocol end to end
    on one GPU (its only flag is its own), eager and then replayed from a
    CUDA graph over several steps, so both slots alternate; every output
    equals the FP32 oracle."""
    import iris_kernel
    from iris_kernel import parallel as P

    c = cases.decode_random(seed=420, B=4, Hq=32, Hkv=8, D=128, lens=[700, 1, 2049, 300])
    t = to_dev(c, cases.DECODE_KEYS)
    B, Hq, D = t["query"].shape
    ref = orc.decode_attention(*[c[k] for k in cases.DECODE_KEYS])
    plan = P.plan_split_context(c["seq_lens"], 1, 0, split_tokens=256)
    dec = P.SplitContextDecoder(plan, t["block_table"], Hq, D, transport="p2p")
    try:
        for _ in range(3):
            out = dec(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"]).clone()
            torch.cuda.synchronize()
            assert_decode_close(out, ref)
        iris_kernel.set_validation_mode("deferred")
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                dec(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                res = dec(t["query"], t["k_data"], t["v_data"], t["k_scale"], t["v_scale"])
            for _ in range(3):
                res.zero_()
                g.replay()
                torch.cuda.synchronize()
                iris_kernel.check_errors()
                assert_decode_close(res, ref)
            del g
        finally:
            iris_kernel.set_validation_mode("sync")
    finally:
        dec.close()
