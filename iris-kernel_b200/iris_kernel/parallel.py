"""Decode over several GPUs, one process per GPU.

The reference runs on one GPU only; these are the two ways this package
spreads a decode batch over N GPUs of a node (torch.distributed, NCCL):

* Sequence sharding (no collective).  Every GPU owns whole sequences: their
  pages live in its own cache and it decodes them with
  ``fused_int4_paged_decode_attention``; outputs stay where their sequences
  live.  :func:`balance_sequences` assigns sequences to GPUs greedily,
  longest first, by token count (the decode's cost is proportional to the
  tokens read, not to the number of sequences).

* Split-context (one exchange of partials).  Every sequence's context is cut into
  page-aligned splits of ``split_tokens`` tokens and the splits are dealt out
  to the GPUs (:func:`plan_split_context`); a GPU's cache holds the pages of
  its own splits.  Each GPU runs one log-sum-exp-form decode over the tokens
  it holds, packs ``(O, lse)`` into one buffer, exchanges it, and merges the
  N partials (:func:`split_context_decode`, :class:`SplitContextDecoder`).  A GPU's splits of one sequence
  are handed to the kernel as a single virtual sequence: attention does not
  depend on the order of the tokens, and only a sequence's final split can end
  in a partly filled page, which the concatenation keeps last.

Nothing here moves KV pages between GPUs; remote data arrives only as the
partials.  Two transports carry them:

* ``"nccl"``: one ``all_gather_into_tensor`` of the packed partials, then
  the merge kernel;
* ``"p2p"`` (:class:`PeerExchange`): one kernel per GPU and step publishes
  its partial in a buffer the other GPUs have mapped (CUDA IPC; two slots
  used on alternate steps) and merges every partial read from its owner's
  memory over NVLink, with bounded waits on per-GPU step flags
  (``iris_b200_xchg_*``).  Faster than the all-gather: config 4 at 8 GPUs
  takes 99.8 us per step against 117.0 us.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, _runtime
from .fused_attention import decode_partial, merge_lse_packed


def balance_sequences(seq_lens, world: int) -> list[list[int]]:
    """Assign sequence indices to ``world`` GPUs, longest first, each to the
    GPU with the fewest tokens so far (ties: lowest rank).  Every GPU's list
    is returned in ascending order."""
    if world <= 0:
        raise ValueError("world must be positive")
    lens = np.asarray(seq_lens, dtype=np.int64).reshape(-1)
    load = np.zeros(world, dtype=np.int64)
    owned: list[list[int]] = [[] for _ in range(world)]
    for b in np.argsort(-lens, kind="stable"):
        g = int(np.argmin(load))
        owned[g].append(int(b))
        load[g] += lens[b]
    return [sorted(o) for o in owned]


@dataclass
class SplitPlan:
    """What one GPU decodes in split-context mode.

    ``seqs [Bl]``: global indices of the sequences this GPU holds tokens of
    (ascending).  ``cols [Bl, W]``: for each of them the block-table columns
    (page numbers within the sequence) of this GPU's splits, concatenated in
    split order; entries past ``ceil(lens/page_size)`` are padding (column 0)
    and never read.  ``lens [Bl]``: tokens this GPU holds per sequence.
    ``batch``: the global batch size."""

    rank: int
    world: int
    batch: int
    seqs: np.ndarray
    cols: np.ndarray
    lens: np.ndarray

    @property
    def covers_every_sequence(self) -> bool:
        return len(self.seqs) == self.batch


def split_owner(seq: int, split: int, num_splits: int, world: int, mode: str) -> int:
    """GPU that decodes split ``split`` (of ``num_splits``) of sequence ``seq``.

    ``"strided"``: splits are dealt round-robin, starting one GPU further for
    each sequence so that short sequences do not all land on GPU 0.
    ``"contiguous"``: each GPU takes one contiguous block of a sequence's
    splits (GPU g: splits [g*n/N, (g+1)*n/N))."""
    if mode == "strided":
        return (split + seq) % world
    if mode == "contiguous":
        return split * world // num_splits
    raise ValueError(f"unknown split mode {mode!r}")


def plan_split_context(seq_lens, world: int, rank: int, *, split_tokens: int = 8192, page_size: int = 16,
                       mode: str = "strided") -> SplitPlan:
    """The split-context plan of GPU ``rank`` for host-side ``seq_lens``."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if split_tokens <= 0 or split_tokens % page_size:
        raise ValueError("split_tokens must be a positive multiple of page_size")
    lens = np.asarray(seq_lens, dtype=np.int64).reshape(-1)
    if (lens <= 0).any():
        raise ValueError("seq_lens must be positive")
    pages_per_split = split_tokens // page_size
    seqs, cols, counts = [], [], []
    for b, L in enumerate(lens.tolist()):
        n = -(-L // split_tokens)
        mine = [j for j in range(n) if split_owner(b, j, n, world, mode) == rank]
        if not mine:
            continue
        c = []
        tokens = 0
        for j in mine:
            t0, t1 = j * split_tokens, min((j + 1) * split_tokens, L)
            tokens += t1 - t0
            c.append(np.arange(j * pages_per_split, j * pages_per_split + -(-(t1 - t0) // page_size)))
        seqs.append(b)
        cols.append(np.concatenate(c))
        counts.append(tokens)
    width = max((len(c) for c in cols), default=1)
    table = np.zeros((len(cols), width), dtype=np.int64)
    for i, c in enumerate(cols):
        table[i, :len(c)] = c
    return SplitPlan(rank, world, len(lens), np.asarray(seqs, dtype=np.int64), table,
                     np.asarray(counts, dtype=np.int64))


def local_block_table(plan: SplitPlan, block_table: torch.Tensor) -> torch.Tensor:
    """This GPU's block table: row i lists the page ids of ``plan.seqs[i]``'s
    local splits (gathered on the block table's device)."""
    dev = block_table.device
    if len(plan.seqs) == 0:
        return torch.zeros((0, 1), dtype=block_table.dtype, device=dev)
    rows = block_table.index_select(0, torch.from_numpy(plan.seqs).to(dev))
    return torch.gather(rows, 1, torch.from_numpy(plan.cols).to(dev)).contiguous()


def packed_size(batch: int, num_q_heads: int, head_dim: int) -> int:
    """Floats in one GPU's packed partial: O [B, Hq, D] then lse [B, Hq]."""
    return batch * num_q_heads * (head_dim + 1)


def packed_views(buf: torch.Tensor, batch: int, num_q_heads: int, head_dim: int):
    """``(o [B, Hq, D], lse [B, Hq])`` views of one packed partial."""
    n = batch * num_q_heads * head_dim
    return buf[:n].view(batch, num_q_heads, head_dim), buf[n:n + batch * num_q_heads].view(batch, num_q_heads)


def pack_partials(o_local: torch.Tensor, lse_local: torch.Tensor, seqs, batch: int) -> torch.Tensor:
    """Pack this GPU's partials of sequences ``seqs`` into a full-batch buffer;
    sequences it holds no tokens of get lse = -inf (and O = 0)."""
    _, hq, d = o_local.shape
    buf = torch.zeros(packed_size(batch, hq, d), dtype=torch.float32, device=o_local.device)
    o, lse = packed_views(buf, batch, hq, d)
    lse.fill_(float("-inf"))
    idx = torch.as_tensor(np.asarray(seqs, dtype=np.int64), device=o_local.device)
    if idx.numel():
        o.index_copy_(0, idx, o_local)
        lse.index_copy_(0, idx, lse_local)
    return buf


def _device_floats(ptr: int, n: int, device: torch.device) -> torch.Tensor:
    """A float32 tensor of ``n`` elements over device memory the library
    allocated (no copy; the caller keeps the memory alive)."""

    class _Mem:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                    "strides": None}

    with torch.cuda.device(device):
        return torch.as_tensor(_Mem(), device=device)


class PeerExchange:
    """Split-context merge over NVLink peer memory for one GPU of a process
    group: an exchange buffer on this GPU, mapped by every other GPU of the
    group (CUDA IPC handles swapped over the group once), and the mapped
    addresses of theirs.  Per step every GPU calls :meth:`merge` with its
    LSE-form partial (``o [rows, D]``, ``lse [rows]`` fp32): one kernel
    publishes it in this GPU's buffer and merges every GPU's (CUDA-graph
    capturable; two slots on alternate steps, so no step waits for the
    others to finish reading).  A GPU that does not arrive within
    ``limit_s`` makes the merge record a pipeline timeout (raised as
    RuntimeError) instead of waiting forever; the exchange must then be
    rebuilt.  Call :meth:`close` on every GPU (it synchronises the group)
    before destroying the process group."""

    def __init__(self, rows: int, head_dim: int, *, group=None, limit_s: float = 2.0):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows, self.head_dim = rows, head_dim
        self.limit_ns = int(limit_s * 1e9)
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib
        nbytes = lib.iris_b200_xchg_buffer_bytes(rows, head_dim)
        if nbytes == 0:
            raise ValueError("exchange buffer: rows > 0 and head_dim a multiple of 4 required")
        buf = ctypes.c_void_p()
        _lib.check_status(lib.iris_b200_xchg_alloc(nbytes, ctypes.byref(buf)), "iris_b200_xchg_alloc")
        self.buf = buf.value
        self.peers: list[int] = []
        ptrs = []
        if self.world > 1:
            handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
            _lib.check_status(lib.iris_b200_ipc_export(self.buf, ctypes.addressof(handle)), "iris_b200_ipc_export")
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            for k, h in enumerate(handles):
                if k == self.rank:
                    ptrs.append(self.buf)
                    continue
                hb = (ctypes.c_char * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
                p = ctypes.c_void_p()
                _lib.check_status(lib.iris_b200_ipc_open(ctypes.addressof(hb), ctypes.byref(p)), "iris_b200_ipc_open")
                self.peers.append(p.value)
                ptrs.append(p.value)
        else:
            ptrs.append(self.buf)
        self.bufs = (ctypes.c_void_p * self.world)(*ptrs)

    def merge(self, output: torch.Tensor, o: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
        """Publish this GPU's partial of the step (``o [rows, D]``, ``lse
        [rows]`` fp32, contiguous, written earlier on the current stream) and
        merge every GPU's into ``output [rows, D]`` fp16."""
        word = _runtime.error_word(self.device)
        _lib.check_status(
            _lib.lib.iris_b200_xchg_merge(self.bufs, self.world, self.rank, self.rows, self.head_dim, o.data_ptr(),
                                          lse.data_ptr(), output.data_ptr(), word.data_ptr(), self.limit_ns,
                                          _runtime.stream_ptr(self.device)),
            "iris_b200_xchg_merge")
        if _runtime.validation_mode() == "sync":
            _runtime.raise_for_bits(_runtime.read_and_clear(word))
        return output

    def close(self) -> None:
        import torch.distributed as dist

        if self.buf is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self.peers:
            _lib.lib.iris_b200_ipc_close(p)
        self.peers = []
        if self.world > 1:
            dist.barrier(group=self.group)  # no GPU still maps this buffer
        _lib.lib.iris_b200_xchg_free(self.buf)
        self.buf = None


class SplitContextDecoder:
    """Split-context decode for one GPU's plan, with everything that does not
    change between steps (the local block table, the token counts, the
    exchange buffers) prepared once, so that a CUDA graph can capture a step.
    With ``transport="nccl"`` a step is the LSE decode, one all-gather and
    the merge kernel; with ``"p2p"`` the decode writes into the
    :class:`PeerExchange` buffer and one merge kernel reads the other GPUs'
    partials over NVLink (call :meth:`close` on every GPU before the process
    group goes).

    ``block_table`` maps this GPU's splits to pages of its own cache; entries
    of other GPUs' splits are not read."""

    def __init__(self, plan: SplitPlan, block_table: torch.Tensor, num_q_heads: int, head_dim: int, *, group=None,
                 page_size: int = 16, group_size: int = 32, softmax_scale=None, transport: str = "nccl"):
        import torch.distributed as dist

        self.plan, self.group = plan, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if plan.world != self.world:
            raise ValueError("plan does not match the process group")
        dev = block_table.device
        self.hq, self.d = num_q_heads, head_dim
        self.kw = dict(page_size=page_size, group_size=group_size, softmax_scale=softmax_scale)
        self.local_bt = local_block_table(plan, block_table)
        self.lens = torch.from_numpy(plan.lens.astype(np.int32)).to(dev)
        self.idx = torch.from_numpy(plan.seqs).to(dev)
        if transport not in ("nccl", "p2p"):
            raise ValueError("transport must be 'nccl' or 'p2p'")
        self.transport = transport
        n = packed_size(plan.batch, num_q_heads, head_dim)
        if transport == "p2p":
            self.xchg = PeerExchange(plan.batch * num_q_heads, head_dim, group=group)
            self.send, self.recv = torch.zeros(n, dtype=torch.float32, device=dev), None
        else:
            self.xchg = None
            self.send = torch.zeros(n, dtype=torch.float32, device=dev)
            self.recv = torch.empty(self.world * n, dtype=torch.float32, device=dev)
        self.output = torch.empty((plan.batch, num_q_heads, head_dim), dtype=torch.float16, device=dev)
        o, lse = packed_views(self.send, plan.batch, num_q_heads, head_dim)
        o.zero_()
        lse.fill_(float("-inf"))  # sequences without local tokens keep lse = -inf
        self._o, self._lse = o, lse
        m = len(plan.seqs)
        self._o_l = torch.empty((m, num_q_heads, head_dim), dtype=torch.float32, device=dev)
        self._lse_l = torch.empty((m, num_q_heads), dtype=torch.float32, device=dev)

    def close(self) -> None:
        """Release the peer exchange (every GPU of the group must call it)."""
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None

    def __call__(self, query, k_data, v_data, k_scale, v_scale) -> torch.Tensor:
        import torch.distributed as dist

        plan = self.plan
        if query.shape != (plan.batch, self.hq, self.d):
            raise ValueError("query does not match the plan")
        if len(plan.seqs):
            if plan.covers_every_sequence:
                decode_partial(query, k_data, v_data, k_scale, v_scale, self.local_bt, self.lens, out=self._o,
                               lse=self._lse, **self.kw)
            else:
                decode_partial(query.index_select(0, self.idx), k_data, v_data, k_scale, v_scale, self.local_bt,
                               self.lens, out=self._o_l, lse=self._lse_l, **self.kw)
                self._o.index_copy_(0, self.idx, self._o_l)
                self._lse.index_copy_(0, self.idx, self._lse_l)
        if self.xchg is not None:
            self.xchg.merge(self.output.view(-1, self.d), self._o.view(-1, self.d), self._lse.view(-1))
            return self.output
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
            parts = self.recv
        else:
            parts = self.send
        return merge_lse_packed(parts, self.world, plan.batch, self.hq, self.d, self.output)


def split_context_decode(query, k_data, v_data, k_scale, v_scale, block_table, plan: SplitPlan, *,
                         group=None, page_size: int = 16, group_size: int = 32, softmax_scale=None,
                         output: torch.Tensor | None = None) -> torch.Tensor:
    """Split-context decode on this GPU, then all-gather + merge.

    ``query [B, Hq, D]`` is the full batch (identical on every GPU);
    ``block_table`` maps this GPU's splits to pages of its own cache
    (``k_data`` ... ``v_scale``); entries of other GPUs' splits are not read.
    Every GPU of ``group`` must call this with the same B, Hq, D.  Returns the
    fp16 output ``[B, Hq, D]`` (the same on every GPU)."""
    import torch.distributed as dist

    batch, hq, d = query.shape
    world = dist.get_world_size(group)
    if plan.world != world or plan.batch != batch:
        raise ValueError("plan does not match the process group or the batch")
    dev = query.device
    kw = dict(page_size=page_size, group_size=group_size, softmax_scale=softmax_scale)
    if plan.covers_every_sequence:
        # the decode writes straight into the send buffer
        send = torch.empty(packed_size(batch, hq, d), dtype=torch.float32, device=dev)
        o, lse = packed_views(send, batch, hq, d)
        lens = torch.from_numpy(plan.lens.astype(np.int32)).to(dev)
        decode_partial(query, k_data, v_data, k_scale, v_scale, local_block_table(plan, block_table), lens, out=o,
                       lse=lse, **kw)
    elif len(plan.seqs):
        idx = torch.from_numpy(plan.seqs).to(dev)
        lens = torch.from_numpy(plan.lens.astype(np.int32)).to(dev)
        o_l, lse_l = decode_partial(query.index_select(0, idx).contiguous(), k_data, v_data, k_scale, v_scale,
                                    local_block_table(plan, block_table), lens, **kw)
        send = pack_partials(o_l, lse_l, plan.seqs, batch)
    else:
        send = pack_partials(query.new_empty((0, hq, d), dtype=torch.float32),
                             query.new_empty((0, hq), dtype=torch.float32), plan.seqs, batch)
    recv = torch.empty(world * send.numel(), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(recv, send, group=group)
    return merge_lse_packed(recv, world, batch, hq, d, output)
