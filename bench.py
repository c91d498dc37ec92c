"""Benchmark of the INT4 paged KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--only all|c2|c3|c4|c5a|c5b|f16|next|sweep] [--no-cpu-baseline]

Workload (Llama-3-8B shape): 64 sequences x 4096 tokens
of INT4 paged cache (Hq=32, Hkv=8, D=128, page 16, group 32, pages scattered
by a random permutation; K/V ~N(0,1) fp16 with 4 outlier K channels x8,
written by the fused append), then per step

    decode attention over the 4096 cached tokens of every sequence, and
    a batched 1-token fused RoPE+INT4 append per sequence at position 4096
    (the next step's token; the decode does not read it, so the step's graph
    runs the append beside the decode rather than after it).

One process per GPU (torchrun for N > 1).  The 64 sequences are sharded
64/N per GPU (sequence sharding: no collective), so the total work is fixed
and ``scaling`` is "strong"; ``value`` is the whole batch's algorithmic bytes
/ the max-over-ranks step time.

``value``: algorithmic bytes of the step (KV pages + scales read once, query
read, output written, block table; append: fp16 K/V read, packed bytes and
scales written, slots/positions and one RoPE row) / step time, in TB/s, with
inputs resident in HBM; the step is replayed from a CUDA graph (validation in
deferred mode, no host syncs).  Inputs (303 MB per step at N=1) exceed
twice the 126 MB L2, so no flush is needed between steps.  A GPU whose share
is under twice the L2 (config 2 at N >= 2, config 3 at N = 8, config 5a)
times its steps one by one, each after a 256 MB write and a 256 MB read of
another buffer that evict the L2 (the read leaves clean lines behind).
``e2e``: the same metric through the public Python API with host buffers:
per step the new query / K / V / positions / slots are copied from pinned
host memory, the decode and append calls run, the fp16 output is copied
back and the step's error word is read on the host.  The query copy comes
first and the decode starts as soon as it lands; the K/V copy and the
append run on a second stream meanwhile.

Also reported: config 5b prefill append, config 5a decode-style append,
config 4 split-context decode over the ranks (merged over NVLink peer memory
at N > 1, the NCCL all-gather path timed beside it,
with a per-stage breakdown and an FP32 parity self-check on two sequences),
config 3 sequence-sharded decode, and the matched FP16 decode.

``--only sweep`` (one GPU) prints the reference benchmarks' tables instead:
INT4 vs matched FP16 decode over L in (128, 512, 2048, 4096) at batch 1 with
the output cosine and RMSE, and the append over T in (1, 8, 32, 128), each
beside the reference's torch eager code on the same GPU.

``--impl reference`` times the reference's own CPU path (its torch eager
``torch_eager_int4_paged_decode_attention`` + ``torch_eager_append``, from
the unmodified install in ``baseline/_ref``) on the same workload, rank 0
only, every step a measured step.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "iris-kernel_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, L, HQ, HKV, D, P, G = 64, 4096, 32, 8, 128, 16, 32
OUTLIER_CH = (3, 40, 77, 121)
SPEC_TBS = 8.0


def decode_bytes(nseq, ctx=L, hq=HQ, hkv=HKV, d=D):
    """KV pages + scales read once, Q read, O written, block table read."""
    return nseq * ctx * hkv * (d + d // 8) + 2 * nseq * hq * d * 2 + nseq * (ctx // P + 1) * 4


def append_bytes(tokens, hkv=HKV, d=D, rope_rows=1):
    """fp16 K and V read, packed bytes + scales written, slot + position, RoPE rows."""
    return tokens * hkv * (4 * d + d + d // 8) + tokens * 8 + rope_rows * 2 * (d // 2) * 2


DECODE_BYTES = decode_bytes(B)
APPEND_BYTES = append_bytes(B)
STEP_BYTES = DECODE_BYTES + APPEND_BYTES
FP16_BYTES = B * L * HKV * D * 2 * 2 + 2 * B * HQ * D * 2 + B * (L // P + 1) * 4

# BASELINE config 5a: decode-style append, 2048 sequences x 1 token, Hkv 1, D 128, positions
# ~U[0, 32768), RoPE base 500000, scattered pages.
A5_T, A5_MAXPOS = 2048, 32768
A5_BYTES = A5_T * (4 * D + D + D // 8) + A5_T * 8 + A5_T * 2 * (D // 2) * 2
# BASELINE config 5b: prefill-style append, 8 sequences x 8192 new tokens, Hkv 8, D 128, fresh
# permuted pages, 1% of entries x20, RoPE base 500000.
PF_S, PF_L = 8, 8192
PF_BYTES = PF_S * PF_L * HKV * (4 * D + D + D // 8) + PF_S * PF_L * 8 + PF_L * 2 * (D // 2) * 2
# BASELINE config 4 (70B-shaped long context): 16 sequences x 131,072 tokens, Hq 64, Hkv 8, D 128;
# split-context over the ranks in 8192-token splits, every rank's cache holding only its splits;
# one NCCL all-gather + merge.
C4_B, C4_L, C4_HQ, C4_HKV, C4_SPLIT = 16, 131072, 64, 8, 8192
C4_BYTES = C4_B * C4_L * C4_HKV * (D + D // 8) + 2 * C4_B * C4_HQ * D * 2 + C4_B * (C4_L // P) * 4 + C4_B * 4
C4_CHECK_SEQS = 2  # sequences the FP32 self-check covers
# BASELINE config 3 (MHA, D 64, varlen): 128 sequences, Hq = Hkv = 16, L ~ U[1, 16384] (seed 1);
# whole sequences sharded over the ranks by token count.
C3_B, C3_H, C3_D, C3_LMAX = 128, 16, 64, 16384


def rope_tables(max_pos, dim, dev, base=10000.0):
    """fp16 cos/sin tables [max_pos, dim/2] (NeoX rotation, angles in fp32)."""
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32, device=dev) / dim))
    f = torch.arange(max_pos, dtype=torch.float32, device=dev)[:, None] * inv[None, :]
    return f.cos().half().contiguous(), f.sin().half().contiguous()


def shard(world, rank, n=B):
    """Sequences [lo, hi) of the config-2 batch that rank owns."""
    return rank * n // world, (rank + 1) * n // world


# ----------------------------------------------------------------- workloads

def _fill_cache(dev, g, kd, vd, ks, vs, slots, positions, hkv, d, cos, sin, chunk=65536, std=0.5):
    """Write synthetic K/V ~ N(0, std) through the fused append, in chunks."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    for t0 in range(0, slots.numel(), chunk):
        t1 = min(slots.numel(), t0 + chunk)
        k = (torch.randn(t1 - t0, hkv, d, generator=g, device=dev) * std).half()
        v = (torch.randn(t1 - t0, hkv, d, generator=g, device=dev) * std).half()
        fused_rope_int4_paged_append(k, v, positions[t0:t1].contiguous(), slots[t0:t1].contiguous(), cos, sin,
                                     kd, vd, ks, vs, rotary_dim=d, page_size=P)


def build_c2(dev, seed, nseq):
    """This rank's shard of config 2: nseq sequences of 4096 cached tokens
    (257 pages each: the 1-token append at position 4096 needs one more)."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    g = torch.Generator(device=dev).manual_seed(seed)
    pool = nseq * (L // P + 1)
    bt = torch.randperm(pool, generator=g, device=dev).int().view(nseq, L // P + 1).contiguous()
    kd = torch.zeros(pool, P, HKV, D // 2, dtype=torch.uint8, device=dev)
    vd = torch.zeros_like(kd)
    ks = torch.zeros(pool, P, HKV, D // G, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    cos, sin = rope_tables(L + 1, D, dev)
    pos = torch.arange(L, device=dev, dtype=torch.int32)
    for b in range(nseq):
        k = torch.randn(L, HKV, D, generator=g, device=dev)
        k[..., list(OUTLIER_CH)] *= 8
        v = torch.randn(L, HKV, D, generator=g, device=dev)
        slots = (bt[b, (pos // P).long()] * P + pos % P).int()
        fused_rope_int4_paged_append(k.half(), v.half(), pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                     page_size=P)
    q = torch.randn(nseq, HQ, D, generator=g, device=dev).half()
    knew = torch.randn(nseq, HKV, D, generator=g, device=dev)
    knew[..., list(OUTLIER_CH)] *= 8
    vnew = torch.randn(nseq, HKV, D, generator=g, device=dev)
    w = dict(q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt, cos=cos, sin=sin,
             lens=torch.full((nseq,), L, dtype=torch.int32, device=dev),
             knew=knew.half(), vnew=vnew.half(), newpos=torch.full((nseq,), L, dtype=torch.int32, device=dev),
             newslot=(bt[:, L // P] * P).int().contiguous(),
             out=torch.empty(nseq, HQ, D, dtype=torch.float16, device=dev))
    torch.cuda.synchronize(dev)
    return w


def build_prefill(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    T = PF_S * PF_L
    k = torch.randn(T, HKV, D, generator=g, device=dev)
    v = torch.randn(T, HKV, D, generator=g, device=dev)
    k[torch.rand(k.shape, generator=g, device=dev) < 0.01] *= 20
    v[torch.rand(v.shape, generator=g, device=dev) < 0.01] *= 20
    npages = T // P
    pages = torch.randperm(npages, generator=g, device=dev).view(PF_S, PF_L // P)
    pos = torch.arange(PF_L, device=dev, dtype=torch.int32).repeat(PF_S)
    slots = (pages.repeat_interleave(P, dim=1) * P + torch.arange(PF_L, device=dev) % P).view(-1).int()
    cos, sin = rope_tables(PF_L, D, dev, 500000.0)
    return dict(k=k.half(), v=v.half(), pos=pos, slots=slots.contiguous(), cos=cos, sin=sin,
                kd=torch.zeros(npages, P, HKV, D // 2, dtype=torch.uint8, device=dev),
                vd=torch.zeros(npages, P, HKV, D // 2, dtype=torch.uint8, device=dev),
                ks=torch.zeros(npages, P, HKV, D // G, dtype=torch.float16, device=dev),
                vs=torch.zeros(npages, P, HKV, D // G, dtype=torch.float16, device=dev))


def build_c5a(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(A5_T, 1, D, generator=g, device=dev)
    v = torch.randn(A5_T, 1, D, generator=g, device=dev)
    k[torch.rand(k.shape, generator=g, device=dev) < 0.01] *= 20
    v[torch.rand(v.shape, generator=g, device=dev) < 0.01] *= 20
    npages = 2 * A5_T
    pages = torch.randperm(npages, generator=g, device=dev)[:A5_T]
    slots = (pages * P + torch.randint(0, P, (A5_T,), generator=g, device=dev)).int()
    pos = torch.randint(0, A5_MAXPOS, (A5_T,), generator=g, device=dev).int()
    cos, sin = rope_tables(A5_MAXPOS, D, dev, 500000.0)
    return dict(k=k.half(), v=v.half(), pos=pos, slots=slots, cos=cos, sin=sin,
                kd=torch.zeros(npages, P, 1, D // 2, dtype=torch.uint8, device=dev),
                vd=torch.zeros(npages, P, 1, D // 2, dtype=torch.uint8, device=dev),
                ks=torch.zeros(npages, P, 1, D // G, dtype=torch.float16, device=dev),
                vs=torch.zeros(npages, P, 1, D // G, dtype=torch.float16, device=dev))


def build_c4(dev, rank, world, seed):
    """This rank's share of config 4: only the pages of its splits exist in
    its cache; the block table maps its split columns to them."""
    from iris_kernel import parallel

    plan = parallel.plan_split_context([C4_L] * C4_B, world, rank, split_tokens=C4_SPLIT)
    g = torch.Generator(device=dev).manual_seed(seed)
    n_local = int(sum(-(-int(x) // P) for x in plan.lens))
    perm = torch.randperm(n_local, generator=g, device=dev).int()
    bt = torch.zeros(C4_B, C4_L // P, dtype=torch.int32, device=dev)
    cols = torch.from_numpy(plan.cols).to(dev)
    npg = torch.from_numpy((plan.lens + P - 1) // P).to(dev)
    off = 0
    slot_l, pos_l = [], []
    for i, b in enumerate(plan.seqs.tolist()):
        n = int(npg[i])
        pages = perm[off:off + n]
        bt[b, cols[i, :n]] = pages
        tok = (cols[i, :n].int()[:, None] * P + torch.arange(P, device=dev, dtype=torch.int32)).reshape(-1)
        slot_l.append((pages[:, None] * P + torch.arange(P, device=dev, dtype=torch.int32)).reshape(-1))
        pos_l.append(tok)
        off += n
    kd = torch.zeros(n_local, P, C4_HKV, D // 2, dtype=torch.uint8, device=dev)
    vd = torch.zeros_like(kd)
    ks = torch.zeros(n_local, P, C4_HKV, D // G, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    cos, sin = rope_tables(C4_L, D, dev, 500000.0)
    _fill_cache(dev, g, kd, vd, ks, vs, torch.cat(slot_l), torch.cat(pos_l), C4_HKV, D, cos, sin)
    q = torch.randn(C4_B, C4_HQ, D, generator=torch.Generator(device=dev).manual_seed(4), device=dev).half()
    return dict(plan=plan, q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt)


def build_c3(dev, rank, world, seed):
    """This rank's shard of config 3 (whole sequences, balanced by tokens)."""
    from iris_kernel import parallel

    lens_all = np.random.default_rng(1).integers(1, C3_LMAX + 1, size=C3_B)
    mine = parallel.balance_sequences(lens_all, world)[rank]
    lens = lens_all[mine]
    g = torch.Generator(device=dev).manual_seed(seed)
    npg = (lens + P - 1) // P
    pool = int(npg.sum())
    perm = torch.randperm(pool, generator=g, device=dev).int()
    width = int(npg.max())
    bt = torch.zeros(len(mine), width, dtype=torch.int32, device=dev)
    off = 0
    slot_l, pos_l = [], []
    for i, L_ in enumerate(lens.tolist()):
        n = int(npg[i])
        pages = perm[off:off + n]
        bt[i, :n] = pages
        slot_l.append((pages[:, None] * P + torch.arange(P, device=dev, dtype=torch.int32)).reshape(-1)[:L_])
        pos_l.append(torch.arange(L_, device=dev, dtype=torch.int32))
        off += n
    kd = torch.zeros(pool, P, C3_H, C3_D // 2, dtype=torch.uint8, device=dev)
    vd = torch.zeros_like(kd)
    ks = torch.zeros(pool, P, C3_H, C3_D // G, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    cos, sin = rope_tables(C3_LMAX, C3_D, dev)
    _fill_cache(dev, g, kd, vd, ks, vs, torch.cat(slot_l), torch.cat(pos_l), C3_H, C3_D, cos, sin, std=1.0)
    q = torch.randn(len(mine), C3_H, C3_D, generator=g, device=dev).half()
    nbytes = int(lens.sum()) * C3_H * (C3_D + C3_D // 8) + 2 * len(mine) * C3_H * C3_D * 2 + int(npg.sum()) * 4
    total = int(lens_all.sum()) * C3_H * (C3_D + C3_D // 8) + 2 * C3_B * C3_H * C3_D * 2 + int(
        ((lens_all + P - 1) // P).sum()) * 4
    return dict(q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt,
                lens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                out=torch.empty_like(q), bytes=nbytes, total_bytes=total)


# ------------------------------------------------------------------ timing

def _peak_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _dist():
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        return dist, dist.get_rank(), dist.get_world_size(), local
    return None, 0, 1, 0


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while running
    (samples go to a temporary file)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"iris_clocks_{index}_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            t0 = time.time()  # start timing only once samples are flowing
            while time.time() - t0 < 10 and os.path.getsize(self.path) == 0:
                time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
                except ValueError:
                    continue
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


def graph_of(fn, dev):
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        fn()
    torch.cuda.synchronize(dev)
    return gr


L2_BYTES = 126 * 2**20
FLUSH_BYTES = 256 * 2**20


class L2Flush:
    """Evicts the L2 between timed steps: a 256 MB write (twice the L2), then
    a 256 MB read of another buffer, so that the L2 holds clean lines and the
    next step does not pay for writing the flush's dirty lines back."""

    def __init__(self, dev):
        self.buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.rd = torch.zeros(FLUSH_BYTES // 8, dtype=torch.int64, device=dev)

    def __call__(self):
        self.buf.zero_()
        self.rd.sum()


def needs_flush(step_bytes):
    """A step whose inputs on one GPU are under twice the L2 would find them
    there from the previous step: such steps are timed one by one with the
    L2 flushed in between."""
    return step_bytes < 2 * L2_BYTES


def timed(fn, steps, dev, dist, warmup, flush=None):
    """Warm up, barrier + sync, time exactly `steps` calls with CUDA events
    on the current stream, barrier + sync; returns ms for all steps.  With
    `flush`, every call (warm-up included) follows an L2 flush, and each call
    is timed between its own events, so the flushes are not counted."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        fn()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if flush is None:
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(steps):
            fn()
        en.record()
        torch.cuda.synchronize(dev)
        total = st.elapsed_time(en)
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for st, en in evs:
            flush()
            st.record()
            fn()
            en.record()
        torch.cuda.synchronize(dev)
        total = sum(st.elapsed_time(en) for st, en in evs)
    if dist is not None:
        dist.barrier()
    return total


def reduce_over_ranks(x, dist, dev, op="max"):
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


# ------------------------------------------------------- the reference's CPU path

def load_reference_eager():
    """The reference's eager modules from the unmodified install in
    baseline/_ref, loaded by file under private names (they import only
    torch and math), or None when the install is absent."""
    base = os.path.join(ROOT, "baseline", "_ref", "iris_kernel")
    mods = {}
    for name in ("torch_eager_attention", "torch_eager_kv"):
        path = os.path.join(base, name + ".py")
        if not os.path.isfile(path):
            return None
        spec = importlib.util.spec_from_file_location(f"_iris_reference_{name}", path)
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def _host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


class CpuStep:
    """Config 2 on the host for the reference's eager code: the whole cache
    (64 x 4096 tokens, random packed bytes and positive fp16 scales; the eager
    code's cost does not depend on the values), queries, and the new tokens.
    ``step(seqs)`` runs ``torch_eager_int4_paged_decode_attention`` over
    sequences [0, seqs) and ``torch_eager_append`` of their new tokens, and
    returns the algorithmic bytes it covered."""

    def __init__(self, ref):
        self.dec = ref["torch_eager_attention"].torch_eager_int4_paged_decode_attention
        self.app = ref["torch_eager_kv"].torch_eager_append
        g = torch.Generator().manual_seed(0)
        pool = B * (L // P + 1)
        self.kd = torch.randint(0, 256, (pool, P, HKV, D // 2), dtype=torch.uint8, generator=g)
        self.vd = torch.randint(0, 256, (pool, P, HKV, D // 2), dtype=torch.uint8, generator=g)
        self.ks = (torch.rand((pool, P, HKV, D // G), generator=g) * 0.99 + 0.01).half()
        self.vs = (torch.rand((pool, P, HKV, D // G), generator=g) * 0.99 + 0.01).half()
        self.bt = torch.randperm(pool, generator=g).int().view(B, L // P + 1).contiguous()
        self.lens = torch.full((B,), L, dtype=torch.int32)
        self.q = torch.randn(B, HQ, D, generator=g).half()
        self.knew = torch.randn(B, HKV, D, generator=g).half()
        self.vnew = torch.randn(B, HKV, D, generator=g).half()
        self.pos = torch.full((B,), L, dtype=torch.int32)
        self.slot = (self.bt[:, L // P] * P).int().contiguous()
        inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        f = torch.arange(L + 1, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = f.cos().half(), f.sin().half()

    def step(self, seqs):
        self.dec(self.q[:seqs], self.kd, self.vd, self.ks, self.vs, self.bt[:seqs], self.lens[:seqs],
                 page_size=P, group_size=G)
        self.app(self.knew[:seqs], self.vnew[:seqs], self.pos[:seqs], self.slot[:seqs], self.cos, self.sin,
                 self.kd, self.vd, self.ks, self.vs, rotary_dim=D, group_size=G, page_size=P)
        return decode_bytes(seqs) + append_bytes(seqs)


def cpu_baseline_sample(seconds_budget=15.0):
    """The reference's eager CPU path (or, without the install, the numpy
    port of it) on a bounded sample of the workload: repeated steps over 4 of
    the 64 sequences until the budget is used.  Returns the line's
    cpu_baseline object."""
    threads = _host_threads()
    torch.set_num_threads(threads)
    ref = load_reference_eager()
    if ref is not None:
        smp = CpuStep(ref)
        smp.step(1)  # first touch
        done, reps = 0, 0
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds_budget:
            done += smp.step(4)
            reps += 1
        dt = time.perf_counter() - t0
        return {"value": done / dt / 1e12, "unit": "TB/s", "cores": threads, "kind": "reference",
                "code": "torch_eager_int4_paged_decode_attention + torch_eager_append (baseline/_ref, unmodified)",
                "sample": f"{reps} x (decode of 4 of the 64 config-2 sequences x 4096 tokens + their 1-token "
                          f"appends), {dt:.1f} s", "cpu_model": _cpu_model(), "torch_threads": threads}
    sys.path.insert(0, ROOT)
    from oracle import iris_oracle as orc  # the numpy port, only when the reference is not installed

    rng = np.random.default_rng(0)
    nseq = 4
    nps = nseq * (L // P)
    kd = rng.integers(0, 256, (nps, P, HKV, D // 2), dtype=np.uint8)
    vd = rng.integers(0, 256, (nps, P, HKV, D // 2), dtype=np.uint8)
    ks = rng.uniform(0.01, 1, (nps, P, HKV, D // G)).astype(np.float16)
    vs = rng.uniform(0.01, 1, (nps, P, HKV, D // G)).astype(np.float16)
    bt = rng.permutation(nps).astype(np.int32).reshape(nseq, L // P)
    q = rng.standard_normal((nseq, HQ, D)).astype(np.float16)
    done, reps = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds_budget:
        orc.decode_attention(q, kd, vd, ks, vs, bt, np.full(nseq, L, np.int32))
        done += decode_bytes(nseq)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": done / dt / 1e12, "unit": "TB/s", "cores": 1, "kind": "port",
            "sample": f"{reps} x decode of 4 of the 64 config-2 sequences (numpy port; reference not installed), "
                      f"{dt:.1f} s", "cpu_model": _cpu_model()}


TILELANG_APPEND_UNAVAILABLE = ("unavailable: the image's tilelang 0.1.9 cannot trace it (fused_kv.py:562 calls "
                               "T.round(..., rounding_mode=...), which 0.1.9 lacks; the reference pins tilelang>=0.1.13)")


def run_tilelang(args):
    """The reference's own GPU decode kernel, _int4_paged_decode_attention
    (fused_attention.py:11-220, TileLang, JIT-compiled here by the image's
    tilelang) on config 2, loaded by file from the unmodified install in
    baseline/_ref.  Prints one JSON line: the kernel's time replayed from a
    CUDA graph, the public wrapper's time (its per-call host checks
    included), and its max error against an FP32 dequantise-then-attend
    reference on two sequences."""
    path = os.path.join(ROOT, "baseline", "_ref", "iris_kernel", "fused_attention.py")
    if not os.path.isfile(path):
        print(json.dumps({"impl": "tilelang", "unavailable": "reference not installed in baseline/_ref"}), flush=True)
        return
    res = {"impl": "tilelang", "kernel": "_int4_paged_decode_attention (reference, TileLang JIT)",
           "append": TILELANG_APPEND_UNAVAILABLE}
    try:
        import tilelang

        res["tilelang"] = tilelang.__version__
        t0 = time.time()
        spec = importlib.util.spec_from_file_location("_iris_reference_fused_attention", path)
        fa = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(fa)
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(0)
        pool = B * (L // P + 1)
        kd = torch.randint(0, 256, (pool, P, HKV, D // 2), dtype=torch.uint8, device=dev, generator=g)
        vd = torch.randint(0, 256, (pool, P, HKV, D // 2), dtype=torch.uint8, device=dev, generator=g)
        ks = (torch.rand((pool, P, HKV, D // G), device=dev, generator=g) * 0.1 + 0.01).half()
        vs = (torch.rand((pool, P, HKV, D // G), device=dev, generator=g) * 0.1 + 0.01).half()
        bt = torch.randperm(pool, device=dev, generator=g).int().view(B, L // P + 1).contiguous()
        lens = torch.full((B,), L, dtype=torch.int32, device=dev)
        q = torch.randn(B, HQ, D, device=dev, generator=g).half()
        out = torch.empty_like(q)
        fa.fused_int4_paged_decode_attention(q, kd, vd, ks, vs, bt, lens, out)  # JIT compile
        torch.cuda.synchronize()
        res["jit_s"] = round(time.time() - t0, 1)
        err = 0.0
        for b in range(2):
            o, _ = _fp32_partial(q[b], kd, vd, ks, vs, bt[b], L, HQ)
            err = max(err, float((out[b].float() - o).abs().max()))
        res["max_abs_err_vs_fp32"] = err
        raw = lambda: fa._int4_paged_decode_attention(q, kd, vd, ks, vs, bt, lens, out, D, P, G, 16, 32, 128, 0.0)
        gr = graph_of(raw, dev)
        n = max(10, min(args.steps, 50))
        us = timed(gr.replay, n, dev, None, 3) / n * 1e3
        res["decode_us"] = us
        res["decode_tbs"] = DECODE_BYTES / (us * 1e-6) / 1e12
        n_api = 5
        res["api_us"] = timed(lambda: fa.fused_int4_paged_decode_attention(q, kd, vd, ks, vs, bt, lens, out), n_api,
                              dev, None, 2) / n_api * 1e3
        del gr
    except Exception as e:  # report why, as the line's result
        res["unavailable"] = f"{type(e).__name__}: {str(e)[:300]}"
    print(json.dumps(res), flush=True)


def tilelang_leg(args, dec_us):
    """Runs run_tilelang in a child process (the JIT and the reference's
    modules stay out of this process) and returns its result."""
    try:
        out = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "tilelang", "--steps",
                              str(args.steps)], capture_output=True, text=True, timeout=420)
        lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
        res = json.loads(lines[-1]) if lines else {"unavailable": (out.stderr or out.stdout)[-300:]}
    except Exception as e:
        res = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
    res.pop("impl", None)
    if "decode_us" in res:
        res["ours_speedup"] = res["decode_us"] / dec_us
    return res


def run_reference(args, dist, rank, world):
    """The reference's CPU path on the host cores, rank 0 only: every step
    is a measured run of torch_eager_int4_paged_decode_attention over the
    step's sequences plus torch_eager_append of their new tokens.  A step is
    the full 64-sequence config-2 step unless warm-up + steps would then take
    more than ~150 s; then every step covers the first n sequences (n sized
    from a timed first step) and the line says so."""
    if rank != 0:
        return
    ref = load_reference_eager()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref "
                                                              "(python oracle/install_reference.py <checkout>)"}),
              flush=True)
        return
    threads = _host_threads()
    torch.set_num_threads(threads)
    smp = CpuStep(ref)
    smp.step(1)  # first touch of the arrays
    t0 = time.perf_counter()
    smp.step(B)  # calibration: one full step
    t_full = time.perf_counter() - t0
    seqs = B
    if (args.steps + args.warmup) * t_full > 150.0:
        seqs = max(1, min(B, int(B * 150.0 / ((args.steps + args.warmup) * t_full))))
    for _ in range(args.warmup):
        smp.step(seqs)
    done = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        done += smp.step(seqs)
    dt = time.perf_counter() - t0
    value = done / dt / 1e12
    sample = (f"{args.steps} measured steps, each the eager decode of {seqs} of the 64 sequences x 4096 tokens "
              f"+ their 1-token appends{'' if seqs == B else ' (a full step would exceed the run budget)'}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16/int4->fp32",
        "data": "synthetic", "config": _config(world), "step_sequences": seqs, "run_s": dt,
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "reference",
                         "code": "torch_eager_int4_paged_decode_attention + torch_eager_append "
                                 "(baseline/_ref, unmodified)", "sample": sample, "cpu_model": _cpu_model(),
                         "torch_threads": threads},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "decode-attn achieved HBM TB/s (% of B200 peak) + us/step; append tokens/s"


SWEEP_LENS = (128, 512, 2048, 4096)  # the reference's decode sweep (tests/bench_attention.py:291)
SWEEP_TOKENS = (1, 8, 32, 128)  # the reference's append sweep (tests/bench.py:550)


def p50_us(fn, inner, samples=50, warmup=20):
    """Median over `samples` event-timed runs of `inner` back-to-back calls,
    per call, in µs (the reference benchmarks' measure, warm L2)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    res = []
    for _ in range(samples):
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(inner):
            fn()
        en.record()
        en.synchronize()
        res.append(st.elapsed_time(en) * 1e3 / inner)
    return statistics.median(res)


def _neox(x, cos, sin):
    """NeoX rotation of the last dimension with fp16 cos/sin rows (set-up only)."""
    h = x.shape[-1] // 2
    a, b = x[..., :h].float(), x[..., h:].float()
    c, s = cos.float(), sin.float()
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).half()


def run_sweep(args, dev):
    """The reference benchmarks' two tables on this GPU, one JSON line.

    Decode (batch 1, Hq 32, Hkv 8, D 128, L in SWEEP_LENS): the INT4 and the
    matched FP16 decode through the public API (deferred validation, calls
    back to back) and replayed from a graph, the reference's torch eager INT4
    decode on the same GPU when its install is present, and the INT4 output's
    cosine and RMSE against the FP16 one.  Both caches are written by this
    library's appends from the same K/V ~ N(0, 1).
    Append (Hkv 4, D 128, T in SWEEP_TOKENS new tokens into fresh pages): the
    INT4 append through the public API and from a graph, and the reference's
    torch eager append on the same GPU.  The inputs fit in L2 and stay there,
    as in the reference's benchmarks."""
    import iris_kernel
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention, fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_fp16_append, fused_rope_int4_paged_append

    ref = load_reference_eager()
    hq, hkv = 32, 8
    rows = []
    iris_kernel.set_validation_mode("deferred")
    for seq_len in SWEEP_LENS:
        g = torch.Generator(device=dev).manual_seed(3407 + seq_len)
        npg = -(-seq_len // P)
        bt = torch.randperm(npg, generator=g, device=dev).int().view(1, npg).contiguous()
        lens = torch.full((1,), seq_len, dtype=torch.int32, device=dev)
        pos = torch.arange(seq_len, dtype=torch.int32, device=dev)
        slots = (bt[0, pos.long() // P] * P + pos % P).int().contiguous()
        cos, sin = rope_tables(seq_len, D, dev)
        k = torch.randn(seq_len, hkv, D, generator=g, device=dev).half()
        v = torch.randn(seq_len, hkv, D, generator=g, device=dev).half()
        kd = torch.empty(npg, P, hkv, D // 2, dtype=torch.uint8, device=dev)
        vd = torch.empty_like(kd)
        ks = torch.empty(npg, P, hkv, D // G, dtype=torch.float16, device=dev)
        vs = torch.empty_like(ks)
        kc = torch.zeros(npg, P, hkv, D, dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        fused_rope_int4_paged_append(k, v, pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D, page_size=P)
        fused_rope_fp16_append(k, v, pos, slots, cos, sin, kc, vc, rotary_dim=D, page_size=P)
        q = _neox(torch.randn(1, hq, D, generator=g, device=dev).half(), cos[seq_len - 1], sin[seq_len - 1])
        o4, o16 = torch.empty_like(q), torch.empty_like(q)
        i4 = lambda: fused_int4_paged_decode_attention(q, kd, vd, ks, vs, bt, lens, o4)
        f16 = lambda: fused_fp16_paged_decode_attention(q, kc, vc, bt, lens, o16)
        inner = 50 if seq_len <= 512 else 20
        row = {"seq_len": seq_len, "int4_us": p50_us(i4, inner), "fp16_us": p50_us(f16, inner)}
        g4, g16 = graph_of(i4, dev), graph_of(f16, dev)
        row["int4_graph_us"] = p50_us(g4.replay, inner)
        row["fp16_graph_us"] = p50_us(g16.replay, inner)
        del g4, g16
        if ref is not None:
            eager = ref["torch_eager_attention"].torch_eager_int4_paged_decode_attention
            row["eager_int4_us"] = p50_us(lambda: eager(q, kd, vd, ks, vs, bt, lens, page_size=P, group_size=G),
                                          max(1, inner // 5), samples=20, warmup=3)
        torch.cuda.synchronize(dev)
        iris_kernel.check_errors(dev)
        a, b = o4.float().flatten(0, 1), o16.float().flatten(0, 1)
        row["vs_fp16"] = row["fp16_us"] / row["int4_us"]
        row["output_cosine"] = float(torch.nn.functional.cosine_similarity(a, b, dim=-1).mean())
        row["output_rmse"] = float(((a - b) ** 2).mean().sqrt())
        rows.append({kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in row.items()})
    app_rows = []
    for tokens in SWEEP_TOKENS:
        g = torch.Generator(device=dev).manual_seed(11 + tokens)
        npg = -(-tokens // P)
        k = torch.randn(tokens, 4, D, generator=g, device=dev).half()
        v = torch.randn_like(k)
        pos = torch.arange(tokens, dtype=torch.int32, device=dev)
        slots = pos.clone()
        cos, sin = rope_tables(max(tokens, 1), D, dev)
        kd = torch.empty(npg, P, 4, D // 2, dtype=torch.uint8, device=dev)
        vd = torch.empty_like(kd)
        ks = torch.empty(npg, P, 4, D // G, dtype=torch.float16, device=dev)
        vs = torch.empty_like(ks)
        ap = lambda: fused_rope_int4_paged_append(k, v, pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                                  page_size=P)
        row = {"tokens": tokens, "fused_us": p50_us(ap, 50)}
        ga = graph_of(ap, dev)
        row["graph_us"] = p50_us(ga.replay, 50)
        del ga
        if ref is not None:
            eager = ref["torch_eager_kv"].torch_eager_append
            row["eager_us"] = p50_us(lambda: eager(k, v, pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                                   group_size=G, page_size=P), 10, samples=20, warmup=3)
            row["vs_eager"] = row["eager_us"] / row["fused_us"]
        row["tokens_per_s"] = tokens / (row["fused_us"] * 1e-6)
        torch.cuda.synchronize(dev)
        iris_kernel.check_errors(dev)
        app_rows.append({kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in row.items()})
    iris_kernel.set_validation_mode("sync")
    print(json.dumps({"only": "sweep", "n_gpus": 1, "l2": "warm (inputs fit in L2; calls back to back)",
                      "decode": rows, "append": app_rows,
                      "eager": "reference torch eager on this GPU" if ref is not None else "not installed"}),
          flush=True)


def _config(world):
    nseq = B // world if B % world == 0 else -(-B // world)
    mb = (decode_bytes(nseq) + append_bytes(nseq)) / 1e6
    return {"workload": "BASELINE config 2: INT4 paged decode 64 x 4096 (Hq 32, Hkv 8, D 128) + 1-token append",
            "batch": B, "context": L, "page_size": P, "group": G,
            "parallelism": f"sequence-sharded {B // world if B % world == 0 else '~' + str(B // world)} seqs/GPU"
                           if world > 1 else "one GPU",
            "l2": (f"flushed: {mb:.0f} MB of cache per GPU per step < 2 x 126 MB L2, so every timed step follows "
                   "a 256 MB write and a 256 MB read of another buffer and is timed between its own events"
                   if needs_flush(decode_bytes(nseq) + append_bytes(nseq))
                   else f"no flush: {mb:.0f} MB of cache per GPU per step > 2 x 126 MB L2")}


# ------------------------------------------------------------- config 4 pieces

def _fp32_partial(q, kd, vd, ks, vs, bt_row, ntok, hq):
    """FP32 (o, lse natural) of one sequence over `ntok` tokens of its local
    pages, dequantised in torch (an independent restatement for the
    self-check; not the timed path)."""
    hkv = kd.shape[2]
    rep = hq // hkv
    npg = -(-ntok // P)
    ids = bt_row[:npg].long()
    o = torch.empty(hq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(hq, dtype=torch.float32, device=q.device)

    def deq(packed, scales):
        lo = (packed & 0x0F).to(torch.int16)
        hi = (packed >> 4).to(torch.int16)
        lo = torch.where(lo >= 8, lo - 16, lo)
        hi = torch.where(hi >= 8, hi - 16, hi)
        x = torch.stack((lo, hi), dim=-1).flatten(-2).float()
        return x * scales.float().repeat_interleave(G, dim=-1)

    for h in range(hkv):
        k = deq(kd[ids, :, h].reshape(-1, D // 2)[:ntok], ks[ids, :, h].reshape(-1, D // G)[:ntok])
        v = deq(vd[ids, :, h].reshape(-1, D // 2)[:ntok], vs[ids, :, h].reshape(-1, D // G)[:ntok])
        logits = (q[h * rep:(h + 1) * rep].float() @ k.T) * (D ** -0.5)
        lse[h * rep:(h + 1) * rep] = torch.logsumexp(logits, dim=-1)
        o[h * rep:(h + 1) * rep] = torch.softmax(logits, dim=-1) @ v
    return o, lse


def c4_self_check(c4, dec4, out, dist, rank, world, dev):
    """Rank 0 compares the split-context output of sequences 0..1 with an
    FP32 reference assembled from every rank's FP32 partial over its own
    splits (log-sum-exp merge in fp64).  Every rank takes the same
    collective steps."""
    plan = c4["plan"]
    n = C4_CHECK_SEQS
    po = torch.zeros(n, C4_HQ, D, dtype=torch.float32, device=dev)
    pl = torch.full((n, C4_HQ), float("-inf"), dtype=torch.float32, device=dev)
    for i, b in enumerate(plan.seqs.tolist()):
        if b < n:
            po[b], pl[b] = _fp32_partial(c4["q"][b], c4["kd"], c4["vd"], c4["ks"], c4["vs"], dec4.local_bt[i],
                                         int(plan.lens[i]), C4_HQ)
    if dist is not None:
        ao = torch.empty(world, *po.shape, dtype=po.dtype, device=dev)
        al = torch.empty(world, *pl.shape, dtype=pl.dtype, device=dev)
        dist.all_gather_into_tensor(ao, po)
        dist.all_gather_into_tensor(al, pl)
    else:
        ao, al = po[None], pl[None]
    if rank != 0:
        return None
    lse = al.double()
    m = lse.max(dim=0).values
    w = torch.exp(lse - m)
    w = w / w.sum(dim=0)
    ref = (w[..., None] * ao.double()).sum(dim=0).float()
    got = out[:n].float()
    err = (got - ref).abs()
    ok = bool((err <= 2e-3 + 1e-2 * ref.abs()).all() and torch.isfinite(got).all())
    return {"max_abs_err": float(err.max()), "pass": ok, "seqs": n, "tol": "2e-3 + 1e-2|ref|"}


def c4_breakdown(c4, dec4, steps, dev, dist, warmup):
    """Per-stage device times of the split-context step, each stage replayed
    from its own graph: the local LSE decode, then the peer-memory merge
    (which publishes the partial), or for NCCL the all-gather and the
    merge.  Returns max-over-ranks us per step of each, and the min over ranks
    of the decode (the spread is the rank skew the exchange absorbs)."""
    from iris_kernel.fused_attention import decode_partial, merge_lse_packed

    plan = dec4.plan

    def dec():
        decode_partial(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"], dec4.local_bt, dec4.lens, out=dec4._o,
                       lse=dec4._lse)

    def gather():
        dist.all_gather_into_tensor(dec4.recv, dec4.send)

    def merge():
        merge_lse_packed(dec4.recv if dist is not None else dec4.send, dec4.world, plan.batch, C4_HQ, D,
                         dec4.output)

    stages = [("decode", dec)]
    if dec4.xchg is not None:
        stages += [("p2p_merge", lambda: dec4.xchg.merge(dec4.output.view(-1, D), dec4._o.view(-1, D),
                                                          dec4._lse.view(-1)))]
    else:
        stages += [("merge", merge)] + ([("allgather", gather)] if dist is not None else [])
    res = {}
    for name, fn in stages:
        g = graph_of(fn, dev)
        ms = timed(g.replay, steps, dev, dist, warmup) / steps
        res[name + "_us"] = reduce_over_ranks(ms, dist, dev) * 1e3
        if name == "decode":
            res["decode_us_min_rank"] = reduce_over_ranks(ms, dist, dev, "min") * 1e3
        del g
    return res


# --------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "tilelang"])
    ap.add_argument("--only", default="all", choices=["all", "c2", "c3", "c4", "c5a", "c5b", "f16", "next", "sweep"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "tilelang":  # the reference's TileLang decode on one GPU (a child of the N=1 run)
        run_tilelang(args)
        return
    if args.impl == "reference":
        # host work only: no process group; under torchrun rank 0 alone runs it
        run_reference(args, None, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    dist, rank, world, local = _dist()

    import iris_kernel
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.only == "sweep":  # the reference benchmarks' tables, one GPU, not part of the default run
        if rank == 0 and world == 1:
            run_sweep(args, dev)
        if dist is not None:
            dist.destroy_process_group()
        return
    run = (lambda name: args.only in ("all", name))
    x_steps = max(10, min(args.steps, 100))
    peak, peak_kind = _peak_gbs()
    extra = {}
    clocks = None

    # ---- config 2 step: value (graph replay, inputs resident) ----
    lo, hi = shard(world, rank)
    nseq = hi - lo
    # this GPU's share of the step under twice the L2: flush between timed steps
    c2_flush = L2Flush(dev) if needs_flush(decode_bytes(nseq) + append_bytes(nseq)) else None
    if run("c2"):
        w = build_c2(dev, 1234 + rank, nseq)

        def step_decode():
            fused_int4_paged_decode_attention(w["q"], w["kd"], w["vd"], w["ks"], w["vs"], w["bt"], w["lens"],
                                              w["out"])

        def step_append():
            fused_rope_int4_paged_append(w["knew"], w["vnew"], w["newpos"], w["newslot"], w["cos"], w["sin"],
                                         w["kd"], w["vd"], w["ks"], w["vs"], rotary_dim=D, page_size=P)

        side = torch.cuda.Stream(dev)

        def step_both():
            # the append writes token 4096 (page 256 of every sequence), which the decode over
            # tokens 0..4095 does not read: the graph runs it as a second branch beside the decode
            # (its 64-thread CTAs fit in the registers the decode leaves free on every SM)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                step_append()
            step_decode()
            torch.cuda.current_stream(dev).wait_stream(side)

        iris_kernel.set_validation_mode("deferred")
        g_step = graph_of(step_both, dev)
        g_dec = graph_of(step_decode, dev)
        g_app = graph_of(step_append, dev)
        clk = Clocks(local).__enter__()
        ms = timed(g_step.replay, args.steps, dev, dist, args.warmup, c2_flush)
        d_steps = max(args.steps, 200)
        ms_dec = timed(g_dec.replay, d_steps, dev, dist, args.warmup, c2_flush) / d_steps
        ms_app = timed(g_app.replay, d_steps, dev, dist, args.warmup, c2_flush) / d_steps
        iris_kernel.check_errors(dev)
        del g_step, g_dec, g_app
        ms = reduce_over_ranks(ms, dist, dev)
        dec_us = reduce_over_ranks(ms_dec, dist, dev) * 1e3
        app_us = reduce_over_ranks(ms_app, dist, dev) * 1e3
        step_ms = ms / args.steps
        e2e = run_e2e(w, args, dev, dist, world, c2_flush)
        clk.__exit__(None, None, None)
        clocks = clk.summary()
        del w
    # ---- config 5b prefill append and config 5a decode-style append ----
    if run("c5b"):
        x = build_prefill(dev, seed=99 + rank)
        iris_kernel.set_validation_mode("deferred")
        g_pf = graph_of(lambda: fused_rope_int4_paged_append(x["k"], x["v"], x["pos"], x["slots"], x["cos"],
                                                             x["sin"], x["kd"], x["vd"], x["ks"], x["vs"],
                                                             rotary_dim=D, page_size=P), dev)
        pf_us = reduce_over_ranks(timed(g_pf.replay, x_steps, dev, dist, args.warmup), dist, dev) / x_steps * 1e3
        iris_kernel.check_errors(dev)
        del g_pf, x
        extra["c5b"] = {"us": pf_us, "tbs": world * PF_BYTES / (pf_us * 1e-6) / 1e12,
                        "frac": PF_BYTES / (pf_us * 1e-6) / 1e9 / peak,
                        "tokens_per_s": world * PF_S * PF_L / (pf_us * 1e-6)}
    # ---- the standalone write-path kernels at the config-5b shape (one GPU) ----
    if run("next") and world == 1:
        from iris_kernel.fused_kv import fused_quantize_pack_int4, fused_rope_fp16_append

        x = build_prefill(dev, seed=77)
        T = PF_S * PF_L
        pk = torch.empty(T, HKV, D // 2, dtype=torch.uint8, device=dev)
        sc = torch.empty(T, HKV, D // G, dtype=torch.float16, device=dev)
        iris_kernel.set_validation_mode("deferred")
        g_q = graph_of(lambda: fused_quantize_pack_int4(x["k"], pk, sc), dev)
        q_bytes = T * HKV * (2 * D + D // 2 + D // 16)  # fp16 in, packed bytes and scales out
        q_flush = L2Flush(dev) if needs_flush(q_bytes) else None
        q_us = timed(g_q.replay, x_steps, dev, None, args.warmup, q_flush) / x_steps * 1e3
        del g_q, pk, sc, q_flush
        kc = torch.zeros(T // P, P, HKV, D, dtype=torch.float16, device=dev)
        vc = torch.zeros_like(kc)
        g_a = graph_of(lambda: fused_rope_fp16_append(x["k"], x["v"], x["pos"], x["slots"], x["cos"], x["sin"], kc,
                                                      vc, rotary_dim=D, page_size=P), dev)
        # K, V fp16 in and out, slots and positions, one cos and one sin row per position
        a_bytes = T * HKV * 8 * D + T * 8 + PF_L * 2 * (D // 2) * 2
        a_us = timed(g_a.replay, x_steps, dev, None, args.warmup) / x_steps * 1e3
        iris_kernel.check_errors(dev)
        del g_a, kc, vc, x
        extra["qpack"] = {"us": round(q_us, 2), "tbs": round(q_bytes / (q_us * 1e-6) / 1e12, 3),
                          "frac": round(q_bytes / (q_us * 1e-6) / 1e9 / peak, 4), "shape": "65536 x 8 x 128",
                          "l2": "flushed" if needs_flush(q_bytes) else "no flush"}
        extra["f16_append"] = {"us": round(a_us, 2), "tbs": round(a_bytes / (a_us * 1e-6) / 1e12, 3),
                               "frac": round(a_bytes / (a_us * 1e-6) / 1e9 / peak, 4),
                               "tokens_per_s": T / (a_us * 1e-6), "shape": "8 x 8192 tokens, Hkv 8, D 128"}
    if run("c5a"):
        x5 = build_c5a(dev, seed=55 + rank)
        iris_kernel.set_validation_mode("deferred")
        g_a5 = graph_of(lambda: fused_rope_int4_paged_append(x5["k"], x5["v"], x5["pos"], x5["slots"], x5["cos"],
                                                             x5["sin"], x5["kd"], x5["vd"], x5["ks"], x5["vs"],
                                                             rotary_dim=D, page_size=P), dev)
        a5_flush = L2Flush(dev) if needs_flush(A5_BYTES) else None
        a5_us = reduce_over_ranks(timed(g_a5.replay, x_steps, dev, dist, args.warmup, a5_flush), dist, dev) / x_steps * 1e3
        del a5_flush
        iris_kernel.check_errors(dev)
        del g_a5, x5
        extra["c5a"] = {"us": a5_us, "tokens_per_s": world * A5_T / (a5_us * 1e-6)}
    # ---- config 4: split-context decode over the ranks (peer-memory merge; NCCL beside it) ----
    if run("c4"):
        from iris_kernel import parallel

        c4 = build_c4(dev, rank, world, seed=44 + rank)
        # over NVLink peer memory at N > 1 (CUDA IPC exchange buffers, one merge kernel reading every
        # GPU's partial); NCCL all-gather + merge timed beside it
        transports = ["p2p", "nccl"] if world > 1 else ["nccl"]
        times = {}
        for tr in transports:
            dec4 = parallel.SplitContextDecoder(c4["plan"], c4["bt"], C4_HQ, D, transport=tr)
            iris_kernel.set_validation_mode("deferred")
            g_c4 = graph_of(lambda: dec4(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"]), dev)
            ms_c4 = timed(g_c4.replay, x_steps, dev, dist, args.warmup)
            iris_kernel.check_errors(dev)
            del g_c4  # a graph holding an NCCL call is released before the process group
            times[tr] = reduce_over_ranks(ms_c4, dist, dev) / x_steps * 1e3
            if tr == transports[0]:
                parts = c4_breakdown(c4, dec4, x_steps, dev, dist, args.warmup)
                iris_kernel.set_validation_mode("sync")
                out4 = dec4(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"])
                torch.cuda.synchronize(dev)
                check = c4_self_check(c4, dec4, out4, dist, rank, world, dev)
            iris_kernel.set_validation_mode("sync")
            dec4.close()
            del dec4
        c4_us = times[transports[0]]
        extra["c4"] = {"us": c4_us, "tbs": C4_BYTES / (c4_us * 1e-6) / 1e12,
                       "frac": C4_BYTES / (c4_us * 1e-6) / 1e9 / (world * peak), "transport": transports[0],
                       **({"nccl_us": round(times["nccl"], 2)} if world > 1 else {}),
                       **{k: round(v, 2) for k, v in parts.items()}, "check": check}
        del c4
    # ---- the matched FP16 decode on the config-2 shape ----
    if run("f16") and world == 1:
        from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

        g16 = torch.Generator(device=dev).manual_seed(16 + rank)
        pool = B * (L // P + 1)
        kc = (torch.randn(pool, P, HKV, D, generator=g16, device=dev) * 0.5).half()
        vc = (torch.randn(pool, P, HKV, D, generator=g16, device=dev) * 0.5).half()
        q16 = torch.randn(B, HQ, D, generator=g16, device=dev).half()
        bt16 = torch.randperm(pool, generator=g16, device=dev).int().view(B, L // P + 1).contiguous()
        lens16 = torch.full((B,), L, dtype=torch.int32, device=dev)
        out16 = torch.empty_like(q16)
        iris_kernel.set_validation_mode("deferred")
        g_f16 = graph_of(lambda: fused_fp16_paged_decode_attention(q16, kc, vc, bt16, lens16, out16), dev)
        f16_us = timed(g_f16.replay, x_steps, dev, dist, args.warmup) / x_steps * 1e3
        iris_kernel.check_errors(dev)
        del g_f16, kc, vc
        extra["f16"] = {"us": f16_us, "tbs": FP16_BYTES / (f16_us * 1e-6) / 1e12,
                        "frac": FP16_BYTES / (f16_us * 1e-6) / 1e9 / peak}
    # ---- config 3: sequence-sharded MHA decode, no collective ----
    if run("c3"):
        c3 = build_c3(dev, rank, world, seed=33 + rank)
        iris_kernel.set_validation_mode("deferred")
        g_c3 = graph_of(lambda: fused_int4_paged_decode_attention(c3["q"], c3["kd"], c3["vd"], c3["ks"], c3["vs"],
                                                                  c3["bt"], c3["lens"], c3["out"]), dev)
        c3_flush = L2Flush(dev) if needs_flush(c3["bytes"]) else None
        c3_us = reduce_over_ranks(timed(g_c3.replay, x_steps, dev, dist, args.warmup, c3_flush), dist, dev) / x_steps * 1e3
        del c3_flush
        iris_kernel.check_errors(dev)
        extra["c3"] = {"us": c3_us, "tbs": c3["total_bytes"] / (c3_us * 1e-6) / 1e12,
                       "frac": c3["total_bytes"] / (c3_us * 1e-6) / 1e9 / (world * peak)}
        del g_c3, c3
    iris_kernel.set_validation_mode("sync")

    cpu, tl = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and run("c2"):
        cpu = cpu_baseline_sample(seconds_budget=15.0)
        torch.cuda.empty_cache()
        tl = tilelang_leg(args, dec_us)

    if rank == 0:
        if not run("c2"):
            print(json.dumps({"only": args.only, "n_gpus": world, **extra, "clocks": clocks}), flush=True)
        else:
            dec_local = decode_bytes(nseq)
            achieved = dec_local / (dec_us * 1e-6) / 1e9
            traffic = None
            tpath = os.path.join(ROOT, "profiles", "decode_c2_traffic.json")
            if os.path.exists(tpath) and world == 1:
                try:
                    with open(tpath) as f:
                        traffic = json.load(f).get("dram_bytes_per_launch")
                except Exception:
                    traffic = None
            value = STEP_BYTES / (step_ms * 1e-3) / 1e12
            compact = {}
            for k in ("c3", "c4"):
                if k in extra:
                    compact[k + "_us"] = round(extra[k]["us"], 2)
                    compact[k + "_frac"] = round(extra[k]["frac"], 3)
            if "c4" in extra and extra["c4"]["check"] is not None:
                compact["c4_max_abs_err"] = extra["c4"]["check"]["max_abs_err"]
                compact["c4_parity"] = extra["c4"]["check"]["pass"]
            line = {
                "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, **compact,
                "dtype": "fp16/int4->fp32", "data": "synthetic (seeded N(0,1), random page permutation)",
                "config": _config(world),
                "decode_us": dec_us, "decode_tbs": dec_local / (dec_us * 1e-6) / 1e12,
                "decode_pct_of_8tbs": 100 * dec_local / (dec_us * 1e-6) / 1e12 / SPEC_TBS,
                "append_us": app_us, "append_tokens_per_s": B / (app_us * 1e-6),
                "e2e": e2e,
                "gpu_launches": 3 * args.steps,  # decode, combine, append per step (graph replay)
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                             "kernel": "decode + combine (graph), per GPU"},
                "cpu_baseline": cpu, "clocks": clocks, **{k: _round(v) for k, v in extra.items()},
                "tilelang_ref": _round(tl) if tl is not None else None,
            }
            print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _round(d):
    if isinstance(d, dict):
        return {k: _round(v) for k, v in d.items()}
    if isinstance(d, float):
        return float(f"{d:.4g}")
    return d


def run_e2e(w, args, dev, dist, world, flush=None):
    """The step through the public Python API with host buffers (deferred
    validation, the step's error word read on the host once per step).  The
    query copy leads and the decode starts as soon as it has landed, the
    output copy right after it; the new K/V copy and the append run
    meanwhile on a second stream.  ``graph_ms_per_step``: the same step,
    copies included, captured once in a CUDA graph and replayed (one
    launch per step), with the same host read.  Returns the line's e2e
    object."""
    import iris_kernel
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    parts = [("q", w["q"]), ("k", w["knew"]), ("v", w["vnew"]), ("p", w["newpos"]), ("s", w["newslot"])]
    offs, total = {}, 0
    for name, t in parts:
        offs[name] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    host_in = torch.empty(total, dtype=torch.uint8).pin_memory()
    dev_in = torch.empty(total, dtype=torch.uint8, device=dev)

    def view(buf, name, like):
        n = like.numel() * like.element_size()
        return buf[offs[name]:offs[name] + n].view(like.dtype).view(like.shape)

    for name, t in parts:
        view(host_in, name, t).copy_(t.cpu())
    hout = torch.empty_like(w["out"], device="cpu").pin_memory()
    h2d = sum(t.numel() * t.element_size() for _, t in parts)
    d2h = hout.numel() * hout.element_size()
    q, k, v, pp, ss = (view(dev_in, name, t) for name, t in parts)
    q_bytes = offs["k"]
    out_dev = torch.empty_like(w["out"])
    side = torch.cuda.Stream(dev)
    calls = {"dec": lambda: fused_int4_paged_decode_attention(q, w["kd"], w["vd"], w["ks"], w["vs"], w["bt"],
                                                              w["lens"], out_dev),
             "app": lambda: fused_rope_int4_paged_append(k, v, pp, ss, w["cos"], w["sin"], w["kd"], w["vd"], w["ks"],
                                                         w["vs"], rotary_dim=D, page_size=P)}

    def body():
        cur = torch.cuda.current_stream(dev)
        dev_in[:q_bytes].copy_(host_in[:q_bytes], non_blocking=True)
        side.wait_stream(cur)  # the K/V copy follows the query copy
        calls["dec"]()
        hout.copy_(out_dev, non_blocking=True)
        with torch.cuda.stream(side):  # the append runs beside the decode (it writes token 4096 only)
            dev_in[q_bytes:].copy_(host_in[q_bytes:], non_blocking=True)
            calls["app"]()
        cur.wait_stream(side)

    def e2e_step():
        body()
        iris_kernel.check_errors(dev)  # one host read of the error word per step (syncs)

    iris_kernel.set_validation_mode("deferred")
    ms = timed(e2e_step, args.steps, dev, dist, args.warmup, flush)
    # the same step (copies, calls, output copy) captured once in a CUDA graph and replayed
    g_e2e = graph_of(body, dev)

    def e2e_graph_step():
        g_e2e.replay()
        iris_kernel.check_errors(dev)

    ms_graph = timed(e2e_graph_step, args.steps, dev, dist, args.warmup, flush)
    del g_e2e
    iris_kernel.set_validation_mode("sync")
    ms = reduce_over_ranks(ms, dist, dev)
    ms_graph = reduce_over_ranks(ms_graph, dist, dev)
    return {"value": STEP_BYTES / (ms / args.steps * 1e-3) / 1e12, "unit": "TB/s", "ms_per_step": ms / args.steps,
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "path": "public Python API, deferred validation, error word read per step",
            "graph_ms_per_step": ms_graph / args.steps}


if __name__ == "__main__":
    main()
