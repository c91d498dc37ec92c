"""Benchmark of the INT4 paged KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (Llama-3-8B shape): 64 sequences x 4096 tokens
of INT4 paged cache (Hq=32, Hkv=8, D=128, page 16, group 32, pages scattered
by a random permutation over a pool of 64 x 257 pages; K/V ~N(0,1) fp16 with
4 outlier K channels x8, written by the fused append), then per step

    decode attention over the 4096 cached tokens of every sequence, and
    a batched 1-token fused RoPE+INT4 append per sequence at position 4096.

One process per GPU (torchrun for N > 1): every rank owns an independent
copy of the workload (sequences are partitioned across GPUs, no collective),
so ``scaling`` is "weak" and ``value`` is the aggregate over ranks.

``value``: algorithmic bytes of the step (decode + append) x N /
max-over-ranks step time, in TB/s, with inputs resident in HBM; the step is
replayed from a CUDA graph (validation in deferred mode, no host syncs).
``e2e``: the same metric through the public Python API with host buffers:
per step the new query / K / V / positions / slots are copied from pinned
host memory, the decode and append calls run, the fp16 output is copied
back, and any error the step's kernels recorded is raised (one host read per
step, deferred validation mode).  ``e2e_sync`` is the same loop with every
call reading the error word before it returns (the reference's per-call
exceptions).

Also reported: config 5b prefill append, config 4 split-context decode over
the ranks (one NCCL all-gather per step), config 3 sequence-sharded decode.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "iris-kernel_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, L, HQ, HKV, D, P, G = 64, 4096, 32, 8, 128, 16, 32
POOL = B * (L // P + 1)
OUTLIER_CH = (3, 40, 77, 121)

# algorithmic bytes (DESIGN.md "Measurement"): KV pages + scales read once,
# Q read, O written, block table read; append reads K, V (fp16) and writes
# packed bytes + scales, plus slots/positions and one cos/sin row.
DECODE_BYTES = B * L * HKV * (D + D // 8) + 2 * B * HQ * D * 2 + B * (L // P + 1) * 4
APPEND_BYTES = B * HKV * (4 * D + D + D // 8) + B * 8 + 2 * (D // 2) * 2
STEP_BYTES = DECODE_BYTES + APPEND_BYTES
FP16_BYTES = B * L * HKV * D * 2 * 2 + 2 * B * HQ * D * 2 + B * (L // P + 1) * 4
SPEC_TBS = 8.0

# BASELINE config 5b: prefill-style append, 8 sequences x 8192 new tokens,
# Hkv=8, D=128, fresh permuted pages, 1% of entries x20, RoPE base 500000.
# BASELINE config 5a: decode-style append, 2048 sequences x 1 token, Hkv 1, D 128, positions
# ~U[0, 32768), RoPE base 500000, scattered pages
A5_T, A5_MAXPOS = 2048, 32768
A5_BYTES = A5_T * (4 * D + D + D // 8) + A5_T * 8 + A5_T * 2 * (D // 2) * 2
PF_S, PF_L = 8, 8192
PF_BYTES = PF_S * PF_L * HKV * (4 * D + D + D // 8) + PF_S * PF_L * 8 + PF_L * 2 * (D // 2) * 2


# BASELINE config 4 (70B-shaped long context): 16 sequences x 131,072 tokens,
# Hq 64, Hkv 8, D 128; split-context over the ranks in 8192-token splits,
# every rank's cache holding only its splits; one NCCL all-gather + merge.
C4_B, C4_L, C4_HQ, C4_HKV, C4_SPLIT = 16, 131072, 64, 8, 8192
C4_BYTES = C4_B * C4_L * C4_HKV * (D + D // 8) + 2 * C4_B * C4_HQ * D * 2 + C4_B * (C4_L // P) * 4 + C4_B * 4
# BASELINE config 3 (MHA, D 64, varlen): 128 sequences, Hq = Hkv = 16,
# L ~ U[1, 16384] (seed 1); sequences sharded over the ranks by token count.
C3_B, C3_H, C3_D, C3_LMAX = 128, 16, 64, 16384


def _fill_cache(dev, g, kd, vd, ks, vs, slots, positions, hkv, d, cos, sin, chunk=65536):
    """Write synthetic K/V ~ N(0, 0.5) through the fused append, in chunks."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    for t0 in range(0, slots.numel(), chunk):
        t1 = min(slots.numel(), t0 + chunk)
        k = (torch.randn(t1 - t0, hkv, d, generator=g, device=dev) * 0.5).half()
        v = (torch.randn(t1 - t0, hkv, d, generator=g, device=dev) * 0.5).half()
        fused_rope_int4_paged_append(k, v, positions[t0:t1].contiguous(), slots[t0:t1].contiguous(), cos, sin,
                                     kd, vd, ks, vs, rotary_dim=d, page_size=P)


def build_c4(dev, rank, world, seed):
    """This rank's share of config 4: only the pages of its splits exist in
    its cache; the block table maps its split columns to them."""
    from iris_kernel import parallel
    from oracle import iris_oracle as orc  # RoPE table builder only (host arrays)

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
    cos_np, sin_np = orc.rope_cache(C4_L, D, 500000.0)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    _fill_cache(dev, g, kd, vd, ks, vs, torch.cat(slot_l), torch.cat(pos_l), C4_HKV, D, cos, sin)
    q = torch.randn(C4_B, C4_HQ, D, generator=torch.Generator(device=dev).manual_seed(4), device=dev).half()
    return dict(plan=plan, q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt)


def build_c3(dev, rank, world, seed):
    """This rank's shard of config 3 (whole sequences, balanced by tokens)."""
    from iris_kernel import parallel
    from oracle import iris_oracle as orc  # RoPE table builder only (host arrays)

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
    cos_np, sin_np = orc.rope_cache(C3_LMAX, C3_D)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    _fill_cache(dev, g, kd, vd, ks, vs, torch.cat(slot_l), torch.cat(pos_l), C3_H, C3_D, cos, sin)
    q = torch.randn(len(mine), C3_H, C3_D, generator=g, device=dev).half()
    nbytes = int(lens.sum()) * C3_H * (C3_D + C3_D // 8) + 2 * len(mine) * C3_H * C3_D * 2 + int(npg.sum()) * 4
    total = int(lens_all.sum()) * C3_H * (C3_D + C3_D // 8) + 2 * C3_B * C3_H * C3_D * 2 + int(
        ((lens_all + P - 1) // P).sum()) * 4
    return dict(q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt,
                lens=torch.from_numpy(lens.astype(np.int32)).to(dev),
                out=torch.empty_like(q), bytes=nbytes, total_bytes=total)


def _peak_gbs():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return 6650.0, "fallback"


def _dist():
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), dist.get_world_size(), local
    return None, 0, 1, 0


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{index}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            if os.path.exists(self.path):
                os.remove(self.path)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            t0 = time.time()  # start timing only once samples are flowing
            while time.time() - t0 < 10 and (not os.path.exists(self.path) or os.path.getsize(self.path) == 0):
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
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


def build_workload(dev, seed):
    """Cache written by the fused append from synthetic K/V (config 2)."""
    from iris_kernel.fused_kv import fused_rope_int4_paged_append
    from oracle import iris_oracle as orc  # RoPE table builder only (host arrays)

    g = torch.Generator(device=dev).manual_seed(seed)
    perm = torch.randperm(POOL, generator=g, device=dev).int()
    bt = perm.view(B, L // P + 1).contiguous()
    kd = torch.zeros(POOL, P, HKV, D // 2, dtype=torch.uint8, device=dev)
    vd = torch.zeros_like(kd)
    ks = torch.zeros(POOL, P, HKV, D // G, dtype=torch.float16, device=dev)
    vs = torch.zeros_like(ks)
    cos_np, sin_np = orc.rope_cache(L + 1, D)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    pos = torch.arange(L, device=dev, dtype=torch.int32)
    for b in range(B):
        k = torch.randn(L, HKV, D, generator=g, device=dev)
        k[..., list(OUTLIER_CH)] *= 8
        v = torch.randn(L, HKV, D, generator=g, device=dev)
        slots = (bt[b, (pos // P).long()] * P + pos % P).int()
        fused_rope_int4_paged_append(k.half(), v.half(), pos, slots, cos, sin, kd, vd, ks, vs, rotary_dim=D,
                                     page_size=P)
    q = torch.randn(B, HQ, D, generator=g, device=dev).half()
    knew = torch.randn(B, HKV, D, generator=g, device=dev)
    knew[..., list(OUTLIER_CH)] *= 8
    vnew = torch.randn(B, HKV, D, generator=g, device=dev)
    w = dict(q=q, kd=kd, vd=vd, ks=ks, vs=vs, bt=bt, cos=cos, sin=sin,
             lens=torch.full((B,), L, dtype=torch.int32, device=dev),
             knew=knew.half(), vnew=vnew.half(), newpos=torch.full((B,), L, dtype=torch.int32, device=dev),
             newslot=(bt[:, L // P] * P).int().contiguous(), out=torch.empty(B, HQ, D, dtype=torch.float16,
                                                                             device=dev))
    torch.cuda.synchronize(dev)
    return w


def build_prefill(dev, seed):
    from oracle import iris_oracle as orc  # RoPE table builder only (host arrays)

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
    cos_np, sin_np = orc.rope_cache(PF_L, D, 500000.0)
    return dict(k=k.half(), v=v.half(), pos=pos, slots=slots.contiguous(), cos=torch.from_numpy(cos_np).to(dev),
                sin=torch.from_numpy(sin_np).to(dev),
                kd=torch.zeros(npages, P, HKV, D // 2, dtype=torch.uint8, device=dev),
                vd=torch.zeros(npages, P, HKV, D // 2, dtype=torch.uint8, device=dev),
                ks=torch.zeros(npages, P, HKV, D // G, dtype=torch.float16, device=dev),
                vs=torch.zeros(npages, P, HKV, D // G, dtype=torch.float16, device=dev))


def build_c5a(dev, seed):
    from oracle import iris_oracle as orc  # RoPE table builder only (host arrays)

    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(A5_T, 1, D, generator=g, device=dev)
    v = torch.randn(A5_T, 1, D, generator=g, device=dev)
    k[torch.rand(k.shape, generator=g, device=dev) < 0.01] *= 20
    v[torch.rand(v.shape, generator=g, device=dev) < 0.01] *= 20
    npages = 2 * A5_T
    pages = torch.randperm(npages, generator=g, device=dev)[:A5_T]
    slots = (pages * P + torch.randint(0, P, (A5_T,), generator=g, device=dev)).int()
    pos = torch.randint(0, A5_MAXPOS, (A5_T,), generator=g, device=dev).int()
    cos_np, sin_np = orc.rope_cache(A5_MAXPOS, D, 500000.0)
    return dict(k=k.half(), v=v.half(), pos=pos, slots=slots, cos=torch.from_numpy(cos_np).to(dev),
                sin=torch.from_numpy(sin_np).to(dev),
                kd=torch.zeros(npages, P, 1, D // 2, dtype=torch.uint8, device=dev),
                vd=torch.zeros(npages, P, 1, D // 2, dtype=torch.uint8, device=dev),
                ks=torch.zeros(npages, P, 1, D // G, dtype=torch.float16, device=dev),
                vs=torch.zeros(npages, P, 1, D // G, dtype=torch.float16, device=dev))


def step_prefill(x):
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    fused_rope_int4_paged_append(x["k"], x["v"], x["pos"], x["slots"], x["cos"], x["sin"], x["kd"], x["vd"], x["ks"],
                                 x["vs"], rotary_dim=D, page_size=P)


def step_decode(w):
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention

    fused_int4_paged_decode_attention(w["q"], w["kd"], w["vd"], w["ks"], w["vs"], w["bt"], w["lens"], w["out"])


def step_append(w):
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    fused_rope_int4_paged_append(w["knew"], w["vnew"], w["newpos"], w["newslot"], w["cos"], w["sin"], w["kd"],
                                 w["vd"], w["ks"], w["vs"], rotary_dim=D, page_size=P)


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


def timed(fn, steps, dev, dist, warmup):
    """Warm up, barrier + sync, time exactly `steps` calls with CUDA events
    on the current stream, barrier + sync; returns ms for all steps."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(steps):
        fn()
    en.record()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    return st.elapsed_time(en)


def max_over_ranks(x, dist, dev):
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_baseline_sample(seconds_budget=15.0):
    """The CPU oracle (numpy port of the reference's eager path) on a bounded
    sample of the same workload: decode of whole 4096-token sequences plus the
    64-token append, repeated until the budget is used.  Returns TB/s of
    algorithmic bytes and a description."""
    from oracle import iris_oracle as orc

    rng = np.random.default_rng(0)
    nseq = 4
    NPs = nseq * (L // P)
    kd = rng.integers(0, 256, (NPs, P, HKV, D // 2), dtype=np.uint8)
    vd = rng.integers(0, 256, (NPs, P, HKV, D // 2), dtype=np.uint8)
    ks = rng.uniform(0.01, 1, (NPs, P, HKV, D // G)).astype(np.float16)
    vs = rng.uniform(0.01, 1, (NPs, P, HKV, D // G)).astype(np.float16)
    bt = rng.permutation(NPs).astype(np.int32).reshape(nseq, L // P)
    lens = np.full(nseq, L, np.int32)
    q = rng.standard_normal((nseq, HQ, D)).astype(np.float16)
    cos, sin = orc.rope_cache(L + 1, D)
    knew = rng.standard_normal((B, HKV, D)).astype(np.float16)
    vnew = rng.standard_normal((B, HKV, D)).astype(np.float16)
    apool = B
    akd = np.zeros((apool, P, HKV, D // 2), np.uint8)
    avd, aks, avs = akd.copy(), np.zeros((apool, P, HKV, D // G), np.float16), None
    avs = aks.copy()
    done_bytes = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        orc.decode_attention(q, kd, vd, ks, vs, bt, lens)
        orc.append(knew, vnew, np.full(B, L, np.int32), (np.arange(B) * P).astype(np.int32), cos, sin, akd, avd, aks,
                   avs, rotary_dim=D, group_size=G, page_size=P)
        reps += 1
        done_bytes += nseq * L * HKV * (D + D // 8) + 2 * nseq * HQ * D * 2 + nseq * (L // P) * 4 + APPEND_BYTES
        if time.perf_counter() - t0 > seconds_budget:
            break
    dt = time.perf_counter() - t0
    return done_bytes / dt / 1e12, (f"{reps} x (decode of {nseq} of the 64 sequences x 4096 tokens + the 64-token "
                                    f"append), numpy oracle, {dt:.1f} s"), dt


def _cpu_info():
    """The host CPU the baseline ran on: model name and torch's intra-op thread count."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "torch_threads": torch.get_num_threads()}


class _CpuSample:
    """The reference arm's CPU workload, built once: 4 of the config-2
    sequences (4096 tokens each, random cache contents) and their new tokens.
    A step is the numpy oracle's decode of one sequence over its first
    `pages` pages plus the append of that sequence's new token."""

    def __init__(self, nseq=4):
        from oracle import iris_oracle as orc

        self.orc = orc
        rng = np.random.default_rng(0)
        self.nseq = nseq
        NPs = nseq * (L // P)
        self.kd = rng.integers(0, 256, (NPs, P, HKV, D // 2), dtype=np.uint8)
        self.vd = rng.integers(0, 256, (NPs, P, HKV, D // 2), dtype=np.uint8)
        self.ks = rng.uniform(0.01, 1, (NPs, P, HKV, D // G)).astype(np.float16)
        self.vs = rng.uniform(0.01, 1, (NPs, P, HKV, D // G)).astype(np.float16)
        self.bt = rng.permutation(NPs).astype(np.int32).reshape(nseq, L // P)
        self.q = rng.standard_normal((nseq, HQ, D)).astype(np.float16)
        self.cos, self.sin = orc.rope_cache(L + 1, D)
        self.knew = rng.standard_normal((nseq, 1, HKV, D)).astype(np.float16)
        self.vnew = rng.standard_normal((nseq, 1, HKV, D)).astype(np.float16)
        self.akd = np.zeros((nseq, P, HKV, D // 2), np.uint8)
        self.avd = self.akd.copy()
        self.aks = np.zeros((nseq, P, HKV, D // G), np.float16)
        self.avs = self.aks.copy()
        self.i = 0

    def step(self, pages):
        """One step; returns its algorithmic bytes."""
        b = self.i % self.nseq
        self.i += 1
        self.orc.decode_attention(self.q[b:b + 1], self.kd, self.vd, self.ks, self.vs, self.bt[b:b + 1],
                                  np.array([pages * P], np.int32))
        self.orc.append(self.knew[b], self.vnew[b], np.array([L], np.int32), np.array([b * P], np.int32), self.cos,
                        self.sin, self.akd, self.avd, self.aks, self.avs, rotary_dim=D, group_size=G, page_size=P)
        return pages * P * HKV * (D + D // 8) + 2 * HQ * D * 2 + pages * 4 + APPEND_BYTES // B


def run_reference(args, dist, rank, world):
    """The reference's CPU path (numpy port of its eager code; the reference
    itself does not travel to the GPU box) on host cores, rank 0 only.  Each
    step decodes a chunk of one sequence, sized so that warm-up plus timed
    steps take about 90 s whatever their number."""
    if rank != 0:
        return
    smp = _CpuSample()
    smp.step(L // P)  # first touch of the arrays
    t0 = time.perf_counter()
    smp.step(L // P)  # calibration: one whole 4096-token sequence, warm
    t_full = time.perf_counter() - t0
    per_step = min(1.0, 90.0 / max(1, args.steps + args.warmup))
    pages = int(max(1, min(L // P, round((L // P) * per_step / max(t_full, 1e-6)))))
    for _ in range(args.warmup):
        smp.step(pages)
    done = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        done += smp.step(pages)
    dt = time.perf_counter() - t0
    value = done / dt / 1e12
    cores = os.cpu_count()
    desc = (f"{args.steps} steps x (decode of one of 4 config-2 sequences over its first {pages * P} tokens + "
            f"its 1-token append), numpy oracle, {dt:.1f} s")
    line = {
        "impl": "reference", "metric": "decode-attn achieved HBM TB/s (% of B200 peak) + us/step; append tokens/s",
        "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": STEP_BYTES / (value * 1e12) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16/int4->fp32", "data": "synthetic",
        "config": _config(),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": cores, "kind": "port", "sample": desc,
                         **_cpu_info()},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config():
    return {"workload": "BASELINE config 2: Llama-3-8B-shaped INT4 paged decode 64 x 4096 + 1-token append",
            "batch": B, "context": L, "hq": HQ, "hkv": HKV, "head_dim": D, "page_size": P, "group": G,
            "pool_pages": POOL, "l2": "no flush: each step reads 303 MB of cache > 126 MB L2",
            "parallelism": "sequence-sharded replicas (one 64x4096 batch per GPU)",
            "validation": "deferred (value, e2e), synchronous per call (e2e_sync)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    dist, rank, world, local = _dist()
    if args.impl == "reference":
        run_reference(args, dist, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    import iris_kernel
    from iris_kernel.fused_attention import fused_int4_paged_decode_attention
    from iris_kernel.fused_kv import fused_rope_int4_paged_append

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = build_workload(dev, seed=1234 + rank)

    # ---- value: graph-replayed steps, inputs resident ----
    iris_kernel.set_validation_mode("deferred")
    g_step = graph_of(lambda: (step_decode(w), step_append(w)), dev)
    g_dec = graph_of(lambda: step_decode(w), dev)
    g_app = graph_of(lambda: step_append(w), dev)
    clk = Clocks(local).__enter__()
    ms = timed(g_step.replay, args.steps, dev, dist, args.warmup)
    ms_dec = timed(g_dec.replay, args.steps, dev, dist, args.warmup)
    ms_app = timed(g_app.replay, args.steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    iris_kernel.set_validation_mode("sync")
    # config 5b prefill append (its own inputs; not part of the step)
    x = build_prefill(dev, seed=99 + rank)
    iris_kernel.set_validation_mode("deferred")
    g_pf = graph_of(lambda: step_prefill(x), dev)
    pf_steps = max(10, min(args.steps, 200))
    ms_pf = timed(g_pf.replay, pf_steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    iris_kernel.set_validation_mode("sync")
    del g_pf, x
    ms_pf = max_over_ranks(ms_pf, dist, dev)
    pf_us = ms_pf / pf_steps * 1e3
    # config 5a decode-style append (2048 x 1 token, Hkv 1; its own inputs)
    x5 = build_c5a(dev, seed=55 + rank)
    iris_kernel.set_validation_mode("deferred")
    g_a5 = graph_of(lambda: step_prefill(x5), dev)
    ms_a5 = timed(g_a5.replay, pf_steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    iris_kernel.set_validation_mode("sync")
    del g_a5, x5
    a5_us = max_over_ranks(ms_a5, dist, dev) / pf_steps * 1e3

    # config 4: split-context decode over the ranks (one NCCL all-gather per step)
    from iris_kernel import parallel

    c4 = build_c4(dev, rank, world, seed=44 + rank)
    dec4 = parallel.SplitContextDecoder(c4["plan"], c4["bt"], C4_HQ, D)
    iris_kernel.set_validation_mode("deferred")
    g_c4 = graph_of(lambda: dec4(c4["q"], c4["kd"], c4["vd"], c4["ks"], c4["vs"]), dev)
    x_steps = max(10, min(args.steps, 100))
    ms_c4 = timed(g_c4.replay, x_steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    del g_c4, dec4, c4  # the graph holds an NCCL call: released before the process group
    # the matched FP16 decode on the config-2 shape (the INT4 cache's baseline)
    from iris_kernel.fused_attention import fused_fp16_paged_decode_attention

    g16 = torch.Generator(device=dev).manual_seed(16 + rank)
    kc = (torch.randn(POOL, P, HKV, D, generator=g16, device=dev) * 0.5).half()
    vc = (torch.randn(POOL, P, HKV, D, generator=g16, device=dev) * 0.5).half()
    out16 = torch.empty_like(w["q"])
    g_f16 = graph_of(lambda: fused_fp16_paged_decode_attention(w["q"], kc, vc, w["bt"], w["lens"], out16), dev)
    ms_f16 = timed(g_f16.replay, x_steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    del g_f16, kc, vc
    # config 3: sequence-sharded MHA decode, no collective
    c3 = build_c3(dev, rank, world, seed=33 + rank)
    g_c3 = graph_of(lambda: fused_int4_paged_decode_attention(c3["q"], c3["kd"], c3["vd"], c3["ks"], c3["vs"],
                                                              c3["bt"], c3["lens"], c3["out"]), dev)
    ms_c3 = timed(g_c3.replay, x_steps, dev, dist, args.warmup)
    iris_kernel.check_errors(dev)
    iris_kernel.set_validation_mode("sync")
    c3_total = c3["total_bytes"]
    del g_c3, c3
    f16_us = max_over_ranks(ms_f16, dist, dev) / x_steps * 1e3
    c4_us = max_over_ranks(ms_c4, dist, dev) / x_steps * 1e3
    c3_us = max_over_ranks(ms_c3, dist, dev) / x_steps * 1e3
    ms = max_over_ranks(ms, dist, dev)
    ms_dec = max_over_ranks(ms_dec, dist, dev)
    ms_app = max_over_ranks(ms_app, dist, dev)
    step_ms = ms / args.steps
    dec_us = ms_dec / args.steps * 1e3
    app_us = ms_app / args.steps * 1e3
    value = world * STEP_BYTES / (step_ms * 1e-3) / 1e12

    # ---- e2e: public API with host buffers ----
    # The step's inputs (new query, K, V, positions, slots) sit in one pinned
    # host buffer and go to the device in one copy; the fp16 output comes back
    # in one copy.
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
    out_dev = torch.empty_like(w["out"])

    def calls():
        fused_int4_paged_decode_attention(q, w["kd"], w["vd"], w["ks"], w["vs"], w["bt"], w["lens"], out_dev)
        fused_rope_int4_paged_append(k, v, pp, ss, w["cos"], w["sin"], w["kd"], w["vd"], w["ks"], w["vs"],
                                     rotary_dim=D, page_size=P)

    def e2e_step(replay=None):
        dev_in.copy_(host_in, non_blocking=True)
        if replay is None:
            calls()
        else:
            replay()
        hout.copy_(out_dev, non_blocking=True)
        if iris_kernel.validation_mode() == "deferred":
            iris_kernel.check_errors(dev)  # one host read per step raises any error of the step

    # e2e: eager calls, deferred validation, errors raised once per step (the
    # host prepares the next call while the GPU runs).  e2e_sync: every call
    # reads the error word before it returns, as the reference's calls raise.
    # e2e_graph: the two calls captured once in a CUDA graph and replayed.
    iris_kernel.set_validation_mode("deferred")
    ms_e2e = timed(e2e_step, args.steps, dev, dist, args.warmup)
    g_e2e = graph_of(calls, dev)
    ms_e2e_graph = timed(lambda: e2e_step(g_e2e.replay), args.steps, dev, dist, args.warmup)
    iris_kernel.set_validation_mode("sync")
    ms_e2e_sync = timed(e2e_step, args.steps, dev, dist, args.warmup)
    del g_e2e
    clk.__exit__(None, None, None)
    ms_e2e = max_over_ranks(ms_e2e, dist, dev)
    ms_e2e_sync = max_over_ranks(ms_e2e_sync, dist, dev)
    ms_e2e_graph = max_over_ranks(ms_e2e_graph, dist, dev)
    e2e_value = world * STEP_BYTES / (ms_e2e / args.steps * 1e-3) / 1e12
    e2e_sync_value = world * STEP_BYTES / (ms_e2e_sync / args.steps * 1e-3) / 1e12
    e2e_graph_value = world * STEP_BYTES / (ms_e2e_graph / args.steps * 1e-3) / 1e12

    clocks = clk.summary()
    peak, peak_kind = _peak_gbs()
    achieved = DECODE_BYTES / (dec_us * 1e-6) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_c2_traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, desc, _ = cpu_baseline_sample(seconds_budget=15.0)
        cpu = {"value": v, "unit": "TB/s", "cores": os.cpu_count(), "kind": "port", "sample": desc, **_cpu_info()}

    if rank == 0:
        line = {
            "metric": "decode-attn achieved HBM TB/s (% of B200 peak) + us/step; append tokens/s",
            "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16/int4->fp32", "data": "synthetic (seeded N(0,1), random page permutation)",
            "config": _config(),
            "us_per_step": step_ms * 1e3,
            "decode_us": dec_us, "decode_tbs": DECODE_BYTES / (dec_us * 1e-6) / 1e12,
            "decode_pct_of_8tbs": 100 * DECODE_BYTES / (dec_us * 1e-6) / 1e12 / SPEC_TBS,
            "decode_pct_of_measured": 100 * achieved / peak,
            "append_us": app_us, "append_tokens_per_s": world * B / (app_us * 1e-6),
            "prefill_append": {"config": "BASELINE config 5b: 8 x 8192 tokens, Hkv 8, D 128",
                               "us": pf_us, "tbs": world * PF_BYTES / (pf_us * 1e-6) / 1e12,
                               "pct_of_measured": 100 * PF_BYTES / (pf_us * 1e-6) / 1e9 / _peak_gbs()[0],
                               "tokens_per_s": world * PF_S * PF_L / (pf_us * 1e-6), "bytes": PF_BYTES},
            "config5a_append": {"config": "BASELINE config 5a: 2048 sequences x 1 token, Hkv 1, D 128, "
                                          "positions ~U[0, 32768)",
                                "us": a5_us, "tbs": world * A5_BYTES / (a5_us * 1e-6) / 1e12,
                                "tokens_per_s": world * A5_T / (a5_us * 1e-6), "bytes": A5_BYTES},
            "config4_split_context": {
                "config": "BASELINE config 4: 16 x 131072 tokens, Hq 64, Hkv 8, D 128, 8192-token splits dealt "
                          "over the ranks; each rank's cache holds only its splits",
                "us": c4_us, "tbs": C4_BYTES / (c4_us * 1e-6) / 1e12, "bytes": C4_BYTES,
                "collective": "one NCCL all_gather_into_tensor of packed (O, lse) fp32 per step" if world > 1
                              else "none (one GPU)"},
            "fp16_decode_c2": {
                "config": "matched FP16 paged decode on the config-2 shape (64 x 4096, Hq 32, Hkv 8, D 128)",
                "us": f16_us, "tbs": FP16_BYTES / (f16_us * 1e-6) / 1e12, "bytes": FP16_BYTES,
                "int4_speedup": f16_us / dec_us},
            "config3_sharded": {
                "config": "BASELINE config 3: 128 sequences, L ~ U[1,16384] (seed 1), Hq = Hkv = 16, D 64; "
                          "whole sequences sharded over the ranks by token count, no collective",
                "us": c3_us, "tbs": c3_total / (c3_us * 1e-6) / 1e12, "bytes": c3_total},
            "step_bytes": STEP_BYTES, "decode_bytes": DECODE_BYTES, "append_bytes": APPEND_BYTES,
            "e2e": {"value": e2e_value, "unit": "TB/s", "ms_per_step": ms_e2e / args.steps,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "validation": "deferred, errors raised once per step (iris_kernel.check_errors)"},
            "e2e_sync": {"value": e2e_sync_value, "unit": "TB/s", "ms_per_step": ms_e2e_sync / args.steps,
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "validation": "synchronous: every call reads the error word before returning"},
            "e2e_graph": {"value": e2e_graph_value, "unit": "TB/s", "ms_per_step": ms_e2e_graph / args.steps,
                          "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                          "validation": "deferred, errors raised once per step; the two calls replayed from a "
                                        "CUDA graph captured once"},
            "gpu_launches": 3 * args.steps,  # decode, combine, append (a 64-token batch validates itself)
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "decode (decode + combine launches) timed alone from a CUDA graph"},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del g_step, g_dec, g_app
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
