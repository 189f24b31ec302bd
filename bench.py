"""Benchmark of the bitcache decode-attention hot path on B200.

Metric: decode-attention cache GB/s (and % of HBM peak) and
us/step at S=65536, H=32, d=128 -- workload C3 (B=1, H=32, S=65536, d=128,
compensated attention, K/V ~ N(0, 1/128) with 1% outlier channels x8).
A step is one decode-attention pass over the whole cache.  GB/s counts the
algorithmic cache bytes 2*B*Hkv*S*82 (the reference README's 82-byte
binary+INT4 footprint per vector at d=128), read once per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one rank per GPU, NCCL): --split heads (default) shards the
KV heads across ranks with no data-path collective; --split seq splits every
head's positions across ranks and merges the per-rank log-sum-exp triples
after an NCCL all-gather.  The total workload is fixed (strong scaling).

--impl reference runs the reference algorithm on the host cores (the C
restatement of the reference kernels under oracle/, OpenMP over heads; the
reference ships no CPU code of its own) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="C3", choices=["C1", "C2", "C3", "C4", "C5"])
    ap.add_argument("--split", default="heads", choices=["heads", "seq", "seqx"],
                    help="N>1: shard heads, split the sequence with an NCCL all-gather + merge (seq), or split "
                         "the sequence with the kernel's own peer-memory exchange (seqx)")
    ap.add_argument("--binary", action="store_true", help="binary-only attention instead of compensated")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--cpu-sample-s", type=float, default=12.0)
    ap.add_argument("--profile", action="store_true",
                    help="small profiling run: one cache copy, only the decode kernel, warmup+steps launches")
    ap.add_argument("--profile-seq", type=int, default=0,
                    help="with --profile: override the config's sequence length (a smaller capture)")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_from_profiles(workload: str, world: int) -> float | None:
    """Per-launch DRAM bytes from the committed ncu summary of this workload, if any."""
    p = os.path.join(ROOT, "profiles", f"decode_planes_{workload}.md")
    if not os.path.exists(p) or world != 1:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is busy."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# Reference arm: the reference algorithm on the host cores
# ---------------------------------------------------------------------------
def cpu_workload_planes(cfg: str, heads: int | None = None):
    """Workload on the host, encoded by the C oracle (no GPU kernels involved)."""
    from bitcache_b200 import workloads
    from oracle import oracle as O

    w = workloads.make(cfg, device="cpu")
    if heads is not None:
        w.k, w.v, w.q = w.k[:, :heads], w.v[:, :heads], w.q[:, :heads]
    n_slots = w.k.shape[0] * w.k.shape[1]
    S, d = w.seq_len, w.head_dim

    def enc(x):
        xs = x.reshape(-1, d).numpy()
        words, bs = O.binary_encode(xs)
        nib, rs, _ = O.residual_encode(xs, words, bs)
        return {"words": words.reshape(n_slots, S, d // 32), "bscale": bs.reshape(n_slots, S),
                "nib": nib.reshape(n_slots, S, d // 2), "rscale": rs.reshape(n_slots, S)}

    K, V = enc(w.k), enc(w.v)
    q = w.q.reshape(-1, d).numpy()
    return w, q, K, V


def time_cpu_steps(q, K, V, group, S, comp, n_steps, nthreads):
    from oracle import oracle as O

    t0 = time.perf_counter()
    for _ in range(n_steps):
        O.attention(q, K, V, group, S, S, comp, nthreads)
    return time.perf_counter() - t0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from bitcache_b200 import workloads
    from oracle import oracle as O

    comp = not args.binary
    w, q, K, V = cpu_workload_planes(args.config)
    threads = O.num_threads()
    S, d = w.seq_len, w.head_dim
    used = min(threads, q.shape[0])  # the port parallelises over query heads
    bytes_step = workloads.step_cache_bytes(w.batch, w.n_kv_heads, S, d, comp)
    if comp and args.config == "C5":  # adaptive config: the same byte model as our arm
        bytes_step = workloads.adaptive_step_bytes(w.batch, w.n_kv_heads, S, d, w.extra.get("keep", 0.25))
    for _ in range(max(0, args.warmup)):
        time_cpu_steps(q, K, V, w.group, S, comp, 1, threads)
    t = time_cpu_steps(q, K, V, w.group, S, comp, args.steps, threads)
    ms = t * 1e3 / args.steps
    gbs = bytes_step / (ms * 1e-3) / 1e9
    line = {
        "impl": "reference", "metric": "decode-attention cache GB/s", "value": gbs, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak" if args.split == "heads" else "strong", "vs_baseline": None,
        "dtype": "u32/u8 codes, f32 accumulate",
        "data": "synthetic (seeded torch generator)",
        "config": {"workload": f"{args.config}: B={w.batch} H={w.n_heads} Hkv={w.n_kv_heads} S={S} d={d} "
                               f"{'compensated' if comp else 'binary'}", "layout": "planes (host arrays)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": used, "kind": "port",
                         "sample": f"{args.steps} full decode steps of {args.config} (all heads, all positions)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_profile(args):
    """Minimal run for ncu: one cache copy of the workload (> L2), fp16 inputs freed,
    then warmup + steps launches of the decode kernel and nothing else."""
    from bitcache_b200 import planes, workloads

    dev = torch.device("cuda", 0)
    comp = not args.binary
    w = workloads.make(args.config, device=dev, **({"seq_len": args.profile_seq} if args.profile_seq else {}))
    S, d, n = w.seq_len, w.head_dim, w.n_slots
    K = planes.Planes.empty(n, planes.round_stride(S), d, comp, dev, zero=False)
    V = planes.Planes.empty(n, planes.round_stride(S), d, comp, dev, zero=False)
    rm = planes.RES_FP16_SCALE if comp else planes.RES_NONE
    planes.encode_planes(w.k.reshape(n, S, d), K, rm)
    planes.encode_planes(w.v.reshape(n, S, d), V, rm)
    q = w.q.reshape(-1, d).contiguous()
    w_extra = dict(w.extra)
    del w
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    out = torch.empty((q.shape[0], d), dtype=torch.float16, device=dev)
    keep_frac = w_extra.get("keep") if (comp and args.config == "C5") else None
    if keep_frac is not None:  # C5: the compact adaptive cache and its decode
        n_keep = planes.keep_count(S, keep_frac)
        keep = planes.select_positions_topk(K, V, S, n_keep)
        K, V = planes.compact_adaptive(K, V, keep, S, n_keep)
        del keep
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        for _ in range(args.warmup + args.steps):
            planes.decode_attention_adaptive(q, K, V, S, n_keep, out=out)
        nbytes = workloads.adaptive_step_bytes(1, n, S, d, keep_frac)
    else:
        for _ in range(args.warmup + args.steps):
            planes.decode_attention(q, K, V, S, mode, out=out)
        nbytes = workloads.step_cache_bytes(1, n, S, d, comp)
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.config, "launches": args.warmup + args.steps, "bytes_per_launch": nbytes}))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.profile:
        run_profile(args)
        return

    from bitcache_b200 import BitCache, _lib, planes, workloads
    from bitcache_b200 import dist as bdist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep rank 0's stdout to the one JSON line
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = tdist
    comp = not args.binary
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    res_mode = planes.RES_FP16_SCALE if comp else planes.RES_NONE

    # Head sharding (the default) is weak scaling: heads are independent, so
    # every rank holds a full config-sized shard of a global batch N times the
    # config's (rank 0's data is the single-GPU workload) and no collective
    # runs on the data path.  The sequence splits divide one config-sized
    # workload across the ranks (strong scaling) and merge across GPUs.
    weak = args.split == "heads"
    w = workloads.make(args.config, device=dev,
                       seed=None if (rank == 0 or not weak) else 1000 * rank + 7)
    S, d, G = w.seq_len, w.head_dim, w.group
    n_slots = w.n_slots
    if world > 1 and args.split == "heads":
        a, b = 0, n_slots
        s_a, s_b = 0, S
    elif world > 1:
        a, b = 0, n_slots
        s_a, s_b = bdist.seq_range(S, world, rank)
    else:
        a, b, s_a, s_b = 0, n_slots, 0, S
    my_slots, my_S = b - a, s_b - s_a
    k_all = w.k.reshape(n_slots, S, d)[a:b, s_a:s_b].contiguous()
    v_all = w.v.reshape(n_slots, S, d)[a:b, s_a:s_b].contiguous()
    q_all = w.q.reshape(n_slots * G, d)[a * G:b * G].contiguous()
    stride = planes.round_stride(my_S)
    # C5 is the adaptive-precision config: the residual is kept for a fraction of
    # the positions (compact layout, unkept residuals neither stored nor read)
    keep_frac = w.extra.get("keep") if (comp and args.config == "C5") else None
    adaptive = keep_frac is not None
    n_keep = planes.keep_count(my_S, keep_frac) if adaptive else my_S
    if adaptive:
        bytes_rank = workloads.adaptive_step_bytes(1, my_slots, my_S, d, keep_frac)
        bytes_total = workloads.adaptive_step_bytes(w.batch, w.n_kv_heads, S, d, keep_frac)
    else:
        bytes_rank = workloads.step_cache_bytes(1, my_slots, my_S, d, comp)
        bytes_total = workloads.step_cache_bytes(w.batch, w.n_kv_heads, S, d, comp)
    if weak:
        bytes_total *= world
    # Inputs larger than L2: rotate through enough cache copies that one step's
    # data is evicted before it is read again.
    copies = max(1, math.ceil(3 * L2_BYTES / max(1, bytes_rank)))
    Ks, Vs = [], []
    for _ in range(copies):
        K = planes.Planes.empty(my_slots, stride, d, comp, dev, zero=False)
        V = planes.Planes.empty(my_slots, stride, d, comp, dev, zero=False)
        planes.encode_planes(k_all, K, res_mode)
        planes.encode_planes(v_all, V, res_mode)
        if adaptive:
            keep = planes.select_positions_topk(K, V, my_S, n_keep)
            K, V = planes.compact_adaptive(K, V, keep, my_S, n_keep)
            del keep
            torch.cuda.empty_cache()
        Ks.append(K)
        Vs.append(V)
    torch.cuda.synchronize()
    out = torch.empty((my_slots * G, d), dtype=torch.float16, device=dev)
    part = torch.empty((my_slots * G, d + 2), dtype=torch.float32, device=dev)
    seq_split = world > 1 and args.split == "seq"
    xchg = bdist.PeerExchange(my_slots * G, d) if (world > 1 and args.split == "seqx") else None

    def step(i):
        K, V = Ks[i % copies], Vs[i % copies]
        if adaptive:
            planes.decode_attention_adaptive(q_all, K, V, my_S, n_keep, out=out)
        elif xchg is not None:
            xchg.decode(q_all, K, V, my_S, mode, out=out)
        elif seq_split:
            planes.decode_attention(q_all, K, V, my_S, mode, partial=part, want_out=False)
        else:
            planes.decode_attention(q_all, K, V, my_S, mode, out=out)

    gather = bdist.nccl_all_gather() if seq_split else None

    def full_step(i):
        step(i)
        if seq_split:
            planes.lse_merge(gather(part), out=out)

    def barrier():
        if pg is not None:
            pg.barrier()

    for i in range(max(3, args.warmup)):
        full_step(i)
    torch.cuda.synchronize()
    barrier()

    # clocks sampled over a busy window that contains the timed region
    sampler = ClockSampler(local)
    sampler.start()
    t_busy = time.perf_counter()
    i = 0
    while time.perf_counter() - t_busy < 0.6:
        for _ in range(50):
            full_step(i)
            i += 1
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    # Timed region: K steps back to back on the stream.  The GPU first runs a
    # short spin (outside the region) so that the host has queued the steps
    # before they start; consecutive decode launches then overlap their
    # ramp-up with the previous step's tail (programmatic dependent launch).
    tot0, tot1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(40_000_000)
    tot0.record(stream)
    for j in range(args.steps):
        full_step(i + j)
    tot1.record(stream)
    torch.cuda.synchronize()
    barrier()
    i += args.steps
    # Kernel duration for the roofline: the same steps, each launch bracketed
    # by its own events (isolated launches, no overlap with a neighbour).
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda._sleep(40_000_000)
    for j in range(args.steps):
        starts[j].record(stream)
        step(i + j)
        ends[j].record(stream)
        if seq_split:
            planes.lse_merge(gather(part), out=out)
    torch.cuda.synchronize()
    barrier()
    i += args.steps
    t_busy = time.perf_counter()
    while time.perf_counter() - t_busy < 0.4:
        for _ in range(50):
            full_step(i)
            i += 1
        torch.cuda.synchronize()
    clocks = sampler.stop()
    iso_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    step_ms = tot0.elapsed_time(tot1) / args.steps
    if pg is not None:
        t = torch.tensor([step_ms, iso_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        step_ms, iso_ms = float(t[0]), float(t[1])
    # The kernel's average launch duration: over the timed region when each
    # step is that one launch (its duration there matches ncu's per-launch
    # gpu__time_duration); with a separate merge launch per step, the
    # isolated-launch events, which also count the launch gap.
    kern_ms = iso_ms if seq_split else step_ms
    assert _lib.device_error() == 0, "device-side timeout during the benchmark"

    # ---- end to end through the public API (pinned host buffers) ----------
    e2e = None
    if adaptive:
        # adaptive cache (snapshot after selection): pinned host Q in, output out
        qh = q_all.cpu().pin_memory()
        oh = torch.empty(q_all.shape, dtype=torch.float16).pin_memory()
        qd = torch.empty_like(q_all)
        Kc, Vc = Ks[0], Vs[0]

        def e2e_step():
            qd.copy_(qh, non_blocking=True)
            o = planes.decode_attention_adaptive(qd, Kc, Vc, my_S, n_keep)
            oh.copy_(o, non_blocking=True)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        if pg is not None:
            t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            e2e_ms = float(t[0])
        e2e = {"value": bytes_total / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": qh.numel() * 2 * world, "d2h_bytes_per_step": oh.numel() * 2 * world,
               "path": "planes.decode_attention_adaptive on the compact cache, pinned host Q in, output out",
               "gpu_launches_per_step": 1}
    elif world == 1 or args.split == "heads":
        cache = BitCache(w.batch if world == 1 else 1, my_slots * G if world > 1 else w.n_heads, d, max_seq=my_S,
                         device=str(dev), compensated=comp, n_kv_heads=my_slots if world > 1 else w.n_kv_heads)
        cache.prefill(k_all.view(cache.batch, cache.n_kv_heads, my_S, d), v_all.view(cache.batch, cache.n_kv_heads, my_S, d))
        del k_all, v_all
        # Pinned host Q, K, V and output: the fused step kernel reads the inputs
        # and writes the output over the host link itself (one launch per step).
        nq, nkv = cache.batch * cache.n_heads * d, cache.batch * cache.n_kv_heads * d
        host_in = torch.empty(nq + 2 * nkv, dtype=torch.float16).pin_memory()
        host_in[:nq] = q_all.reshape(-1).cpu()
        host_in[nq:] = (torch.randn(2 * nkv) / math.sqrt(d)).half()
        oh = torch.empty((cache.batch, cache.n_heads, d), dtype=torch.float16).pin_memory()
        qh = host_in[:nq].view(cache.batch, cache.n_heads, d)
        kh = host_in[nq:nq + nkv].view(cache.batch, cache.n_kv_heads, d)
        vh = host_in[nq + nkv:].view(cache.batch, cache.n_kv_heads, d)

        def e2e_step():
            cache.step(qh, kh, vh, out=oh)  # append + attend, one launch, host operands

        for _ in range(max(3, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        if pg is not None:
            t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            e2e_ms = float(t[0])
        h2d = host_in.numel() * 2 * world
        d2h = oh.numel() * 2 * world
        # the cache in the e2e leg is one copy: its reads may partly hit L2 when it is small
        e2e = {"value": bytes_total / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "BitCache.step (fused append + attend, one launch) on pinned host Q/K/V and output, "
                       "which the kernel reads and writes over the host link",
               "gpu_launches_per_step": 1}

    # ---- prefill encode throughput (fused binary + INT4 residual into planes) ----
    prefill = None
    if rank == 0:
        Kp = planes.Planes.empty(my_slots, stride, d, comp, dev, zero=False)
        src = w.k.reshape(n_slots, S, d)[a:b, s_a:s_b].contiguous()
        for _ in range(3):
            planes.encode_planes(src, Kp, res_mode)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_enc = 10
        p0.record(stream)
        for _ in range(n_enc):
            planes.encode_planes(src, Kp, res_mode)
        p1.record(stream)
        torch.cuda.synchronize()
        enc_ms = p0.elapsed_time(p1) / n_enc
        enc_bytes = src.numel() * 2 + my_slots * my_S * planes.vector_bytes(d, comp)
        prefill = {"value": enc_bytes / (enc_ms * 1e-3) / 1e9, "unit": "GB/s", "ms": enc_ms,
                   "vectors": my_slots * my_S, "bytes": enc_bytes, "kernel": "k_encode_planes",
                   "frac": enc_bytes / (enc_ms * 1e-3) / 1e9 / peaks()[0]}
        del Kp, src

    hbm, peak_kind = peaks()
    achieved = bytes_rank / (kern_ms * 1e-3) / 1e9
    # the committed summaries profile the compensated kernel of each workload
    traffic = traffic_from_profiles(args.config, world) if comp else None
    value = bytes_total / (step_ms * 1e-3) / 1e9

    line = {
        "metric": "decode-attention cache GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3,
        "higher_is_better": True, "scaling": "weak" if weak else "strong", "vs_baseline": None,
        "dtype": "u32 sign words, u8 INT4 codes, f32 accumulate (fp16 in/out)",
        "data": "synthetic (seeded torch generator, BASELINE config shapes)",
        "config": {"workload": f"{args.config}: B={w.batch} H={w.n_heads} Hkv={w.n_kv_heads} S={S} d={d} "
                               + (f"adaptive, residual kept for {keep_frac:.0%} of positions (compact layout)"
                                  if adaptive else ('compensated' if comp else 'binary')),
                   "parallelism": ((f"heads sharded x{world}: each rank a full {args.config} shard, "
                                    f"global batch {world}x the config's" if weak else f"{args.split}-split x{world}")
                                   if world > 1 else "single GPU"),
                   "l2": f"inputs larger than L2: {copies} rotating cache copies of {bytes_rank / 1e6:.1f} MB per rank",
                   "timing": "K steps back to back between two CUDA events (host queued ahead); "
                             "roofline kernel time = the timed region per launch (one launch per step), "
                             "isolated_launch_us from a second pass with events around each launch",
                   "bytes_per_vector": (bytes_total / (2 * w.batch * w.n_kv_heads * S)) if adaptive
                   else workloads.vector_footprint(d, comp),
                   "stored_bytes_per_vector": planes.vector_bytes(d, comp)},
        "pct_of_hbm_peak": 100.0 * value / world / hbm,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": traffic, "kernel": "k_decode_planes",
                     "kernel_us": kern_ms * 1e3, "isolated_launch_us": iso_ms * 1e3, "achieved_84B": achieved * planes.vector_bytes(d, comp) /
                     workloads.vector_footprint(d, comp)},
        "clocks": clocks,
        "gpu_launches": args.steps * (2 if seq_split else 1),
        "e2e": e2e,
        "prefill_encode": prefill,
    }

    if rank == 0 and world == 1 and not args.no_ref_gpu:
        line["ref_gpu"] = reference_gpu(w, comp, dev, bytes_total)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, comp, bytes_total)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if xchg is not None:
        xchg.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def reference_gpu(w, comp, dev, bytes_total):
    """The reference's own CUDA kernel (recompiled for sm_100a) on the same workload, record format."""
    try:
        from bitcache_b200 import _C
        from oracle import refgpu
    except Exception as e:  # pragma: no cover
        return {"unavailable": str(e)}
    if not refgpu.available():
        return {"unavailable": "oracle/_ref not built"}
    d, H = w.head_dim, w.n_slots
    S = w.seq_len
    k = w.k.reshape(-1, d)
    v = w.v.reshape(-1, d)
    kb = refgpu.binary_encode(k)
    vb = refgpu.binary_encode(v)
    kr = refgpu.residual_encode(k, kb) if comp else None
    vr = refgpu.residual_encode(v, vb) if comp else None
    q = w.q.reshape(-1, d)
    refgpu.attention(q, kb, vb, kr, vr, 1, H, S, d)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 2
    e0.record()
    for _ in range(n):
        refgpu.attention(q, kb, vb, kr, vr, 1, H, S, d)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    return {"value": bytes_total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "kind": "reference CUDA kernels (src/*.cu) compiled for sm_100a, record layout, iterations=2"}


def cpu_baseline(args, comp, bytes_total):
    from oracle import oracle as O

    w, q, K, V = cpu_workload_planes(args.config)
    threads = O.num_threads()
    t1 = time_cpu_steps(q, K, V, w.group, w.seq_len, comp, 1, threads)
    n = max(1, int(args.cpu_sample_s / max(t1, 1e-3)))
    t = time_cpu_steps(q, K, V, w.group, w.seq_len, comp, n, threads)
    ms = t * 1e3 / n
    return {"value": bytes_total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "cores": min(threads, q.shape[0]),
            "kind": "port", "sample": f"{n} full decode steps of {args.config} on the host (OpenMP over heads)"}


if __name__ == "__main__":
    main()
