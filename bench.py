"""Benchmark of the bitcache decode-attention hot path on B200.

Metric: decode-attention cache GB/s (and % of HBM peak) and
us/step at S=65536, H=32, d=128 -- workload C3 (B=1, H=32, S=65536, d=128,
compensated attention, K/V ~ N(0, 1/128) with 1% outlier channels x8).
A step is one decode-attention pass over the whole cache.  GB/s counts the
algorithmic cache bytes 2*B*Hkv*S*82 (the reference README's 82-byte
binary+INT4 footprint per vector at d=128), read once per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config C1..C5] [--head-dim D] [--split auto|heads|seq|seqx]

N > 1 (torchrun, one rank per GPU): the configuration's workload is divided
across the ranks (strong scaling; `value` is the whole job's GB/s, the
per-GPU figure is `gbs_per_gpu`).  --split auto (the default) splits C3, the
single-sequence configuration, along the sequence with the decode kernel's
own peer-memory exchange of the per-rank log-sum-exp triples (seqx); the
batched configurations shard their KV heads (heads, no data-path
collective).  --split seq is the sequence split with an NCCL all-gather of
the triples and a merge launch.

--impl reference runs the reference algorithm on the host cores (the C
restatement of the reference kernels under oracle/, OpenMP over query heads
on every core of the host; the reference ships no CPU code of its own) on
the same workload and config, rank 0 only.  It maps no library of the GPU
path.
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
    ap.add_argument("--head-dim", type=int, default=0, help="override the config's head_dim (C5 sweeps 64/128/256)")
    ap.add_argument("--split", default="auto", choices=["auto", "heads", "seq", "seqx"],
                    help="N>1: shard the KV heads (heads), split the sequence with an NCCL all-gather + merge (seq), "
                         "or split the sequence with the kernel's own peer-memory exchange (seqx); auto: seqx for "
                         "C3, heads otherwise")
    ap.add_argument("--binary", action="store_true", help="binary-only attention instead of compensated")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--cpu-sample-s", type=float, default=12.0)
    ap.add_argument("--profile", action="store_true",
                    help="small profiling run: one cache copy, only the decode kernel, warmup+steps launches")
    ap.add_argument("--profile-seq", type=int, default=0,
                    help="with --profile: override the config's sequence length (a smaller capture)")
    ap.add_argument("--profile-kernel", default="decode",
                    choices=["decode", "encode", "append", "entropy", "select", "compact", "merge", "records"],
                    help="with --profile: the kernel whose launches the run makes (warmup + steps of them)")
    return ap.parse_args()


def resolve_split(args, world: int) -> str:
    if world <= 1:
        return "none"
    if args.split != "auto":
        return args.split
    return "seqx" if args.config == "C3" else "heads"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def workload_overrides(args) -> dict:
    return {"head_dim": args.head_dim} if args.head_dim else {}


def host_threads() -> int:
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def traffic_from_profiles(workload: str, head_dim: int, comp: bool, bytes_rank: float) -> tuple[float | None, str]:
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of this
    workload's kernel from the committed ncu summary, scaled to this run's
    per-rank cache bytes (the kernel reads each vector once, so traffic grows
    in proportion).  Returns (bytes or None, where it came from)."""
    name = f"decode_planes_{workload}" + ("" if comp else "_binary") + ("" if head_dim in (0, 128) else f"_d{head_dim}")
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None, "no committed ncu summary for this workload"
    txt = open(p).read()
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    mb = re.search(r"profiled_cache_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    if not m:
        return None, f"profiles/{name}.md has no traffic line"
    t = float(m.group(1))
    if mb:
        t *= bytes_rank / float(mb.group(1))
    return t, (f"ncu capture of the same kernel and workload (profiles/{name}.md), not measured by this run"
               + ("; scaled to this rank's cache bytes" if mb else ""))


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
# The job: workload shape, per-rank partition, bytes, and the config dict
# (identical in both arms: built from the arguments and the shape alone)
# ---------------------------------------------------------------------------
class Job:
    def __init__(self, args, world: int, rank: int):
        from bitcache_b200 import dist as bdist
        from bitcache_b200 import planes, workloads

        cfg = dict(workloads.CONFIGS[args.config])
        cfg.update(workload_overrides(args))
        self.cfg_name = args.config
        self.batch, self.n_heads, self.n_kv_heads = cfg["batch"], cfg["n_heads"], cfg["n_kv_heads"]
        self.S, self.d = cfg["seq_len"], cfg["head_dim"]
        self.G = self.n_heads // self.n_kv_heads
        self.n_slots = self.batch * self.n_kv_heads
        self.comp = not args.binary
        self.world, self.rank = world, rank
        self.split = resolve_split(args, world)
        self.keep_frac = cfg.get("keep") if (self.comp and args.config == "C5") else None
        self.adaptive = self.keep_frac is not None
        if self.split == "heads":
            self.a, self.b = bdist.slot_range(self.n_slots, world, rank)
            self.s_a, self.s_b = 0, self.S
        elif self.split in ("seq", "seqx"):
            self.a, self.b = 0, self.n_slots
            self.s_a, self.s_b = bdist.seq_range(self.S, world, rank)
        else:
            self.a, self.b, self.s_a, self.s_b = 0, self.n_slots, 0, self.S
        self.my_slots, self.my_S = self.b - self.a, self.s_b - self.s_a
        self.stride = planes.round_stride(self.my_S)
        self.n_keep = planes.keep_count(self.my_S, self.keep_frac) if self.adaptive else self.my_S
        d = self.d
        if self.adaptive:
            self.bytes_rank = workloads.adaptive_step_bytes(1, self.my_slots, self.my_S, d, self.keep_frac)
            self.bytes_total = workloads.adaptive_step_bytes(self.batch, self.n_kv_heads, self.S, d, self.keep_frac)
        else:
            self.bytes_rank = workloads.step_cache_bytes(1, self.my_slots, self.my_S, d, self.comp)
            self.bytes_total = workloads.step_cache_bytes(self.batch, self.n_kv_heads, self.S, d, self.comp)
        # Inputs larger than L2: enough rotating cache copies that one step's
        # data is evicted before it is read again.
        self.copies = max(1, math.ceil(3 * L2_BYTES / max(1, self.bytes_rank)))
        self.bytes_per_vector = ((self.bytes_total / (2 * self.batch * self.n_kv_heads * self.S)) if self.adaptive
                                 else workloads.vector_footprint(d, self.comp))
        self.stored_bytes_per_vector = planes.vector_bytes(d, self.comp)

    def workload_str(self) -> str:
        kind = (f"adaptive, residual kept for {self.keep_frac:.0%} of positions (compact layout)" if self.adaptive
                else ("compensated" if self.comp else "binary"))
        return (f"{self.cfg_name}: B={self.batch} H={self.n_heads} Hkv={self.n_kv_heads} S={self.S} d={self.d} "
                f"{kind}")

    def config(self) -> dict:
        if self.split == "none":
            par = "single GPU"
        elif self.split == "heads":
            par = f"KV heads sharded across {self.world} GPUs (no data-path collective)"
        elif self.split == "seqx":
            par = (f"sequence split across {self.world} GPUs, per-rank (m, l, o) triples exchanged and merged by "
                   f"the decode kernel over peer memory")
        else:
            par = f"sequence split across {self.world} GPUs, NCCL all-gather of (m, l, o) + merge launch"
        return {"workload": self.workload_str(), "parallelism": par,
                "l2": f"inputs larger than L2: {self.copies} rotating cache copies of "
                      f"{self.bytes_rank / 1e6:.1f} MB per rank",
                "bytes_per_vector": self.bytes_per_vector, "stored_bytes_per_vector": self.stored_bytes_per_vector}


# ---------------------------------------------------------------------------
# Reference arm: the reference algorithm on the host cores
# ---------------------------------------------------------------------------
def cpu_workload_planes(cfg: str, overrides: dict):
    """Workload on the host, encoded by the C oracle (no GPU kernels involved)."""
    from bitcache_b200 import workloads
    from oracle import oracle as O

    w = workloads.make(cfg, device="cpu", **overrides)
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
    job = Job(args, world, 0)
    comp = job.comp
    w, q, K, V = cpu_workload_planes(args.config, workload_overrides(args))
    threads = host_threads()
    S = w.seq_len
    used = min(threads, q.shape[0])  # the port parallelises over query heads
    for _ in range(max(0, args.warmup)):
        time_cpu_steps(q, K, V, w.group, S, comp, 1, threads)
    t = time_cpu_steps(q, K, V, w.group, S, comp, args.steps, threads)
    ms = t * 1e3 / args.steps
    gbs = job.bytes_total / (ms * 1e-3) / 1e9
    line = {
        "impl": "reference", "metric": "decode-attention cache GB/s", "value": gbs, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u32 sign words, u8 INT4 codes, f32 accumulate (fp16 in/out)",
        "data": "synthetic (seeded torch generator, BASELINE config shapes)",
        "config": job.config(),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": used, "kind": "port",
                         "sample": f"{args.steps} full decode steps of {args.config} (all heads, all positions) on "
                                   f"rank 0's host, OpenMP over {q.shape[0]} query heads with {threads} threads"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_profile_kernel(args, w, dev):
    """--profile with a kernel other than the decode: warmup + steps launches of it
    on the workload `w` (the encoder, the decode-step append, the reference-API
    entropy, the adaptive selection and compaction, the log-sum-exp merge, the
    reference-record attention), nothing else after the set-up.  Prints the
    algorithmic bytes of one launch."""
    import torch

    from bitcache_b200 import _C, planes, workloads

    S, d, n = w.seq_len, w.head_dim, w.n_slots
    comp = not args.binary
    rm = planes.RES_FP16_SCALE if comp else planes.RES_NONE
    launches = args.warmup + args.steps
    kern = args.profile_kernel
    k = w.k.reshape(n, S, d)
    if kern == "encode":  # k_encode_planes_lpv: fp16 in, planes out
        K = planes.Planes.empty(n, planes.round_stride(S), d, comp, dev, zero=False)
        torch.cuda.synchronize()
        for _ in range(launches):
            planes.encode_planes(k, K, rm)
        nbytes = n * S * (2 * d + planes.vector_bytes(d, comp))
    elif kern == "append":  # k_append_kv: one K and one V token per slot
        K = planes.Planes.empty(n, planes.round_stride(S), d, comp, dev)
        V = planes.Planes.empty(n, planes.round_stride(S), d, comp, dev)
        kv = w.k[:, :, :2].reshape(n, 2, d)
        kt, vt = kv[:, 0].contiguous(), kv[:, 1].contiguous()
        torch.cuda.synchronize()
        for i in range(launches):
            planes.append_kv(kt, vt, K, V, i % S, planes.RES_FP32_SCALE if comp else planes.RES_NONE)
        nbytes = 2 * n * (2 * d + planes.vector_bytes(d, comp))
    elif kern == "entropy":  # k_head_entropy on reference records (the reference API)
        kb = _C.binary_encode(k.reshape(-1, d))
        q = w.q.reshape(-1, d)[:n].contiguous()
        torch.cuda.synchronize()
        for _ in range(launches):
            _C.compute_head_entropy(q.view(1, n, d), kb, 1, n, S, d)
        nbytes = n * S * (d // 8 + 2)  # used record fields: sign words + scale
    elif kern in ("select", "compact"):  # k_select_topk (joint K+V) / k_compact_adaptive
        K = planes.Planes.empty(n, planes.round_stride(S), d, True, dev, zero=False)
        V = planes.Planes.empty(n, planes.round_stride(S), d, True, dev, zero=False)
        planes.encode_planes(k, K)
        planes.encode_planes(w.v.reshape(n, S, d), V)
        n_keep = planes.keep_count(S, w.extra.get("keep", 0.25))
        keep = planes.select_positions_topk(K, V, S, n_keep)
        torch.cuda.synchronize()
        for _ in range(launches):
            if kern == "select":
                planes.select_positions_topk(K, V, S, n_keep)
            else:
                planes.compact_adaptive(K, V, keep, S, n_keep)
        if kern == "select":
            nbytes = 2 * n * S * (d // 2 + 2) + n * S  # residual planes of K and V read, keep mask written
        else:  # K and V planes and the mask read; signs and scales of all, residuals of the kept written
            nbytes = (2 * n * S * planes.vector_bytes(d, True) + n * S
                      + 2 * n * (S * planes.vector_bytes(d, False) + n_keep * (d // 2 + 2)))
    elif kern == "merge":  # k_lse_merge of 8 partial triples per head (an 8-way sequence split)
        heads = w.q.numel() // d
        parts = torch.randn(8, heads, d + 2, device=dev)
        out = torch.empty(heads, d, dtype=torch.float16, device=dev)
        torch.cuda.synchronize()
        for _ in range(launches):
            planes.lse_merge(parts, out=out)
        nbytes = parts.numel() * 4 + out.numel() * 2
    else:  # records: k_decode_records, the reference-layout compensated attention
        kb = _C.binary_encode(k.reshape(-1, d))
        vb = _C.binary_encode(w.v.reshape(-1, d))
        kr = _C.residual_encode(k.reshape(-1, d), kb) if comp else None
        vr = _C.residual_encode(w.v.reshape(-1, d), vb) if comp else None
        q = w.q.reshape(-1, d)[:n].contiguous().view(1, n, d)
        torch.cuda.synchronize()
        for _ in range(launches):
            if comp:
                _C.compensated_attention(q, kb, kr, vb, vr, 1, n, S, d)
            else:
                _C.binary_attention(q, kb, vb, 1, n, S, d)
        nbytes = workloads.step_cache_bytes(1, n, S, d, comp)
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.config, "kernel": kern, "launches": launches, "bytes_per_launch": nbytes}))


def run_profile(args):
    """Minimal run for ncu: one cache copy of the workload (> L2), fp16 inputs freed,
    then warmup + steps launches of the decode kernel and nothing else
    (--profile-kernel picks another kernel)."""
    import torch

    from bitcache_b200 import planes, workloads

    dev = torch.device("cuda", 0)
    comp = not args.binary
    over = workload_overrides(args)
    if args.profile_seq:
        over["seq_len"] = args.profile_seq
    w = workloads.make(args.config, device=dev, **over)
    if args.profile_kernel != "decode":
        run_profile_kernel(args, w, dev)
        return
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

    import torch

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
    job = Job(args, world, rank)
    comp, d, G, S = job.comp, job.d, job.G, job.S
    mode = planes.MODE_COMPENSATED if comp else planes.MODE_BINARY
    res_mode = planes.RES_FP16_SCALE if comp else planes.RES_NONE

    # One workload (same seed on every rank); each rank keeps its share.
    w = workloads.make(args.config, device=dev, **workload_overrides(args))
    a, b, s_a, s_b = job.a, job.b, job.s_a, job.s_b
    my_slots, my_S, stride = job.my_slots, job.my_S, job.stride
    k_all = w.k.reshape(job.n_slots, S, d)[a:b, s_a:s_b].contiguous()
    v_all = w.v.reshape(job.n_slots, S, d)[a:b, s_a:s_b].contiguous()
    q_all = w.q.reshape(job.n_slots * G, d)[a * G:b * G].contiguous()
    adaptive, n_keep, copies = job.adaptive, job.n_keep, job.copies
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
    seq_split = job.split == "seq"
    xchg = bdist.PeerExchange(my_slots * G, d) if job.split == "seqx" else None

    def step(i, qq=q_all, o=out):
        K, V = Ks[i % copies], Vs[i % copies]
        if adaptive:
            planes.decode_attention_adaptive(qq, K, V, my_S, n_keep, out=o)
        elif xchg is not None:
            xchg.decode(qq, K, V, my_S, mode, out=o)
        elif seq_split:
            planes.decode_attention(qq, K, V, my_S, mode, partial=part, want_out=False)
        else:
            planes.decode_attention(qq, K, V, my_S, mode, out=o)

    gather = bdist.nccl_all_gather() if seq_split else None

    def full_step(i, qq=q_all, o=out):
        step(i, qq, o)
        if seq_split:
            planes.lse_merge(gather(part), out=o)

    def barrier():
        if pg is not None:
            pg.barrier()

    def agreed_max(x: float) -> float:
        """The largest value of x over the ranks (every rank gets the same)."""
        if pg is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t[0])

    stream = torch.cuda.current_stream(dev)
    n_warm = max(3, args.warmup)
    for i in range(n_warm):
        full_step(i)
    torch.cuda.synchronize()
    barrier()
    # Every rank must run the same number of steps (the sequence splits wait
    # for all ranks inside each step), so the busy-loop length is agreed once,
    # from the wall time of warm steps.
    t0 = time.perf_counter()
    for j in range(20):
        full_step(n_warm + j)
    torch.cuda.synchronize()
    per_step_s = agreed_max((time.perf_counter() - t0) / 20)
    n_busy = max(50, int(0.6 / max(per_step_s, 1e-6)))
    n_tail = max(50, int(0.4 / max(per_step_s, 1e-6)))
    i = n_warm + 20

    # clocks sampled over a busy window that contains the timed region
    sampler = ClockSampler(local)
    sampler.start()
    for j in range(n_busy):
        full_step(i + j)
    i += n_busy
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
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
    for j in range(n_tail):
        full_step(i + j)
    i += n_tail
    torch.cuda.synchronize()
    clocks = sampler.stop()
    iso_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    step_ms = tot0.elapsed_time(tot1) / args.steps
    step_ms, iso_ms = agreed_max(step_ms), agreed_max(iso_ms)
    # The kernel's average launch duration: over the timed region when each
    # step is that one launch (its duration there matches ncu's per-launch
    # gpu__time_duration); with a separate merge launch per step, the
    # isolated-launch events, which also count the launch gap.
    kern_ms = iso_ms if seq_split else step_ms
    assert _lib.device_error() == 0, "device-side timeout during the benchmark"

    # ---- end to end through the public API (pinned host buffers) ----------
    e2e = None
    if adaptive or job.split in ("seq", "seqx"):
        # pinned host Q in, merged output out, the decode on the device
        qh = q_all.cpu().pin_memory()
        oh = torch.empty(q_all.shape, dtype=torch.float16).pin_memory()
        if seq_split:
            qd = torch.empty_like(q_all)
            od = torch.empty_like(out)

            def e2e_step(j):
                qd.copy_(qh, non_blocking=True)
                full_step(j, qd, od)
                oh.copy_(od, non_blocking=True)

            path = ("planes.decode_attention + NCCL all-gather + planes.lse_merge, pinned host Q copied in and "
                    "the output copied out every step")
        else:
            def e2e_step(j):
                full_step(j, qh, oh)  # Q staged by one bc_stage_rows launch; the kernel writes oh over the host link

            path = ("planes.decode_attention_adaptive on the compact cache" if adaptive
                    else "dist.PeerExchange.decode (one decode launch per rank)")
            path += (" on pinned host Q and output: one staging launch copies Q to the device (bc_stage_rows), "
                     "the decode writes the output over the host link")
        h2d, d2h = qh.numel() * 2 * world, oh.numel() * 2 * world
    else:
        cache = BitCache(1 if world > 1 else job.batch, my_slots * G if world > 1 else job.n_heads, d,
                         max_seq=my_S, device=str(dev), compensated=comp,
                         n_kv_heads=my_slots if world > 1 else job.n_kv_heads)
        cache.prefill(k_all.view(cache.batch, cache.n_kv_heads, my_S, d),
                      v_all.view(cache.batch, cache.n_kv_heads, my_S, d))
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

        def e2e_step(j):
            cache.step(qh, kh, vh, out=oh)  # stage the inputs, then append + attend; host operands

        path = ("BitCache.step on pinned host Q/K/V and output: one staging launch copies the inputs to the "
                "device (bc_stage_rows), then the fused append + attend launch writes the output over the host link")
        h2d, d2h = host_in.numel() * 2 * world, oh.numel() * 2 * world
    del k_all, v_all
    for j in range(n_warm):
        e2e_step(i + j)
    i += n_warm
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(args.steps):
        e2e_step(i + j)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    i += args.steps
    e2e_ms = agreed_max(e0.elapsed_time(e1) / args.steps)
    assert _lib.device_error() == 0, "device-side timeout during the end-to-end leg"
    e2e = {"value": job.bytes_total / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "path": path,
           "gpu_launches_per_step": 2}

    # ---- prefill encode throughput (fused binary + INT4 residual into planes) ----
    prefill = None
    if rank == 0:
        Kp = planes.Planes.empty(my_slots, stride, d, comp, dev, zero=False)
        src = w.k.reshape(job.n_slots, S, d)[a:b, s_a:s_b].contiguous()
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
                   "vectors": my_slots * my_S, "bytes": enc_bytes, "kernel": "k_encode_planes_lpv",
                   "frac": enc_bytes / (enc_ms * 1e-3) / 1e9 / peaks()[0]}
        del Kp, src

    hbm, peak_kind = peaks()
    achieved = job.bytes_rank / (kern_ms * 1e-3) / 1e9
    traffic, traffic_src = traffic_from_profiles(args.config, args.head_dim, comp, job.bytes_rank)
    value = job.bytes_total / (step_ms * 1e-3) / 1e9

    line = {
        "metric": "decode-attention cache GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "us_per_step": step_ms * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u32 sign words, u8 INT4 codes, f32 accumulate (fp16 in/out)",
        "data": "synthetic (seeded torch generator, BASELINE config shapes)",
        "config": job.config(),
        "timing": "K steps back to back between two CUDA events on the launching stream (host queued ahead), "
                  "max over ranks; roofline kernel time = the timed region per launch (one launch per step), "
                  "isolated_launch_us from a second pass with events around each launch",
        "gbs_per_gpu": value / world,
        "pct_of_hbm_peak": 100.0 * value / world / hbm,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": traffic, "traffic_source": traffic_src,
                     "kernel": "k_decode_planes", "kernel_us": kern_ms * 1e3, "isolated_launch_us": iso_ms * 1e3,
                     "bytes_per_launch": job.bytes_rank,
                     "achieved_stored_bytes": achieved * job.stored_bytes_per_vector / job.bytes_per_vector},
        "clocks": clocks,
        "gpu_launches": args.steps * (2 if seq_split else 1),
        "e2e": e2e,
        "prefill_encode": prefill,
    }

    if rank == 0 and world == 1 and not args.no_ref_gpu:
        line["ref_gpu"] = reference_gpu(w, comp, job.bytes_total)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, comp, job.bytes_total)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if xchg is not None:
        xchg.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def reference_gpu(w, comp, bytes_total):
    """The reference's own CUDA kernel (recompiled for sm_100a) on the same workload, record format."""
    import torch

    try:
        from oracle import refgpu
    except Exception as e:  # pragma: no cover
        return {"unavailable": str(e)}
    if not refgpu.available():
        return {"unavailable": "oracle/_ref not built"}
    if w.group != 1:
        return {"unavailable": "the reference kernels have no grouped-query heads"}
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
    w, q, K, V = cpu_workload_planes(args.config, workload_overrides(args))
    threads = host_threads()
    t1 = time_cpu_steps(q, K, V, w.group, w.seq_len, comp, 1, threads)
    n = max(1, int(args.cpu_sample_s / max(t1, 1e-3)))
    t = time_cpu_steps(q, K, V, w.group, w.seq_len, comp, n, threads)
    ms = t * 1e3 / n
    return {"value": bytes_total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "cores": min(threads, q.shape[0]),
            "kind": "port", "sample": f"{n} full decode steps of {args.config} on the host "
                                      f"(OpenMP over {q.shape[0]} query heads, {threads} threads)"}


if __name__ == "__main__":
    main()
