"""GPU, 2+ devices: head sharding and the sequence split (NCCL all-gather of
log-sum-exp triples + bc_lse_merge) reproduce the single-GPU decode.
Each rank is its own process on its own GPU (spawned, NCCL over NVLink);
skipped on single-GPU machines."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, out_q):
    import datetime

    import torch.distributed as dist

    from bitcache_b200 import dist as bdist
    from bitcache_b200 import planes, workloads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        w = workloads.make("C3", device=dev, seq_len=8192, n_heads=8, n_kv_heads=8)
        n, S, d = w.n_slots, w.seq_len, w.head_dim
        q = w.q.reshape(n, d)
        if mode == "heads":
            a, b = bdist.slot_range(n, world, rank)
            K = planes.Planes.empty(b - a, S, d, True, dev)
            V = planes.Planes.empty(b - a, S, d, True, dev)
            planes.encode_planes(w.k.reshape(n, S, d)[a:b].contiguous(), K)
            planes.encode_planes(w.v.reshape(n, S, d)[a:b].contiguous(), V)
            mine = planes.decode_attention(q[a:b].contiguous(), K, V, S)
            full = torch.empty(n, d, dtype=torch.float16, device=dev)
            sizes = [bdist.slot_range(n, world, r) for r in range(world)]
            pieces = [torch.empty(e - s_, d, dtype=torch.float16, device=dev) for s_, e in sizes]
            dist.all_gather(pieces, mine)
            full = torch.cat(pieces)
        elif mode == "xchg":
            a, b = bdist.seq_range(S, world, rank)
            K = planes.Planes.empty(n, planes.round_stride(b - a), d, True, dev)
            V = planes.Planes.empty(n, planes.round_stride(b - a), d, True, dev)
            planes.encode_planes(w.k.reshape(n, S, d)[:, a:b].contiguous(), K)
            planes.encode_planes(w.v.reshape(n, S, d)[:, a:b].contiguous(), V)
            x = bdist.PeerExchange(q.shape[0], d)
            for _ in range(3):  # several epochs through the same buffers
                full = x.decode(q, K, V, b - a, planes.MODE_COMPENSATED)
            torch.cuda.synchronize()
            x.close()
        else:
            a, b = bdist.seq_range(S, world, rank)
            K = planes.Planes.empty(n, planes.round_stride(b - a), d, True, dev)
            V = planes.Planes.empty(n, planes.round_stride(b - a), d, True, dev)
            planes.encode_planes(w.k.reshape(n, S, d)[:, a:b].contiguous(), K)
            planes.encode_planes(w.v.reshape(n, S, d)[:, a:b].contiguous(), V)
            part = torch.empty(n, d + 2, dtype=torch.float32, device=dev)

            def local(qq):
                planes.decode_attention(qq, K, V, b - a, partial=part, want_out=False)
                return part

            step = bdist.SeqSplitStep(local, bdist.nccl_all_gather(), planes.lse_merge)
            full = step(q)
        # single-GPU reference on this rank
        Kf = planes.Planes.empty(n, S, d, True, dev)
        Vf = planes.Planes.empty(n, S, d, True, dev)
        planes.encode_planes(w.k.reshape(n, S, d), Kf)
        planes.encode_planes(w.v.reshape(n, S, d), Vf)
        ref = planes.decode_attention(q, Kf, Vf, S)
        torch.cuda.synchronize()
        out_q.put((rank, float((full.float() - ref.float()).abs().max()),
                   float(torch.nn.functional.cosine_similarity(full.float().flatten(), ref.float().flatten(), dim=0))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "seq", "xchg"])
def test_two_gpu_split_matches_single(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [out_q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, err, cos in res:
        assert err <= 2e-3 and cos >= 0.9999
