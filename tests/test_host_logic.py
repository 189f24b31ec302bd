"""CPU: host-side logic -- workload generators, shard planning, the log-sum-exp
merge, and the sequence-split step over gloo with world_size 2."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bitcache_b200 import dist as bdist
from bitcache_b200 import workloads
from oracle import oracle as O


def test_workloads_deterministic_and_shaped():
    a = workloads.make("C1")
    b = workloads.make("C1")
    assert torch.equal(a.k, b.k) and torch.equal(a.q, b.q)
    assert a.q.shape == (1, 8, 128) and a.k.shape == (1, 8, 1024, 128) and a.k.dtype == torch.float16
    std = a.k.float().std().item()
    assert abs(std - 1 / np.sqrt(128)) < 0.01
    c2 = workloads.make("C2", seq_len=256)  # correlated keys present
    qh = c2.q[0, 0].float()
    corr = (c2.k[0, 0].float() @ qh) / (c2.k[0, 0].float().norm(dim=1) * qh.norm())
    assert (corr > 0.1).sum() >= 16


def test_c3_outlier_channels():
    w = workloads.make("C3", seq_len=512, n_heads=2, n_kv_heads=2)
    per_ch = w.k[0, 0].float().std(dim=0)
    assert (per_ch > 4 / np.sqrt(128)).sum() == 2


def test_c5_student_t_variance():
    w = workloads.make("C5", batch=1, n_heads=2, n_kv_heads=2, seq_len=4096, head_dim=64)
    var = w.k.float().var().item()
    assert abs(var - 1 / 64) < 0.002


@pytest.mark.parametrize("seq_len,world", [(65536, 8), (65536, 3), (1000, 4), (7, 2), (0, 2)])
def test_seq_range_partition(seq_len, world):
    rs = [bdist.seq_range(seq_len, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == seq_len
    for (a, b), (c, _) in zip(rs, rs[1:]):
        assert b == c
    for a, _ in rs:
        assert a % 8 == 0 or a == seq_len


@pytest.mark.parametrize("n,world", [(32, 8), (33, 8), (5, 8), (128, 3)])
def test_slot_range_partition(n, world):
    rs = [bdist.slot_range(n, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == n
    sizes = [b - a for a, b in rs]
    assert max(sizes) - min(sizes) <= 1


def _attn_partial_np(q, k, v):
    """float64 partial triple (m, l, o) of exact attention of q [H, d] over k, v [H, S, d]."""
    d = q.shape[-1]
    s = np.einsum("hd,hsd->hs", q, k) / np.sqrt(d)
    if s.shape[1] == 0:
        return np.concatenate([np.full((q.shape[0], 1), -np.inf), np.zeros((q.shape[0], 1 + d))], 1)
    m = s.max(1)
    e = np.exp(s - m[:, None])
    return np.concatenate([m[:, None], e.sum(1)[:, None], np.einsum("hs,hsd->hd", e, v)], 1)


def test_lse_merge_equals_unsplit():
    rng = np.random.default_rng(0)
    H, S, d = 4, 1000, 64
    q = rng.standard_normal((H, d))
    k = rng.standard_normal((H, S, d))
    v = rng.standard_normal((H, S, d))
    full = _attn_partial_np(q, k, v)
    want = full[:, 2:] / full[:, 1:2]
    cuts = [0, 100, 101, 512, 1000, 1000]  # includes an empty part
    parts = np.stack([_attn_partial_np(q, k[:, a:b], v[:, a:b]) for a, b in zip(cuts, cuts[1:])])
    got = O.lse_merge(parts.astype(np.float32))
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
    got_t = bdist.merge_partials_torch(torch.from_numpy(parts)).numpy()
    np.testing.assert_allclose(got_t, want, rtol=1e-5, atol=1e-6)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _seq_split_worker(rank, world, port, q, k, v, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = k.shape[1]
        a, b = bdist.seq_range(S, world, rank)

        def local(qq):
            return torch.from_numpy(_attn_partial_np(qq.numpy(), k[:, a:b], v[:, a:b]))

        def gather(t):
            lst = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(lst, t)
            return torch.stack(lst)

        step = bdist.SeqSplitStep(local, gather, bdist.merge_partials_torch)
        out = step(torch.from_numpy(q))
        out_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def test_seq_split_gloo_world2():
    rng = np.random.default_rng(1)
    H, S, d = 3, 77, 32
    q = rng.standard_normal((H, d))
    k = rng.standard_normal((H, S, d))
    v = rng.standard_normal((H, S, d))
    full = _attn_partial_np(q, k, v)
    want = full[:, 2:] / full[:, 1:2]
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seq_split_worker, args=(r, 2, port, q, k, v, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out_q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        np.testing.assert_allclose(res[r], want, rtol=1e-4, atol=1e-5)


def test_oracle_topk_selection_matches_numpy():
    """The oracle's per-vector selection equals a stable numpy sort on the same keys."""
    rng = np.random.default_rng(3)
    slots, S, d = 2, 200, 64
    nib = rng.integers(0, 256, (slots, S, d // 2), dtype=np.uint8)
    nib[:, 50:60] = nib[:, 5:6]  # ties
    rs = (rng.random((slots, S)) * 0.5).astype(np.float16)
    rs[:, 50:60] = rs[:, 5:6]
    keep = O.select_residual_topk(nib, rs.view(np.uint16), S, 37)
    lo = (nib & 0x0F).astype(np.int64)
    hi = (nib >> 4).astype(np.int64)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    ss = (lo * lo + hi * hi).sum(-1)
    rr = rs.astype(np.float32) * rs.astype(np.float32)
    key = (rr * ss.astype(np.float32)).astype(np.float32)
    for j in range(slots):
        order = sorted(range(S), key=lambda s: (-key[j, s], s))
        want = np.zeros(S, np.uint8)
        want[order[:37]] = 1
        assert np.array_equal(keep[j], want)


def test_oracle_joint_selection_matches_bruteforce():
    rng = np.random.default_rng(9)
    slots, S, d = 2, 150, 32
    kn = rng.integers(0, 256, (slots, S, d // 2), dtype=np.uint8)
    vn = rng.integers(0, 256, (slots, S, d // 2), dtype=np.uint8)
    kn[:, 40:50] = kn[:, 3:4]
    vn[:, 40:50] = vn[:, 3:4]
    kr = (rng.random((slots, S)) * 0.5).astype(np.float16)
    vr = (rng.random((slots, S)) * 0.5).astype(np.float16)
    kr[:, 40:50] = kr[:, 3:4]
    vr[:, 40:50] = vr[:, 3:4]
    keep = O.select_positions_topk(kn, kr.view(np.uint16), vn, vr.view(np.uint16), S, 33)
    key = (O.residual_keys(kn, kr.view(np.uint16)) + O.residual_keys(vn, vr.view(np.uint16))).astype(np.float32)
    for j in range(slots):
        order = sorted(range(S), key=lambda s: (-float(key[j, s]), s))
        want = np.zeros(S, np.uint8)
        want[order[:33]] = 1
        assert np.array_equal(keep[j], want)


def test_bench_job_partition_and_shared_config():
    """bench.py: C3 splits the sequence across GPUs by default, the batched
    configurations shard heads; both arms print the same config dict."""
    import sys
    from types import SimpleNamespace

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    def args(cfg, split="auto"):
        return SimpleNamespace(config=cfg, head_dim=0, split=split, binary=False)

    assert bench.resolve_split(args("C3"), 1) == "none"
    assert bench.resolve_split(args("C3"), 8) == "seqx"
    assert bench.resolve_split(args("C4"), 8) == "heads"
    assert bench.resolve_split(args("C3", "seq"), 2) == "seq"
    for world in (1, 2, 8):
        jobs = [bench.Job(args("C3"), world, r) for r in range(world)]
        assert sum(j.my_S for j in jobs) == 65536 and all(j.my_slots == 32 for j in jobs)
        assert sum(j.bytes_rank for j in jobs) == jobs[0].bytes_total == 343_932_928
        assert all(j.config() == jobs[0].config() for j in jobs)
    jobs = [bench.Job(args("C4"), 8, r) for r in range(8)]
    assert [j.my_slots for j in jobs] == [16] * 8 and all(j.my_S == 32768 for j in jobs)
    c5 = bench.Job(SimpleNamespace(config="C5", head_dim=256, split="auto", binary=False), 1, 0)
    assert c5.d == 256 and c5.adaptive and "d=256" in c5.config()["workload"]


@pytest.mark.parametrize("d", [32, 64, 96, 128, 160, 256])
def test_nibble_plane_layout(d):
    """The plane's nibble order (include/bitcache_b200.h): every dim once; at the
    by-bit head dims each byte holds bits t and t + 4 (t < 4) of one sign byte b,
    placed by the header's table, so that a 16-byte chunk lines up with one
    16-byte window of the sign row; nib_rows inverts nib_interleave."""
    from bitcache_b200 import planes
    lo, hi = planes._nib_dims(d)
    assert torch.equal(torch.cat([lo, hi]).sort().values, torch.arange(d))
    for p in range(d // 2):
        c, j = p // 16, p % 16
        if planes._by_bit(d):
            b, t = int(lo[p]) // 8, int(lo[p]) % 8
            assert t < 4 and int(hi[p]) == int(lo[p]) + 4
            want = {128: (j, c), 256: (16 * (c // 4) + j, c % 4), 64: (j % 8, 2 * c + j // 8)}[d]
            assert (b, t) == want
            assert b // 16 == (c // 4 if d == 256 else 0)  # the chunk's sign window
        else:
            assert (int(lo[p]), int(hi[p])) == (32 * c + 2 * j, 32 * c + 2 * j + 1)
    g = torch.Generator().manual_seed(d)
    rows = torch.randint(0, 256, (3, 16, d // 2), generator=g, dtype=torch.int64).to(torch.uint8)
    assert torch.equal(planes.nib_rows(planes.nib_interleave(rows, d), d), rows)
