"""The multi-GPU split, exchange and merge, checked on CPU with two gloo ranks.

eb_train in a group splits every batch's top-1 into equal slices of
ceil(B / world) positions (emeans_b200.shard_bounds mirrors that split) and
all-gathers the slices' labels and scores. Here each gloo rank scores its
slice with the CPU oracle and all-gathers it; the assembled batch must equal
the oracle over the whole batch, for batch sizes that do not divide evenly.

eb_topk_group ranks each rank's database shard with global ids, all-gathers
the lists and merges them by (larger score, then lower id); here each rank
ranks its shard with the oracle, the lists are all-gathered over gloo and
merged by the same rule (emeans_b200.merge_topk), and the result must equal
the oracle's top-k over the whole database, duplicate rows across the shards
included (equal scores: the lower id wins).

eb_train in group mode 3 (the north-star step) also splits the scatter-add:
each rank sums its slice's rows into partial counts and sums in its share of
the exchange buffer (emeans_b200.reduce_layout mirrors the layout), one
all-gather carries every share, and every rank adds the partials in rank
order and takes the EMA step. Here each gloo rank does the same with the
oracle's ops: both ranks end with the same bits, the counts are exact, and
the sums agree with the single-engine row order to rounding.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import emeans_b200 as eb
import oracle


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_each_position_once():
    for world in (1, 2, 3, 4, 8):
        for b, end in ((0, 16384), (5, 1029), (0, 1), (7, 7), (0, 3)):
            seen = np.zeros(end, int)
            for r in range(world):
                lo, hi = eb.shard_bounds(b, end, r, world)
                assert b <= lo <= hi <= end
                seen[lo:hi] += 1
            assert np.all(seen[b:end] == 1), (world, b, end)


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(5)
        n, d, k = 3001, 24, 37
        x = rng.standard_normal((n, d)).astype(np.float32)
        c = rng.standard_normal((k, d)).astype(np.float32)
        order = rng.permutation(n).astype(np.uint32)
        ok = True
        for b, end in ((0, 1024), (1024, 2047), (2047, 3001)):
            lo, hi = eb.shard_bounds(b, end, rank, world)
            sh = (end - b + world - 1) // world
            stage = np.zeros(2 * sh, np.uint32)
            if hi > lo:
                lab, sco = oracle.top1(x.ravel(), d, c.ravel(), oracle.L2, ids=order[lo:hi])
                stage[:hi - lo] = lab
                stage[sh:sh + hi - lo] = sco.view(np.uint32)
            parts = [torch.zeros(2 * sh, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(stage.astype(np.int64)))
            got_l = np.concatenate([p[:sh].numpy() for p in parts]).astype(np.uint32)[:end - b]
            got_s = np.concatenate([p[sh:].numpy() for p in parts]).astype(np.uint32)[:end - b]
            want_l, want_s = oracle.top1(x.ravel(), d, c.ravel(), oracle.L2, ids=order[b:end])
            ok &= np.array_equal(got_l, want_l) and np.array_equal(got_s, want_s.view(np.uint32))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok)))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, repr(exc)))


def _knn_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(9)
        n, d, m, kk = 2001, 16, 150, 10
        data = rng.standard_normal((n, d)).astype(np.float32)
        data[1500:1520] = data[100:120]  # exact duplicates in the other shard
        queries = np.concatenate([data[:50], rng.standard_normal((m - 50, d)).astype(np.float32)])
        lo, hi = eb.shard_bounds(0, n, rank, world)
        ids, sims = oracle.topk(queries.ravel(), data[lo:hi].ravel(), d, kk)
        ids = np.where(ids == 0xFFFFFFFF, ids, ids + np.uint32(lo)).astype(np.uint32)
        mine = torch.from_numpy(np.concatenate([ids.astype(np.int64),
                                                sims.view(np.uint32).astype(np.int64)]))
        parts = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        lists = []
        for p in parts:
            a = p.numpy()
            lists.append((a[:m * kk].astype(np.uint32),
                          a[m * kk:].astype(np.uint32).view(np.float32)))
        got_i, got_s = eb.merge_topk(lists, kk)
        want_i, want_s = oracle.topk(queries.ravel(), data.ravel(), d, kk)
        ok = np.array_equal(got_i, want_i) and np.array_equal(got_s.view(np.uint32),
                                                              want_s.view(np.uint32))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok)))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, repr(exc)))


def _reduce_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(6)
        n, d, k = 2500, 20, 13
        x = rng.standard_normal((n, d)).astype(np.float32)
        c = rng.standard_normal((k, d)).astype(np.float32)
        order = rng.permutation(n).astype(np.uint32)
        ok, digests = True, []
        pos = c.ravel().copy()
        usage = np.full(k, 1.0 / 65536.0, np.float32)
        for b, end in ((0, 1024), (1024, 2047), (2047, 2500)):
            s, s4, k4, share = eb.reduce_layout(end - b, world, k, d)
            lo, hi = eb.shard_bounds(b, end, rank, world)
            mine = np.zeros(share, np.uint32)
            if hi > lo:
                lab, sco = oracle.top1(x.ravel(), d, pos, oracle.L2, ids=order[lo:hi])
                mine[:hi - lo] = lab
                mine[s4:s4 + hi - lo] = sco.view(np.uint32)
                ps, pc = oracle.scatter_add(x.ravel(), d, lab, k, ids=order[lo:hi])
            else:
                ps, pc = np.zeros(k * d, np.float32), np.zeros(k, np.uint32)
            mine[2 * s4:2 * s4 + k] = pc
            mine[2 * s4 + k4:] = ps.view(np.uint32)
            parts = [torch.zeros(share, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(mine.astype(np.int64)))
            sh = [p.numpy().astype(np.uint32) for p in parts]
            got_l = np.concatenate([a[:s] for a in sh])[:end - b]
            got_s = np.concatenate([a[s4:s4 + s] for a in sh])[:end - b].view(np.float32)
            sums = sh[0][2 * s4 + k4:].view(np.float32).copy()
            for a in sh[1:]:
                sums = (sums + a[2 * s4 + k4:].view(np.float32)).astype(np.float32)
            counts = np.sum([a[2 * s4:2 * s4 + k] for a in sh], axis=0).astype(np.uint32)
            want_l, want_s = oracle.top1(x.ravel(), d, pos, oracle.L2, ids=order[b:end])
            ws, wc = oracle.scatter_add(x.ravel(), d, want_l, k, ids=order[b:end])
            ok &= np.array_equal(got_l, want_l) and np.array_equal(got_s.view(np.uint32),
                                                                   want_s.view(np.uint32))
            ok &= np.array_equal(counts, wc)
            ok &= bool(np.all(np.abs(sums - ws) <= 1e-5 * (np.abs(ws) + 1.0)))
            pos, usage = oracle.ema_update(pos, usage, sums, counts, k, d, 0.5)
            digests.append(pos.view(np.uint32).astype(np.int64).sum())
        every = [None] * world
        dist.all_gather_object(every, digests)
        ok &= all(e == every[0] for e in every)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok)))
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, repr(exc)))


def _run_ranks(target, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=150) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    return results


@pytest.mark.timeout(180)
def test_two_gloo_ranks_merge_sharded_topk():
    assert _run_ranks(_knn_rank) == {0: True, 1: True}


@pytest.mark.timeout(180)
def test_two_gloo_ranks_assemble_the_batch():
    results = _run_ranks(_rank)
    assert results == {0: True, 1: True}, results


def test_reduce_layout_fits_the_shares():
    for batch, world, k, d in ((16384, 2, 1024, 768), (1029, 3, 37, 5), (1, 8, 3, 1)):
        s, s4, k4, share = eb.reduce_layout(batch, world, k, d)
        assert s * world >= batch and s4 >= s and s4 % 4 == 0 and k4 >= k and k4 % 4 == 0
        assert share == 2 * s4 + k4 + k * d and (2 * s4 + k4) % 4 == 0


@pytest.mark.timeout(180)
def test_two_gloo_ranks_reduce_partial_sums():
    assert _run_ranks(_reduce_rank) == {0: True, 1: True}
