"""The multi-GPU split and exchange, checked on CPU with two gloo ranks.

eb_train in a group splits every batch's top-1 into equal slices of
ceil(B / world) positions (emeans_b200.shard_bounds mirrors that split) and
all-gathers the slices' labels and scores. Here each gloo rank scores its
slice with the CPU oracle and all-gathers it; the assembled batch must equal
the oracle over the whole batch, for batch sizes that do not divide evenly.
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


@pytest.mark.timeout(180)
def test_two_gloo_ranks_assemble_the_batch():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=150) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    assert results == {0: True, 1: True}, results
