"""One rank of the multi-GPU group test (launched by tests/test_gpu_group.py
under torch.distributed.run): a joined engine trains with the batch top-1
split across the ranks and the labels/scores all-gathered over NCCL, and
ranks a sharded database with eb_topk_group; both must equal, bit for bit, a
lone engine's results on the same GPU. In group mode 3 (the top-1 and the
scatter-add split, partial sums exchanged) every rank must hold the same
model, within rounding of the lone engine's; and a sharded assign with its
labels and scores all-gathered (eb_group_allgather) equals one engine's, over
NCCL and through the group's exchange region (peer memory over NVLink)."""

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import emeans_b200 as eb  # noqa: E402
from tests.helpers import mixture  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    cases = [
        # (n, d, k, spherical, seed): the C1 shape and an L2 case with revival
        (20000, 64, 32, True, 7),
        (30000, 96, 200, False, 3),
    ]
    group = eb.Engine(local)
    group.join_torch_group()
    assert group.group() == (rank, world)
    solo = eb.Engine(local)
    # Every batch split and exchanged (mode 1), and the default (mode 0: these
    # batches are one wave of row tiles or less, so every rank scores them whole).
    for mode in (1, 0):
        group.set_group_shard(mode)
        for n, d, k, spherical, seed in cases:
            x = mixture(n, d, 24, 0.4, spherical, seed)
            cfg = eb.Config(d=d, k=k, seed=seed, spherical=spherical, nepochs=2.0)
            a = group.train(x, cfg)
            b = solo.train(x, cfg)
            assert np.array_equal(a.centroids.view(np.uint32), b.centroids.view(np.uint32)), \
                f"rank {rank}: centroids differ (n={n}, k={k}, mode {mode})"
            assert np.array_equal(a.labels, b.labels), f"rank {rank}: labels differ"
            assert a.obj == b.obj and a.nsplit == b.nsplit, f"rank {rank}: statistics differ"
    # Mode 3, the north-star step: the top-1 and the scatter-add split, partial
    # sums exchanged and added in rank order. Every rank ends with the same
    # bits; the model agrees with the lone engine's to rounding.
    group.set_group_shard(3)
    for n, d, k, spherical, seed in cases:
        x = mixture(n, d, 24, 0.4, spherical, seed)
        cfg = eb.Config(d=d, k=k, seed=seed, spherical=spherical, nepochs=2.0)
        a = group.train(x, cfg)
        b = solo.train(x, cfg)
        every = [None] * world
        dist.all_gather_object(every, a.centroids.tobytes())
        assert all(v == every[0] for v in every), f"rank {rank}: ranks differ in mode 3"
        assert abs(a.obj[-1] - b.obj[-1]) <= 1e-3 * abs(b.obj[-1]), \
            f"rank {rank}: mode-3 objective {a.obj[-1]} vs {b.obj[-1]}"
    group.set_group_shard(0)
    # knn_self over a database sharded across the ranks, against one engine
    # ranking the whole database.
    rng = np.random.default_rng(11)
    n, d, kk = 5003, 48, 10
    data = rng.standard_normal((n, d)).astype(np.float32)
    data[4000:4010] = data[10:20]  # duplicates across the shards
    lo, hi = eb.shard_bounds(0, n, rank, world)
    for exclude_self in (True, False):
        gi, gs = group.topk_group(data, data[lo:hi], lo, n, d, kk, exclude_self)
        si, ss = solo.topk(data, data, d, kk, exclude_self)
        assert np.array_equal(gi, si), f"rank {rank}: knn ids differ"
        assert np.array_equal(gs.view(np.uint32), ss.view(np.uint32)), f"rank {rank}: knn sims differ"
    # A sharded assign: each rank's top-1 over its rows, then the labels and
    # scores all-gathered so that every rank holds all of them.
    n, d, k = 9001, 64, 300
    x = mixture(n, d, 24, 0.4, False, 5)
    c = x[:k] * np.float32(0.97)
    s = (n + world - 1) // world
    lo, hi = min(rank * s, n), min(rank * s + s, n)
    xb, cb, cn = group.bind(x, d), group.upload_f32(c), group.zeros_f32(k)
    group.row_norms(cb, k, d, cn)
    lab, sco = group.zeros_u32(s * world), group.zeros_f32(s * world)
    group.top1(xb, d, None, range(lo, hi), cb, cn, k, eb.L2, lab, sco)
    group.group_allgather(lab, s)
    group.group_allgather(sco, s)
    sl, ss = solo.assign(x, d, c, eb.L2)
    assert np.array_equal(lab.read(0, n), sl), f"rank {rank}: gathered labels differ"
    assert np.array_equal(sco.read(0, n).view(np.uint32), ss.view(np.uint32)), \
        f"rank {rank}: gathered scores differ"
    # The same sharded assign through the group's exchange region: labels and
    # scores of rank r's rows in its share (labels then scores), pushed into
    # every rank's copy over peer memory by eb_group_allgather.
    s4 = (s + 3) // 4 * 4
    res = group.group_exchange(world * 2 * s4)
    mapped, why = group.group_exchange_info()
    assert mapped, f"rank {rank}: the exchange region is not mapped: {why}"
    plab = group.view(res, rank * 2 * s4, s4, eb.U32)
    psco = group.view(res, rank * 2 * s4 + s4, s4, eb.F32)
    xs = group.bind(x[lo:hi], d)  # this rank's rows: its selection starts at 0
    group.top1(xs, d, None, range(0, hi - lo), cb, cn, k, eb.L2, plab, psco)
    for step in range(3):  # successive calls: the exchange's flags move on
        group.group_allgather(res, 2 * s4)
    got = res.read().reshape(world, 2, s4)
    glab = np.concatenate([got[q, 0, :min(s, n - q * s)] for q in range(world)])
    gsco = np.concatenate([got[q, 1, :min(s, n - q * s)] for q in range(world)]).view(np.float32)
    assert np.array_equal(glab, sl), f"rank {rank}: exchanged labels differ"
    assert np.array_equal(gsco.view(np.uint32), ss.view(np.uint32)), \
        f"rank {rank}: exchanged scores differ"
    # Every rank's share, written with its own pattern, reaches every rank.
    words = 1000
    res2 = group.group_exchange(world * words)
    mine = group.view(res2, rank * words, words, eb.U32)
    mine.write(0, (np.arange(words, dtype=np.uint64) * 2654435761 + rank).astype(np.uint32))
    group.group_allgather(res2, words)
    got2 = res2.read().reshape(world, words)
    for q in range(world):
        want = (np.arange(words, dtype=np.uint64) * 2654435761 + q).astype(np.uint32)
        assert np.array_equal(got2[q], want), f"rank {rank}: share {q} did not arrive"
    group.sync()
    del xb, xs, cb, cn, lab, sco, plab, psco, mine, res, res2
    group.close()
    solo.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: group training equals the lone engine", flush=True)


if __name__ == "__main__":
    main()
