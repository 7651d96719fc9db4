"""The multi-GPU plumbing of bench.py on CPU ranks (gloo, world size 2): each rank owns its own takes (disjoint
shares of one seeded draw, balanced in KV bytes, no collective on the data path) and rank 0 reports the summed
bytes over the max device time."""
import os
import sys
from datetime import timedelta

import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        lens = bench.take_lengths(rank, world)
        per_step = bench.LAYERS * bench.bytes_per_layer(lens)
        ms = 10.0 + 3.0 * rank  # each rank's own (pretend) device time
        total = bench.rank_reduce(per_step, "sum", dist)
        slowest = bench.rank_reduce(ms, "max", dist)
        q.put((rank, [int(x) for x in lens], per_step, total, slowest))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_takes_and_aggregate():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, l0, b0, t0, m0), (_, l1, b1, t1, m1) = res[0], res[1]
    assert len(l0) == len(l1) == 64 and l0 != l1             # each rank its own 64 takes
    assert all(330 <= x <= 4096 for x in l0 + l1)
    from oumu_b200 import synth                              # together: the seeded draw of 128 takes, dealt out
    assert sorted(l0 + l1) == sorted(int(v) for v in synth.uniform_int(0x5EED + 1, 128, 330, 4096))
    assert abs(sum(l0) - sum(l1)) <= 4096                    # balanced to within one take's length
    assert t0 == t1 == b0 + b1                               # bytes of all ranks
    assert m0 == m1 == 13.0                                  # the slowest rank's time


def test_single_process_reduce_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.rank_reduce(5.0, "max") == 5.0


def _gather_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from oumu_b200 import engine
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        B, S = 3, 5
        patches = (torch.arange(B * S * engine.PATCH, dtype=torch.float32).view(B, S, engine.PATCH) + 1000 * rank
                   ).to(torch.bfloat16)
        stop = torch.tensor([10 * rank + k for k in range(B)], dtype=torch.int32)
        gp, gs = engine.gather_patches(patches, stop)
        q.put((rank, gp.view(torch.int16).numpy().copy(), gs.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_gather_finished_patches():
    # the sharded decode's one collective: every rank ends with all takes' patches and stop steps in rank order
    import numpy as np
    import torch
    sys.path.insert(0, ROOT)
    from oumu_b200 import engine
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    B, S = 3, 5
    want = torch.cat([(torch.arange(B * S * engine.PATCH, dtype=torch.float32).view(B, S, engine.PATCH) + 1000 * r
                       ).to(torch.bfloat16) for r in range(2)]).view(torch.int16).numpy()
    for r in range(2):
        assert np.array_equal(res[r][1], want)
        assert res[r][2].tolist() == [0, 1, 2, 10, 11, 12]
    # one process, no group: the tensors come back as they are
    p1, s1 = engine.gather_patches(torch.zeros(2, 3, engine.PATCH, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int32))
    assert p1.shape == (2, 3, engine.PATCH) and s1.shape == (2,)
