"""Multi-rank host logic on CPU (gloo, world size 2): sequence sharding has no collective on the data
path; the only collectives are the barrier and the MAX all-reduce of per-rank timings. configs[4]'s
generated tokens are gathered on the host: every rank copies its rows into one shared host buffer."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import bench


def test_shard_range_partitions_exactly():
    for total in (1, 7, 64):
        for world in (1, 2, 4, 8):
            spans = [bench.shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_lpt_assign_balances_work():
    import numpy as np
    rng = np.random.default_rng(0)
    work = [float(x) ** 2 for x in rng.integers(1, 513, size=64)]  # prompt-length^2 attention cost
    for world in (2, 4, 8):
        bins = bench.lpt_assign(work, world)
        assert sorted(i for b in bins for i in b) == list(range(64))
        loads = [sum(work[i] for i in b) for b in bins]
        assert max(loads) <= sum(work) / world + max(work)  # LPT bound


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    lo, hi = bench.shard_range(64, rank, world)
    # each rank "times" its own shard; the job time is the slowest rank's
    t = bench.max_over_ranks(float(hi - lo) + 0.25 * rank, world)
    bench.barrier(world)
    out[rank] = t
    dist.destroy_process_group()


def test_max_over_ranks_gloo_two_ranks():
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()  # no fork of a possibly multi-threaded test process
    out = mgr.dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    assert out[0] == out[1] == pytest.approx(32.25)


def _gather_worker(rank, world, port, out):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    total, steps = 64, 5
    lo, hi = bench.shard_range(total, rank, world)
    # each rank's "generated tokens": row = global sequence index * 1000 + position
    shard = torch.tensor([[(lo + b) * 1000 + t for t in range(steps)] for b in range(hi - lo)],
                         dtype=torch.int32)
    g = bench.HostGather((total, steps), np.int32, rank, world)
    g.rows(lo, hi).copy_(shard)  # this rank's rows only, no collective
    bench.barrier(world)
    out[rank] = np.array(g.array).tolist()
    path = g.path
    g.close()
    out[f"gone{rank}"] = not os.path.exists(path) if rank == 0 else True


def test_host_gather_assembles_sequences_in_order_without_a_collective():
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()  # no fork of a possibly multi-threaded test process
    out = mgr.dict()
    mp.spawn(_gather_worker, args=(2, port, out), nprocs=2, join=True)
    want = [[s * 1000 + t for t in range(5)] for s in range(64)]
    assert out[0] == want and out[1] == want
    assert out["gone0"]  # the shared file is removed once every rank has closed it
