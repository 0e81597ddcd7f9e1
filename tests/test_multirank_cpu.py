"""The multi-GPU host logic of bench.py on world-size-2 gloo process groups (CPU only).

bench.py shards the work with no collective on the data path: long-Q ranks each run their own batch (weak
scaling), decode ranks split the heads (strong scaling), and the only collectives are the timing barrier and
the max/sum of per-rank timings. These tests run those collectives on CPU ranks, and check that a rank that
drops out is seen by the other through a short process-group timeout rather than a hang.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, seconds=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=seconds))


def _reductions(rank, world, port, out):
    import bench
    _init(rank, world, port)
    try:
        step_ms = [1.25, 3.5][rank]
        flops = [10.0, 30.0][rank]
        bench.barrier(world)
        out[rank] = (bench.max_over_ranks(step_ms, world), bench.sum_over_ranks(flops, world),
                     bench.head_shard(32, rank, world))
    finally:
        dist.destroy_process_group()


def test_timing_reductions_and_head_shards_on_two_ranks():
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.spawn(_reductions, args=(world, port, out), nprocs=world, join=True)
        results = dict(out)
    for rank in range(world):
        step_max, flop_sum, (first, count) = results[rank]
        assert step_max == 3.5      # whole-job time is the slowest rank's
        assert flop_sum == 40.0     # whole-job work is the sum over ranks
        assert (first, count) == (16 * rank, 16)
    shards = sorted(results[r][2] for r in range(world))
    assert [h for first, n in shards for h in range(first, first + n)] == list(range(32))


def test_head_shard_rejects_uneven_split():
    import bench
    with pytest.raises(ValueError):
        bench.head_shard(32, 0, 3)


def _drop_out(rank, world, port, out):
    _init(rank, world, port, seconds=3)
    if rank == 1:
        out[rank] = "left"  # leaves between steps: never reaches the barrier
        return
    try:
        dist.barrier()
        out[rank] = "no error"
    except Exception as exc:  # the short timeout ends the collective with an error
        out[rank] = f"error: {type(exc).__name__}"


def test_rank_that_leaves_is_detected_by_the_timeout():
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_drop_out, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        results = dict(out)
    assert not any(alive), "a rank hung instead of failing"
    assert results[1] == "left"
    assert results[0].startswith("error"), results[0]
