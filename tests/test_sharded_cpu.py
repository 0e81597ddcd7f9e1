"""The multi-GPU product API (``fgw_b200.operators.mha.sharded``) on world-size-2 gloo process groups, CPU only.

Each rank's single-GPU forward is replaced by the NumPy oracle, so these tests check what the sharded API adds:
the head and batch partitions, the LPT request bins, the one all-gather of a gathered call and the assembly of
O[B, Sq, H, D] from the rank outputs, against the oracle on the whole batch.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fgw_b200.operators.mha import sharded

CASE = dict(batch=5, sq=3, heads=4, dim=32, page=16, width=6)
LENGTHS = [90, 0, 17, 64, 33]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed=3):
    c = CASE
    gen = torch.Generator().manual_seed(seed)
    pages = c["batch"] * c["width"] + 2
    table = torch.stack([torch.randperm(pages, generator=gen)[: c["width"]] for _ in range(c["batch"])]).int()
    q = torch.randn(c["batch"], c["sq"], c["heads"], c["dim"], generator=gen)
    k = torch.randn(pages * c["page"], c["heads"], c["dim"], generator=gen)
    v = torch.randn(pages * c["page"], c["heads"], c["dim"], generator=gen)
    return q, k, v, table, torch.tensor(LENGTHS, dtype=torch.int32)


def _oracle_forward(q, k, v, table, lengths, page_size, is_causal=False, **_):
    from oracle import paged_attention
    out = paged_attention(q.numpy(), k.numpy(), v.numpy(), table.numpy(), lengths.numpy(), page_size, is_causal)
    return torch.from_numpy(out)


def _rank(rank, world, port, shard, causal, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        sharded.mha_paged_decode = _oracle_forward  # the per-rank forward, on CPU
        q, k, v, table, lengths = _inputs()
        page = CASE["page"]
        if shard == "heads":
            first, count = sharded.head_shard(CASE["heads"], rank, world)
            heads = slice(first, first + count)
            local = (q[:, :, heads].contiguous(), k[:, heads].contiguous(), v[:, heads].contiguous(), table, lengths)
            bins = None
        else:
            bins = sharded.batch_bins(LENGTHS, world, CASE["sq"], causal)
            rows = torch.tensor(bins[rank], dtype=torch.long)
            local = (q[rows], k, v, table[rows], lengths[rows])
        mine = sharded.mha_paged_decode_sharded(*local, page, causal, shard=shard)
        whole = sharded.mha_paged_decode_sharded(*local, page, causal, shard=shard, gather=True, bins=bins)
        out[rank] = (mine.numpy(), whole.numpy(), bins)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shard,causal", [("heads", False), ("heads", True), ("batch", False), ("batch", True)])
def test_sharded_call_assembles_the_whole_batch(shard, causal):
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.spawn(_rank, args=(world, port, shard, causal, out), nprocs=world, join=True)
        results = dict(out)
    q, k, v, table, lengths = _inputs()
    want = _oracle_forward(q, k, v, table, lengths, CASE["page"], causal).numpy()
    for rank in range(world):
        mine, whole, bins = results[rank]
        np.testing.assert_array_equal(whole, want)  # every rank holds the assembled output
        if shard == "heads":
            first, count = sharded.head_shard(CASE["heads"], rank, world)
            np.testing.assert_array_equal(mine, want[:, :, first:first + count])
        else:
            np.testing.assert_array_equal(mine, want[bins[rank]])


def test_batch_bins_balance_kv_work_longest_first():
    lengths = [32768, 1024, 16384, 16384, 2048, 30000, 4096, 8192]
    bins = sharded.batch_bins(lengths, 3)
    assert sorted(i for b in bins for i in b) == list(range(len(lengths)))
    loads = [sum(lengths[i] for i in b) for b in bins]
    # LPT: 32768 | 30000 | 16384 + 16384 ... no bin exceeds the mean by more than the largest request
    assert max(loads) - sum(loads) / 3 <= max(lengths)
    assert bins == sharded.batch_bins(lengths, 3)  # deterministic
    # causal multi-query work counts the visible keys of every query row
    assert sharded.batch_bins([4, 100], 2, sq=8, causal=True) == [[1], [0]]


def test_head_shard_partitions_the_heads():
    assert [sharded.head_shard(32, r, 8) for r in range(8)] == [(4 * r, 4) for r in range(8)]
    with pytest.raises(ValueError):
        sharded.head_shard(8, 0, 3)
    with pytest.raises(ValueError):
        sharded.head_shard(8, 3, 2)


def test_assembly_of_head_and_batch_parts():
    full = torch.arange(2 * 3 * 4 * 5, dtype=torch.float32).reshape(2, 3, 4, 5)
    parts = [full[:, :, 0:2], full[:, :, 2:4]]
    assert torch.equal(sharded.assemble_heads(parts), full)
    bins = [[0, 2], [1]]  # rank 1's part is padded to the largest bin
    three = torch.arange(3 * 2, dtype=torch.float32).reshape(3, 2)
    parts = [three[[0, 2]], torch.cat([three[[1]], torch.zeros(1, 2)])]
    assert torch.equal(sharded.assemble_batch(parts, bins, 3), three)
