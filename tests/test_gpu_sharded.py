"""The multi-GPU product API on two B200s: one call sharded by head and by request, gathered over NCCL.

Two processes, one per GPU (NCCL, 127.0.0.1 rendezvous, short process-group timeout). Each rank computes its shard
with the CUDA kernels and the gathered output is compared on every rank with the oracle on the whole batch. Skipped
when fewer than two GPUs are visible.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASE = dict(batch=6, sq=3, heads=8, dim=128, page=64, width=40)
LENGTHS = [2560, 0, 17, 1500, 64, 999]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    c = CASE
    gen = torch.Generator().manual_seed(11)
    pages = c["batch"] * c["width"] + 1
    table = torch.stack([torch.randperm(pages, generator=gen)[: c["width"]] for _ in range(c["batch"])]).int()
    q = torch.randn(c["batch"], c["sq"], c["heads"], c["dim"], generator=gen).to(torch.bfloat16)
    k = torch.randn(pages * c["page"], c["heads"], c["dim"], generator=gen).to(torch.bfloat16)
    v = torch.randn(pages * c["page"], c["heads"], c["dim"], generator=gen).to(torch.bfloat16)
    return q, k, v, table, torch.tensor(LENGTHS, dtype=torch.int32)


def _rank(rank, world, port, causal, queue):
    import torch.distributed as dist
    from fgw_b200.operators.mha import sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v, table, lengths = _inputs()
        page = CASE["page"]
        first, count = sharded.head_shard(CASE["heads"], rank, world)
        h = slice(first, first + count)
        by_head = sharded.mha_paged_decode_sharded(q[:, :, h].contiguous().to(dev), k[:, h].contiguous().to(dev),
                                                   v[:, h].contiguous().to(dev), table.to(dev), lengths.to(dev),
                                                   page, causal, shard="heads", gather=True)
        bins = sharded.batch_bins(LENGTHS, world, CASE["sq"], causal)
        rows = torch.tensor(bins[rank], dtype=torch.long)
        by_batch = sharded.mha_paged_decode_sharded(q[rows].to(dev), k.to(dev), v.to(dev), table[rows].to(dev),
                                                    lengths[rows].to(dev), page, causal, shard="batch", gather=True,
                                                    bins=bins)
        torch.cuda.synchronize()
        queue.put((rank, by_head.float().cpu().numpy(), by_batch.float().cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_two_gpu_sharded_call_matches_the_oracle(causal):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from fixtures import MAX_ABS
    from oracle import paged_attention
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, causal, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    q, k, v, table, lengths = _inputs()
    want = paged_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), table.numpy(), lengths.numpy(),
                           CASE["page"], causal)
    for _, by_head, by_batch in results:
        assert np.abs(by_head - want).max() <= MAX_ABS["bfloat16"]
        assert np.abs(by_batch - want).max() <= MAX_ABS["bfloat16"]
        visible = np.asarray(LENGTHS)[:, None] - (CASE["sq"] - 1 - np.arange(CASE["sq"]))[None] if causal \
            else np.repeat(np.asarray(LENGTHS)[:, None], CASE["sq"], 1)
        assert not by_head[visible <= 0].any() and not by_batch[visible <= 0].any()


@pytest.mark.parametrize("causal", [False, True])
def test_device_list_call_from_one_process_matches_the_oracle(causal):
    # mha_paged_decode_devices: the head partition driven from one process, one launch per GPU on its current
    # stream, then the whole output assembled on GPU 0 by peer copies.
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from fixtures import MAX_ABS
    from oracle import paged_attention
    from fgw_b200.operators.mha import sharded
    q, k, v, table, lengths = _inputs()
    shards = []
    for rank in range(2):
        dev = torch.device("cuda", rank)
        first, count = sharded.head_shard(CASE["heads"], rank, 2)
        h = slice(first, first + count)
        shards.append((q[:, :, h].contiguous().to(dev), k[:, h].contiguous().to(dev), v[:, h].contiguous().to(dev),
                       table.to(dev), lengths.to(dev)))
    full = sharded.mha_paged_decode_devices(shards, CASE["page"], causal, gather_device="cuda:0")
    torch.cuda.synchronize()
    got = full.float().cpu().numpy()
    want = paged_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), table.numpy(), lengths.numpy(),
                           CASE["page"], causal)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= MAX_ABS["bfloat16"]
