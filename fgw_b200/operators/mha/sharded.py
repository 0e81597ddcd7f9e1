"""Paged MHA forward over several B200s: one call partitioned over the ranks of a process group.

The reference runs on one device (FGW operators/mha/kernels/mha_paged_decode_ascend_v7.py:516-570). Its work
items, (request, head) pairs, are independent, so on an 8-GPU box a call is partitioned with no collective on the
data path, one process per GPU:

* head sharding (``shard="heads"``, the default): rank r holds heads ``[r H / G, (r + 1) H / G)`` of Q and of the
  K/V pools (``[N, H / G, D]``), the whole block table and lengths, and computes O for those heads. Every rank has
  the same work whatever the spread of cache lengths.
* batch sharding (``shard="batch"``, for H smaller than or not divisible by G): ``batch_bins`` deals the requests
  to the ranks longest-first onto the least-loaded rank (LPT on KV tokens x query rows); rank r holds its
  requests' Q, table rows, lengths and a pool with their pages, in bin order.

``gather=True`` asks for the only collective: one all-gather of the per-rank outputs (NCCL over NVLink on the GPU
box) that assembles O[B, Sq, H, D] on every rank. Without it each rank returns its own shard and nothing crosses
NVLink. Each rank's forward is the single-GPU ``mha_paged_decode`` on its current stream.

``mha_paged_decode_devices`` is the same head partition from one process that drives several GPUs: one launch per
device on that device's current stream, optionally gathered onto one device with peer copies.
"""
import torch
import torch.distributed as dist

from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import mha_paged_decode


def head_shard(heads, rank, world):
    """(first head, head count) of ``rank`` when ``heads`` are split evenly over ``world`` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly over {world} ranks; use shard='batch'")
    per = heads // world
    return rank * per, per


def batch_bins(lengths, world, sq=1, causal=False):
    """Requests per rank: longest-processing-time order (most KV tokens seen first, index breaking ties), each
    onto the rank with the least work so far (lowest rank breaking ties). Work of a request is the KV tokens its
    query rows see. Returns ``world`` lists of request indices, each in ascending order."""
    if world <= 0:
        raise ValueError("world must be positive")

    def work(n):
        if not causal:
            return n * sq
        return sum(max(n - sq + i + 1, 0) for i in range(sq))

    loads = [0] * world
    bins = [[] for _ in range(world)]
    for b in sorted(range(len(lengths)), key=lambda i: (-work(int(lengths[i])), i)):
        r = min(range(world), key=lambda j: (loads[j], j))
        bins[r].append(b)
        loads[r] += work(int(lengths[b]))
    return [sorted(x) for x in bins]


def assemble_heads(parts):
    """O[B, Sq, H, D] from the per-rank outputs of a head-sharded call: a list [G][B, Sq, H / G, D], or those
    stacked in one tensor [G, B, Sq, H / G, D] (one copy either way)."""
    stacked = parts if isinstance(parts, torch.Tensor) else torch.stack(list(parts))  # [G, B, Sq, Hr, D]
    g, b, sq, hr, d = stacked.shape
    return stacked.permute(1, 2, 0, 3, 4).reshape(b, sq, g * hr, d)


def assemble_batch(parts, bins, batch):
    """O[B, Sq, H, D] from the per-rank outputs of a batch-sharded call (rank r's rows are ``bins[r]`` in order;
    a rank's part may carry padding rows past its bin)."""
    first = next(p for p in parts)
    out = first.new_empty((batch,) + tuple(first.shape[1:]))
    for part, rows in zip(parts, bins):
        if rows:
            out[torch.tensor(rows, device=out.device)] = part[: len(rows)]
    return out


def _all_gather(local, group, world):
    """``local`` of every rank over ``group`` (one all-gather), rank order: one stacked tensor on NCCL, a list
    otherwise."""
    if dist.get_backend(group) == "nccl":
        buf = local.new_empty((world,) + tuple(local.shape))
        dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
        return buf
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return parts


def mha_paged_decode_sharded(q, k_cache, v_cache, block_table, cache_seqlens, page_size, is_causal=False, *,
                             shard="heads", group=None, gather=False, bins=None, **kwargs):
    """This rank's part of a paged MHA forward sharded over ``group`` (default: the world).

    ``shard="heads"``: ``q`` [B, Sq, H / G, D] and ``k_cache``/``v_cache`` [N, H / G, D] hold this rank's heads
    (``head_shard``); ``block_table`` and ``cache_seqlens`` are the whole batch's.
    ``shard="batch"``: the tensors hold this rank's requests ``bins[rank]`` (``batch_bins``) in order; with
    ``gather=True``, ``bins`` (every rank's list) says where each rank's rows go.
    Returns this rank's output, or with ``gather=True`` the whole O[B, Sq, H, D] on every rank. Other keyword
    arguments go to ``mha_paged_decode``.
    """
    if shard not in ("heads", "batch"):
        raise ValueError("shard must be 'heads' or 'batch'")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if shard == "batch" and gather and (bins is None or len(bins) != world or len(bins[rank]) != q.shape[0]):
        raise ValueError("a gathered batch-sharded call needs every rank's bin, this rank's matching q")
    if (gather and world > 1 and shard == "heads" and kwargs.get("out") is None
            and dist.get_backend(group) == "nccl"):
        # The forward writes straight into this rank's slot of the gather buffer and the all-gather runs in
        # place, so the only copy is the one that interleaves the ranks' heads into O[B, Sq, H, D].
        buf = q.new_empty((world,) + tuple(q.shape))
        kwargs = dict(kwargs, out=buf[rank])
        mha_paged_decode(q, k_cache, v_cache, block_table, cache_seqlens, page_size, is_causal, **kwargs)
        dist.all_gather_into_tensor(buf, buf[rank], group=group)
        return assemble_heads(buf)
    local = mha_paged_decode(q, k_cache, v_cache, block_table, cache_seqlens, page_size, is_causal, **kwargs)
    if not gather or world == 1:
        return local
    if shard == "heads":
        return assemble_heads(_all_gather(local, group, world))
    most = max(len(x) for x in bins)
    padded = local.new_zeros((most,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    return assemble_batch(_all_gather(padded, group, world), bins, sum(len(x) for x in bins))


def mha_paged_decode_devices(shards, page_size, is_causal=False, *, gather_device=None, **kwargs):
    """Head-sharded forward driven from one process: ``shards`` is one (q, k_cache, v_cache, block_table,
    cache_seqlens) tuple per GPU, each holding that GPU's heads. Every launch goes on its device's current stream,
    so the GPUs run at once. Returns the per-device outputs, or with ``gather_device`` the whole O assembled on
    that device (peer copies ordered after each device's launch)."""
    outs = []
    for q, k, v, table, lengths in shards:
        with torch.cuda.device(q.device):
            outs.append(mha_paged_decode(q, k, v, table, lengths, page_size, is_causal, **kwargs))
    if gather_device is None:
        return outs
    target = torch.device(gather_device)
    moved = []
    for out in outs:
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(out.device))
        torch.cuda.current_stream(target).wait_event(done)
        with torch.cuda.device(target):
            moved.append(out.to(target, non_blocking=True))
    with torch.cuda.device(target):
        return assemble_heads(moved)
