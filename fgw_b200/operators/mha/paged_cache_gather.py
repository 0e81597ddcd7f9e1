"""Paged-cache gather pre-pass: pack the KV rows requests reach into a dense buffer, then attend over it.

FGW pins a TileOPs gather kernel and runs it ahead of its attention as a comparison point
(third_party/tileops_yyttt6/paged_cache_gather.py; benchmarks/mha/external_cache_gather.py). This module is
the B200 counterpart, on the CUDA gather of ``libfgw_mha.so`` (``fgw_paged_cache_gather``):

* ``paged_cache_gather(dst, cache, block_table, cu_seq_lens, seq_starts=None, scale=None)`` takes the
  arguments of the pinned kernel's ``forward`` (paged_cache_gather.py:264-296) and raises ValueError on the
  same mismatches (its ``refusal`` checks, :247-262 and :307-318, and the specialisation checks of
  ``forward``). Row r of request i (``cu_seq_lens[i] <= r < cu_seq_lens[i + 1]``) receives cache row
  ``block_table[i, pos // page] * page + pos % page``, ``pos = r - cu_seq_lens[i] + seq_starts[i]``; an FP8
  (E4M3) cache is dequantised with ``scale`` into an FP16/BF16 ``dst``. Offsets, starts and page ids stay on
  the device.
* ``build_gather_attention(...)`` restates the experiment's pipeline (external_cache_gather.py:38-76):
  request lengths rounded up to whole pages give packed offsets, K and V are gathered into fresh dense
  buffers, and the same attention kernel runs over them through an identity page table with the original
  lengths. Metadata is prepared once, outside the timed call.
"""
import math

import torch

from fgw_b200 import _native
from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import build_kernel

_DTYPES = {torch.float16: _native.DTYPE_FLOAT16, torch.bfloat16: _native.DTYPE_BFLOAT16}
_FP8 = getattr(torch, "float8_e4m3fn", None)
if _FP8 is not None:
    _DTYPES[_FP8] = _native.DTYPE_FLOAT8_E4M3


def _refusal(dtype, out_dtype, batch, num_pages, page_size, table_width, row_width):
    """The pinned kernel's refusal conditions (paged_cache_gather.py:307-318, :247-262 position bound)."""
    if min(batch, num_pages, page_size, table_width, row_width) <= 0:
        return "requires positive cache, table and row extents"
    if page_size * table_width > (1 << 31) - 1:
        return "requires logical positions to fit int32"
    if dtype not in _DTYPES:
        return "requires FP16, BF16 or FP8 E4M3FN cache"
    if dtype == _FP8:
        if out_dtype not in (torch.float16, torch.bfloat16):
            return "FP8 requires FP16/BF16 destination"
    elif out_dtype != dtype:
        return "unquantized gather preserves dtype"
    return None


def paged_cache_gather(dst, cache, block_table, cu_seq_lens, seq_starts=None, scale=None):
    """Write ``dst[r]`` for every output row r (see the module docstring); returns None.

    ``cache`` is ``[num_pages, page_size, *row]``, ``dst`` is ``[total_rows, *row]``, ``block_table``
    ``[batch, table_width]`` int32, ``cu_seq_lens`` ``[batch + 1]`` int32, ``seq_starts`` ``[batch]`` int32 or
    None, ``scale`` ``[1]`` float32 for an FP8 cache, else None. All on one CUDA device and contiguous.
    """
    if cache.dim() < 3 or dst.dim() < 2:
        raise ValueError("cache must be [num_pages, page_size, ...] and dst [rows, ...]")
    batch, table_width = (block_table.shape[0], block_table.shape[1]) if block_table.dim() == 2 else (0, 0)
    num_pages, page_size = cache.shape[0], cache.shape[1]
    row_width = math.prod(cache.shape[2:])
    reason = _refusal(cache.dtype, dst.dtype, batch, num_pages, page_size, table_width, row_width)
    if reason:
        raise ValueError(reason)
    tensors = [dst, cache, block_table, cu_seq_lens] + [t for t in (seq_starts, scale) if t is not None]
    if any(not t.is_cuda for t in tensors) or any(t.device != dst.device for t in tensors):
        raise ValueError("every gather tensor must be on the same CUDA device")
    if (scale is not None) != (cache.dtype == _FP8):
        raise ValueError("optional inputs do not match gather specialization")
    if tuple(dst.shape[1:]) != tuple(cache.shape[2:]):
        raise ValueError("cache/destination does not match gather specialization")
    metadata = [(block_table, (batch, table_width), torch.int32), (cu_seq_lens, (batch + 1,), torch.int32)]
    if seq_starts is not None:
        metadata.append((seq_starts, (batch,), torch.int32))
    if scale is not None:
        metadata.append((scale, (1,), torch.float32))
    if any(tuple(t.shape) != shape or t.dtype != dtype for t, shape, dtype in metadata):
        raise ValueError("gather metadata shape/dtype does not match specialization")
    if any(not t.is_contiguous() for t in tensors):
        raise ValueError("kernel inputs must be contiguous")
    if not dst.numel():
        return None
    p = _native.GatherParams()
    p.dst = dst.data_ptr()
    p.cache = cache.data_ptr()
    p.block_table = block_table.data_ptr()
    p.cu_seq_lens = cu_seq_lens.data_ptr()
    p.seq_starts = seq_starts.data_ptr() if seq_starts is not None else None
    p.scale = scale.data_ptr() if scale is not None else None
    p.total_rows = dst.shape[0]
    p.batch = batch
    p.num_pages = num_pages
    p.page_size = page_size
    p.table_width = table_width
    p.row_width = row_width
    p.dtype = _DTYPES[cache.dtype]
    p.out_dtype = _DTYPES[dst.dtype]
    with torch.cuda.device(dst.device):
        _native.paged_cache_gather(p, torch.cuda.current_stream().cuda_stream)
    return None


def packed_layout(lengths, page_size, table_width):
    """Packed offsets of the gather experiment (external_cache_gather.py:50-58): each request's live length
    rounded up to whole pages, laid end to end. Returns (cu offsets [batch + 1], rows of the dense buffer
    (at least one page), the identity page table [batch][table_width] over the packed rows)."""
    pages = [(int(length) + page_size - 1) // page_size for length in lengths]
    offsets = [0]
    for count in pages:
        offsets.append(offsets[-1] + count * page_size)
    rows = max(page_size, offsets[-1])
    table = [[offsets[i] // page_size + j for j in range(table_width)] for i in range(len(pages))]
    return offsets, rows, table


def build_gather_attention(batch, sq, heads, dim, page_size, table_width, lengths, causal, dtype,
                           device_index=None, num_splits=None):
    """The gather-then-attend pipeline for host-known ``lengths``; returns ``(run, info)``.

    ``run(q, k_cache, v_cache, block_table, cache_seqlens)`` allocates the dense K and V, gathers both
    (two launches) and runs attention over them with the identity table and the original lengths — the
    work the reference experiment times (external_cache_gather.py:60-76). ``info`` describes the layout.
    """
    offsets, rows, table = packed_layout(lengths, page_size, table_width)
    device = torch.device("cuda", torch.cuda.current_device() if device_index is None else device_index)
    cu = torch.tensor(offsets, dtype=torch.int32, device=device)
    dense_table = torch.tensor(table, dtype=torch.int32, device=device)
    dtype_name = str(dtype).replace("torch.", "")
    attention = build_kernel(batch, sq, heads, dim, rows, table_width, page_size, causal, dtype_name,
                             device.index, num_splits=num_splits)

    def gather_pair(k_cache, v_cache, block_table):
        dense_k = torch.empty((rows, heads, dim), dtype=k_cache.dtype, device=k_cache.device)
        dense_v = torch.empty_like(dense_k)
        if offsets[-1]:
            pool_pages = k_cache.shape[0] // page_size
            for src, dst in ((k_cache, dense_k), (v_cache, dense_v)):
                paged_cache_gather(dst[:offsets[-1]], src.view(pool_pages, page_size, heads, dim), block_table, cu)
        return dense_k, dense_v

    def run(q, k_cache, v_cache, block_table, cache_seqlens):
        dense_k, dense_v = gather_pair(k_cache, v_cache, block_table)
        return attention(q, dense_k, dense_v, dense_table, cache_seqlens)

    run.gather_pair = gather_pair
    run.attention = attention
    info = {"packed_rows": offsets[-1], "live_rows": int(sum(int(x) for x in lengths)), "dense_rows": rows,
            "gather_calls_per_attention": 2 if offsets[-1] else 0, "num_splits": attention.num_splits}
    return run, info
