"""NumPy restatement of the paged-cache gather (test infrastructure, not product code; see ``oracle/__init__.py``).

Follows the kernel FGW pins as its gather pre-pass, third_party/tileops_yyttt6/paged_cache_gather.py:
output row ``r`` belongs to the request ``i`` with ``cu[i] <= r < cu[i + 1]`` (the binary search of
:65-72 and :150-157), its logical position is ``pos = r - cu[i] (+ start[i])`` (:73-75, :176-178), and it
receives cache row ``table[i, pos // page] * page + pos % page`` (:76-79, :185-187). FP8 E4M3 codes are
widened to FP32, multiplied by the FP32 scale and converted to the output type (:83-88: vcvt, vmul, vcvt).

Where the reference leaves the result undefined (rows outside every request, positions past the table, page
ids outside the pool) the B200 library writes zeros, and so does this restatement.

Parity anchor: FGW has no stored gather outputs; its experiment checks every gathered row exactly against
``cache.view(-1, page, H, D)[table[i, :pages]]`` (benchmarks/mha/external_cache_gather.py:63-71).
``reference_packed_check`` restates that check, and the CPU tests hold this oracle to it.

16-bit values travel as ``uint16`` bit patterns (BF16 has no NumPy dtype); FP8 caches as ``uint8`` codes.
"""
import numpy as np

from oracle.paged_attention import f32_to_dtype_bits


def e4m3_to_f32(codes):
    """FP8 E4M3 (the "fn" variant: no infinities, S.1111.111 is NaN) codes to FP32, exactly.

    Format: sign bit, 4 exponent bits with bias 7, 3 mantissa bits; exponent 0 is subnormal (m / 8 * 2^-6).
    """
    codes = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    normal = (1.0 + man / 8.0) * np.exp2(exp.astype(np.float64) - 7.0)
    sub = (man / 8.0) * 2.0 ** -6
    value = sign * np.where(exp == 0, sub, normal)
    value = np.where((exp == 15) & (man == 7), np.nan, value)
    return value.astype(np.float32)


def paged_cache_gather(cache, table, cu, total_rows=None, starts=None, scale=None, out_dtype=None):
    """Gathered rows ``[total_rows, *row]``.

    ``cache``: ``[num_pages, page, *row]`` uint16 bits (FP16/BF16) or uint8 codes (FP8, with ``scale`` and
    ``out_dtype`` "float16" / "bfloat16"); ``table`` ``[batch, width]``; ``cu`` ``[batch + 1]``; ``starts``
    ``[batch]`` or None. Returns uint16 bits.
    """
    cache = np.asarray(cache)
    table = np.asarray(table, dtype=np.int64)
    cu = np.asarray(cu, dtype=np.int64)
    num_pages, page = cache.shape[0], cache.shape[1]
    row_shape = cache.shape[2:]
    flat = cache.reshape(num_pages * page, -1)
    batch, width = table.shape
    total = int(cu[-1]) if total_rows is None else int(total_rows)
    fp8 = cache.dtype == np.uint8
    out = np.zeros((total, flat.shape[1]), dtype=np.uint16)
    for r in range(total):
        # the last request whose first row is <= r (request 0 for rows before cu[0])
        i = max(int(np.searchsorted(cu[:batch], r, side="right")) - 1, 0)
        if not (cu[i] <= r < cu[i + 1]):
            continue
        pos = r - int(cu[i]) + (int(starts[i]) if starts is not None else 0)
        if pos < 0 or pos // page >= width:
            continue
        page_id = int(table[i, pos // page])
        if not 0 <= page_id < num_pages:
            continue
        src = flat[page_id * page + pos % page]
        if fp8:
            value = e4m3_to_f32(src) * np.float32(scale)
            out[r] = f32_to_dtype_bits(value.astype(np.float32), out_dtype)
        else:
            out[r] = src
    return out.reshape((total,) + row_shape)


def reference_packed_check(cache, table, lengths, page):
    """The experiment's expected packed cache (external_cache_gather.py:50-58, 63-71): for every request the
    cache pages ``table[i, :ceil(L_i / page)]`` in order, laid end to end."""
    cache = np.asarray(cache)
    parts = []
    for i, length in enumerate(lengths):
        count = (int(length) + page - 1) // page
        if count:
            parts.append(cache[np.asarray(table[i][:count], dtype=np.int64)].reshape((-1,) + cache.shape[2:]))
    if not parts:
        return np.zeros((0,) + cache.shape[2:], dtype=cache.dtype)
    return np.concatenate(parts)
