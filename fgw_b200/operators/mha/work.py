"""Algorithmic work of one paged-MHA forward call, for throughput and roofline reporting.

``useful_flops`` is FGW's FLOP policy for its MFU figures (benchmarks/mha/bench_mha_mfu.py:63-66): QK and PV
over the visible (query, key) pairs only, 4 * H * D FLOPs per pair, where query row i of a request with L keys
sees L keys, or max(L - Sq + i + 1, 0) when causal. ``algorithmic_bytes`` is the least HBM traffic the path
needs: the live K and V rows, Q and O, the block table and the lengths (page rounding and split partials
excluded).
"""


def useful_flops(lengths, sq, heads, dim, causal):
    pairs = 0
    for length in lengths:
        length = int(length)
        if not causal:
            pairs += length * sq
            continue
        # sum over i < sq of max(length - sq + i + 1, 0): an arithmetic series from max(length - sq + 1, 1)
        # up to length
        if length <= 0:
            continue
        low = max(length - sq + 1, 1)
        pairs += (length + low) * (length - low + 1) // 2
    return 4 * heads * dim * pairs


def algorithmic_bytes(lengths, batch, sq, heads, dim, width, elem_bytes):
    live = sum(int(n) for n in lengths)
    return (live * heads * dim * 2 * elem_bytes + 2 * batch * sq * heads * dim * elem_bytes
            + 4 * batch * width + 4 * batch)
