"""Seeded inputs for the paged-MHA parity tests.

The case tables and the adversarial paging fixture follow FGW's accuracy harness
(``tests/mha/test_mha_paged_accuracy.py:17-101``): every case is
``(label, batch, queries, heads, head_dim, page_size, table_width)``; the pool holds one
page that no request references; request 0's first page is shared by every request;
the last request repeats its first physical page as its last one; pool rows that no
request reads are set to NaN before the call (:232-238).  Inputs are drawn from a
``torch.Generator`` in the same order as the harness, so the same seed gives the same
tensors, which is what lets ``tests/golden/`` hold only the expected outputs.
"""
import hashlib

import numpy as np
import torch

# label, batch, queries, heads, head_dim, page_size, table_width  (test_mha_paged_accuracy.py:18-70)
QUICK = [
    ("tiny", 2, 2, 2, 16, 16, 2),
    ("non_power_two_dim", 3, 4, 2, 80, 32, 3),
    ("wide_head", 2, 2, 4, 256, 128, 2),
]
STANDARD = QUICK + [
    ("single_decode", 1, 1, 8, 64, 128, 4),
    ("dim32", 4, 2, 4, 32, 32, 4),
    ("dim128", 2, 4, 4, 128, 64, 4),
    ("many_queries", 2, 8, 2, 64, 16, 8),
    ("many_requests", 8, 2, 2, 64, 64, 4),
    ("page256", 2, 2, 4, 128, 256, 4),
    ("cache2048", 2, 2, 2, 64, 128, 16),
]
EXTENDED = STANDARD + [
    ("dim48", 2, 2, 2, 48, 48, 3),
    ("dim96", 2, 4, 2, 96, 64, 8),
    ("dim192", 2, 2, 2, 192, 128, 4),
    ("cache4096", 2, 2, 2, 128, 256, 16),
    ("cache8192", 2, 2, 2, 64, 256, 32),
]
CUBE = [
    ("cube_decode512", 1, 1, 8, 128, 128, 4),
    ("cube_decode2048", 2, 1, 4, 128, 256, 8),
    ("cube_query4", 2, 4, 4, 128, 128, 16),
    ("cube_q127", 1, 127, 2, 128, 128, 2),
    ("cube_q128", 1, 128, 2, 128, 128, 2),
    ("cube_q129", 1, 129, 2, 128, 128, 2),
    ("cube_q257", 1, 257, 2, 128, 128, 2),
    ("cube_direct_q1", 2, 1, 64, 128, 128, 2),
    ("cube_direct_q129", 2, 129, 64, 128, 128, 2),
    ("cube_direct_q1024", 2, 1024, 8, 128, 128, 2),
]
GENERAL = [
    ("general_d16_page16", 2, 2, 2, 16, 16, 3),
    ("general_d32_q31", 2, 31, 2, 32, 32, 2),
    ("general_d48_page48", 2, 4, 2, 48, 48, 3),
    ("general_d64_q33", 2, 33, 2, 64, 64, 2),
    ("general_d80", 2, 17, 2, 80, 32, 3),
    ("general_d96", 2, 32, 2, 96, 64, 2),
    ("general_d128_q129", 2, 129, 2, 128, 128, 2),
    ("general_d192", 2, 4, 2, 192, 128, 2),
    ("general_d256", 2, 4, 2, 256, 256, 2),
    ("general_decode", 1, 1, 2, 128, 128, 2),
]
SPLIT = [
    ("split_d16_q1", 2, 1, 2, 16, 16, 64),
    ("split_d48_q17", 2, 17, 2, 48, 48, 24),
    ("split_d128_q33", 2, 33, 2, 128, 128, 8),
    ("split_d256_q129", 2, 129, 2, 256, 256, 4),
]
SUITES = {"quick": QUICK, "standard": STANDARD, "extended": EXTENDED, "cube": CUBE,
          "general": GENERAL, "split": SPLIT}
ALL_CASES = {c[0]: c for suite in SUITES.values() for c in suite}
PATTERNS = ("mixed", "full", "empty")
SEEDS = (7, 42, 2026)
TOLERANCE = {"bfloat16": (1e-2, 4e-3), "float16": (2e-3, 2e-3)}  # rtol, atol (test_mha_paged_accuracy.py:264)
MAX_ABS = {"bfloat16": 2e-2, "float16": 5e-3}  # north-star max-abs bound


def lengths_for(case, pattern, seed):
    """Per-request cache lengths for a length pattern (test_mha_paged_accuracy.py:73-83)."""
    _, b, sq, _, _, p, w = case
    capacity = p * w
    if pattern == "empty":
        return [0] * b
    if pattern == "full":
        return [capacity] * b
    ladder = [0, 1, max(0, sq - 1), sq, p - 1, p, p + 1, capacity - 1, capacity]
    return [min(capacity, ladder[(i + seed) % len(ladder)]) for i in range(b)]


def make_inputs(case, seed, dtype):
    """Seeded Q, K pool, V pool and block table (CPU tensors), in harness RNG order."""
    _, b, sq, h, d, p, w = case
    gen = torch.Generator().manual_seed(seed)
    pool_pages = max(w + 3, b * w + 1)
    rows = [torch.randperm(pool_pages - 1, generator=gen)[:w] for _ in range(b)]
    table = torch.stack(rows).to(torch.int32)
    if b > 1:
        table[1:, 0] = table[0, 0]
    if w > 1:
        table[-1, -1] = table[-1, 0]
    q = torch.randn(b, sq, h, d, generator=gen).to(dtype)
    k = torch.randn(pool_pages * p, h, d, generator=gen).to(dtype)
    v = torch.randn(pool_pages * p, h, d, generator=gen).to(dtype)
    return q, k, v, table


def poison_unread(k, v, table, lengths, page_size):
    """Copies of K/V whose rows that no request reads are NaN (accuracy.py:232-238)."""
    live = torch.zeros(k.shape[0], dtype=torch.bool)
    for bi, length in enumerate(lengths):
        pos = torch.arange(int(length))
        live[table[bi, pos // page_size].long() * page_size + pos % page_size] = True
    k, v = k.clone(), v.clone()
    k[~live] = float("nan")
    v[~live] = float("nan")
    return k, v


def build_case(case, seed, dtype, causal, pattern):
    """Everything one parity check needs, on the CPU."""
    q, k, v, table = make_inputs(case, seed, dtype)
    lengths = lengths_for(case, pattern, seed)
    k, v = poison_unread(k, v, table, lengths, case[5])
    return {"case": case, "seed": seed, "dtype": dtype, "causal": causal, "pattern": pattern,
            "q": q, "k": k, "v": v, "table": table,
            "lengths": torch.tensor(lengths, dtype=torch.int32)}


def to_bits(t):
    """uint16 NumPy view of a CPU FP16/BF16 tensor."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def dtype_name(dtype):
    return "bfloat16" if dtype == torch.bfloat16 else "float16"


def input_digest(inputs):
    """SHA-256 over the raw bytes of Q, K, V, table and lengths."""
    h = hashlib.sha256()
    for key in ("q", "k", "v"):
        h.update(to_bits(inputs[key]).tobytes())
    h.update(inputs["table"].numpy().astype(np.int32).tobytes())
    h.update(inputs["lengths"].numpy().astype(np.int32).tobytes())
    return h.hexdigest()


def oracle_output(inputs, chunk=None):
    """Oracle FP32 output for ``build_case`` inputs, as float32 NumPy."""
    from oracle import dtype_bits_to_f32, paged_attention
    name = dtype_name(inputs["dtype"])
    q = dtype_bits_to_f32(to_bits(inputs["q"]), name).reshape(inputs["q"].shape)
    k = dtype_bits_to_f32(to_bits(inputs["k"]), name).reshape(inputs["k"].shape)
    v = dtype_bits_to_f32(to_bits(inputs["v"]), name).reshape(inputs["v"].shape)
    return paged_attention(q, k, v, inputs["table"].numpy(), inputs["lengths"].numpy(),
                           inputs["case"][5], inputs["causal"], chunk=chunk)


def visible_counts(lengths, sq, causal):
    """[B, Sq] number of keys each query row sees."""
    lengths = np.asarray(lengths, dtype=np.int64)[:, None]
    if causal:
        return np.maximum(lengths - sq + np.arange(sq)[None, :] + 1, 0)
    return np.broadcast_to(lengths, (lengths.shape[0], sq))
