"""NumPy FP32 restatement of FGW's CPU reference for paged MHA forward.

Test infrastructure, not product code (see ``oracle/__init__.py``).

Follows ``operators/mha/kernels/mha_paged_decode_ascend_v0.py:129-144`` (``reference``) and
``benchmarks/mha/bench_mha_mfu.py:38-66`` (``chunked_cpu_reference``, ``useful_flops``):

* only live tokens of request ``b`` are read: logical position ``t`` lives in pool row
  ``table[b, t // page] * page + t % page`` (v0.py:136);
* scores are ``q . k * D**-0.5`` in FP32 with the original head dimension D (v0.py:141);
* causal masking is right-aligned: query row ``i`` sees ``max(L - Sq + i + 1, 0)`` keys (v0.py:140);
* a row that sees no key is exactly zero (v0.py:134, 140; bench_mha_mfu.py:58 ``nan_to_num``);
* the FP32 result is cast to the input dtype (v0.py:143).

BF16 has no NumPy dtype, so BF16 tensors travel as ``uint16`` bit patterns; the helpers
below convert them (round-to-nearest-even on the way back, as a BF16 cast does).
"""
import numpy as np

_NAMES = {"bfloat16": "bfloat16", "torch.bfloat16": "bfloat16", "float16": "float16", "torch.float16": "float16"}


def _dtype_name(dtype):
    name = _NAMES.get(str(dtype))
    if name is None:
        raise ValueError(f"unsupported dtype {dtype!r}; expected float16 or bfloat16")
    return name


def bf16_bits_to_f32(bits):
    """Widen BF16 bit patterns (uint16) to float32 exactly."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x):
    """Round float32 to BF16 (nearest, ties to even); NaN stays a quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounded = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return rounded


def dtype_bits_to_f32(bits, dtype):
    """Widen FP16/BF16 bit patterns (uint16 array) to float32."""
    if _dtype_name(dtype) == "bfloat16":
        return bf16_bits_to_f32(bits)
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_dtype_bits(x, dtype):
    """Round float32 to FP16/BF16 and return the uint16 bit patterns."""
    if _dtype_name(dtype) == "bfloat16":
        return f32_to_bf16_bits(x)
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def _live_rows(table, b, length, page_size):
    pos = np.arange(length, dtype=np.int64)
    return table[b, pos // page_size].astype(np.int64) * page_size + pos % page_size


def _attend(query, keys, values, first_row, sq, length, causal, scale):
    """query [H, R, D] (rows first_row..), keys/values [H, L, D] -> [H, R, D] float32."""
    scores = np.matmul(query, keys.transpose(0, 2, 1)) * np.float32(scale)
    rows = query.shape[1]
    if causal:
        visible = np.maximum(length - sq + np.arange(first_row, first_row + rows) + 1, 0)
        mask = np.arange(length)[None, :] >= visible[:, None]
        scores = np.where(mask[None, :, :], np.float32(-np.inf), scores)
    else:
        visible = np.full(rows, length)
    peak = scores.max(axis=-1, keepdims=True)
    peak = np.where(np.isfinite(peak), peak, np.float32(0.0))
    weights = np.exp(scores - peak, dtype=np.float32)
    total = weights.sum(axis=-1, keepdims=True, dtype=np.float32)
    probabilities = weights / np.where(total > 0, total, np.float32(1.0))
    out = np.matmul(probabilities.astype(np.float32), values)
    out[:, visible == 0, :] = 0.0
    return out


def paged_attention(q, k, v, table, lengths, page_size, causal, chunk=None):
    """FP32 paged attention. Returns float32 ``[B, Sq, H, D]`` (cast separately).

    ``q`` is ``[B, Sq, H, D]``, ``k``/``v`` are ``[N, H, D]`` pools (any float dtype, widened
    to float32), ``table`` is ``[B, W]`` physical page ids, ``lengths`` is ``[B]``.
    ``chunk`` bounds the score workspace by processing that many query rows at a time, as
    ``chunked_cpu_reference`` does (bench_mha_mfu.py:51-59); ``None`` processes all rows.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    table = np.asarray(table)
    lengths = np.asarray(lengths)
    batch, sq, heads, dim = q.shape
    if k.shape[1:] != (heads, dim) or v.shape != k.shape:
        raise ValueError("K/V pools must be [N, H, D] matching Q")
    scale = dim ** -0.5
    out = np.zeros((batch, sq, heads, dim), dtype=np.float32)
    step = sq if not chunk else int(chunk)
    for b in range(batch):
        length = int(lengths[b])
        if length <= 0:
            continue
        rows = _live_rows(table, b, length, page_size)
        keys = np.ascontiguousarray(k[rows].transpose(1, 0, 2))
        values = np.ascontiguousarray(v[rows].transpose(1, 0, 2))
        for start in range(0, sq, step):
            stop = min(start + step, sq)
            query = np.ascontiguousarray(q[b, start:stop].transpose(1, 0, 2))
            out[b, start:stop] = _attend(query, keys, values, start, sq, length, causal, scale).transpose(1, 0, 2)
    return out


def paged_attention_chunked(q, k, v, table, lengths, page_size, causal, chunk=128):
    """Bounded-workspace variant used for long queries (bench_mha_mfu.py:38-60)."""
    return paged_attention(q, k, v, table, lengths, page_size, causal, chunk=chunk)


def useful_flops(lengths, sq, heads, dim, causal):
    """QK + PV FLOPs over visible pairs only (bench_mha_mfu.py:63-66)."""
    pairs = 0
    for length in lengths:
        length = int(length)
        if causal:
            # sum_{i<sq} max(length - sq + i + 1, 0), in closed form
            top = length
            bottom = length - sq + 1
            if top <= 0:
                continue
            bottom = max(bottom, 1)
            pairs += (top + bottom) * (top - bottom + 1) // 2
        else:
            pairs += length * sq
    return 4 * heads * dim * pairs


def algorithmic_bytes(lengths, batch, sq, heads, dim, width, elem_bytes):
    """Bytes the path must move at minimum: live K+V, Q+O, block table and lengths."""
    live = sum(int(n) for n in lengths)
    return (live * heads * dim * 2 * elem_bytes + 2 * batch * sq * heads * dim * elem_bytes
            + 4 * batch * width + 4 * batch)
