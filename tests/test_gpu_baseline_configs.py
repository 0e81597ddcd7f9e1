"""GPU parity at every BASELINE configuration's stated shape, against the oracle.

The golden-case tests hold the kernels to FGW's own reference outputs on the accuracy harness's small cases; these
hold them to the oracle (the NumPy restatement of FGW's reference(), pinned to those goldens) at the shapes the
benchmark configurations name:

* config 1: B1 H1 D128 BF16 Q1 KV2048, page 128, table = a seeded 16 of 64 pages;
* config 2: B2 H8 D128 BF16 Q4096 (and Q32768) KV2048, page 128, shuffled table: the whole output;
* config 3: {B1H1, B2H8} x {FP16, BF16} x Q{1, 4, 16, 64, 512} x KV{512, 2048, 8192, 32768}, full caches, page 128,
  at splits 1, 2, 8 and 32 and the automatic choice;
* config 4: B8 H16, D{16..256} x page{16, 64, 128} x causal Q{1, 8, 128}, lengths U[0, 8192] with an empty cache
  and partial tail pages, 1 % of K rows x8, unread pool rows NaN; on AUTO and on both forced kernel paths;
* config 5: B256 H32 D128 BF16 Q1, lengths log-uniform in [1024, 32768], 64-token pages scattered over the shared
  pool (about 39 GB of K and V): 32 requests, every head.

Inputs are drawn on the GPU from seeded generators; the oracle runs on each request's live rows copied back.
Tolerances are the harness's rtol/atol plus the north-star max-abs bound (``fixtures.TOLERANCE``, ``MAX_ABS``);
rows that see no key must be exact zeros.
"""
import numpy as np
import pytest
import torch

from fixtures import MAX_ABS, TOLERANCE, dtype_name
from oracle import dtype_bits_to_f32, paged_attention

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _f32(t):
    """float32 NumPy copy of a CPU or GPU FP16/BF16 tensor (bit-exact widening)."""
    t = t.contiguous().cpu()
    return dtype_bits_to_f32(t.view(torch.int16).numpy().view(np.uint16), dtype_name(t.dtype)).reshape(t.shape)


def _live_rows(table_row, length, page):
    pos = torch.arange(int(length), device=table_row.device)
    return table_row[pos // page].long() * page + pos % page


def _oracle_request(q, k, v, table, lengths, page, causal, b):
    """Oracle output [Sq, H, D] of request b from its live rows (a compact pool with an identity table)."""
    length = int(lengths[b])
    sq, heads, dim = q.shape[1:]
    if length == 0:
        return np.zeros((sq, heads, dim), dtype=np.float32)
    rows = _live_rows(table[b], length, page)
    pages = -(-length // page)
    kk = np.zeros((pages * page, heads, dim), dtype=np.float32)
    vv = np.zeros_like(kk)
    kk[:length] = _f32(k[rows])
    vv[:length] = _f32(v[rows])
    return paged_attention(_f32(q[b:b + 1]), kk, vv, np.arange(pages, dtype=np.int32)[None], np.array([length]),
                           page, causal, chunk=512 if sq > 512 else None)[0]


def _check_request(got, want, length, sq, causal, name, harness=True):
    """Finite, within the north-star max-abs bound and (``harness``) the reference harness's rtol/atol, rows that
    see no key exactly zero. The harness bound is the reference's for N(0,1) data; config 4's 1 % of K rows x8
    makes softmaxes so peaked that BF16 rounding of P (which the reference does too) and of outputs up to |4|
    (half an ulp there is 0.0156) exceed it, so that config is held to the north-star bound alone."""
    rtol, atol = TOLERANCE[name]
    assert np.isfinite(got).all(), "non-finite output"
    err = np.abs(got - want)
    assert err.max() <= MAX_ABS[name], f"max err {err.max()}"
    if harness:
        assert (err <= atol + rtol * np.abs(want)).all(), f"max err {err.max()}"
    vis = np.maximum(length - sq + np.arange(sq) + 1, 0) if causal else np.full(sq, length)
    assert not got[vis == 0].any(), "rows that see no key must be exactly zero"


def _check_all(out, q, k, v, table, lengths, page, causal, requests=None):
    name = dtype_name(q.dtype)
    got = out.float().cpu().numpy()
    for b in (range(q.shape[0]) if requests is None else requests):
        want = _oracle_request(q, k, v, table, lengths, page, causal, b)
        _check_request(got[b], want, int(lengths[b]), q.shape[1], causal, name)


def _pool(rows, heads, dim, dtype, gen):
    k = torch.randn(rows, heads, dim, generator=gen, device=DEV).to(dtype)
    v = torch.randn(rows, heads, dim, generator=gen, device=DEV).to(dtype)
    return k, v


def _poison_unread(k, v, table, lengths, page):
    live = torch.zeros(k.shape[0], dtype=torch.bool, device=DEV)
    for b, length in enumerate(lengths.tolist()):
        live[_live_rows(table[b], length, page)] = True
    k[~live] = float("nan")
    v[~live] = float("nan")


def test_config1_decode():
    gen = torch.Generator(device=DEV).manual_seed(7)
    table = torch.randperm(64, generator=torch.Generator().manual_seed(7))[:16].to(torch.int32)[None].to(DEV)
    k, v = _pool(64 * 128, 1, 128, torch.bfloat16, gen)
    q = torch.randn(1, 1, 1, 128, generator=gen, device=DEV).to(torch.bfloat16)
    lengths = torch.tensor([2048], dtype=torch.int32, device=DEV)
    from fgw_b200.operators.mha.current import mha_paged_decode
    for kwargs in ({}, {"cube_mode": "general", "num_splits": 1}):
        out = mha_paged_decode(q, k, v, table, lengths, 128, **kwargs)
        _check_all(out, q, k, v, table, lengths.cpu(), 128, False)


@pytest.mark.parametrize("sq,kernel", [(4096, "auto"), (4096, "halves"), (4096, "single"), (32768, "auto")])
def test_config2_long_query_whole_output(sq, kernel):
    from fgw_b200.operators.mha.current import mha_paged_decode
    batch, heads, dim, page, kv = 2, 8, 128, 128, 2048
    width = kv // page
    table = torch.randperm(batch * width, generator=torch.Generator().manual_seed(1000)).reshape(batch, width)
    table = table.to(torch.int32).to(DEV)
    gen = torch.Generator(device=DEV).manual_seed(1000)
    q = torch.randn(batch, sq, heads, dim, generator=gen, device=DEV).to(torch.bfloat16)
    k, v = _pool(batch * width * page, heads, dim, torch.bfloat16, gen)
    lengths = torch.full((batch,), kv, dtype=torch.int32, device=DEV)
    out = mha_paged_decode(q, k, v, table, lengths, page, tensor_kernel=kernel)
    _check_all(out, q, k, v, table, lengths.cpu(), page, False)


@pytest.mark.parametrize("dtype,causal,dim,kernel", [
    (torch.bfloat16, True, 128, "auto"), (torch.float16, False, 128, "auto"), (torch.bfloat16, False, 64, "auto"),
    (torch.bfloat16, True, 64, "halves"), (torch.float16, True, 256, "auto")],
    ids=["bf16_causal_d128", "fp16_d128", "bf16_d64", "bf16_causal_d64_halves", "fp16_causal_d256"])
def test_config2_shape_variants_whole_output(dtype, causal, dim, kernel):
    # Config 2's shape (B2 H8 Q4096 KV2048, page 128, shuffled table) with the other dtype, causal masking and the
    # other head-dimension blocks (D64: one 64-column block per operand; D256: the one-tile kernel), whole output.
    from fgw_b200.operators.mha.current import mha_paged_decode
    batch, heads, page, kv, sq = 2, 8, 128, 2048, 4096
    width = kv // page
    table = torch.randperm(batch * width, generator=torch.Generator().manual_seed(77)).reshape(batch, width)
    table = table.to(torch.int32).to(DEV)
    gen = torch.Generator(device=DEV).manual_seed(77 + dim)
    q = torch.randn(batch, sq, heads, dim, generator=gen, device=DEV).to(dtype)
    k, v = _pool(batch * width * page, heads, dim, dtype, gen)
    lengths = torch.tensor([kv, kv - 333], dtype=torch.int32, device=DEV)
    kwargs = {} if kernel == "auto" else {"path": "tensor", "tensor_kernel": kernel}
    out = mha_paged_decode(q, k, v, table, lengths, page, causal, **kwargs)
    _check_all(out, q, k, v, table, lengths.cpu(), page, causal)


CONFIG3 = [(b, h, sq, kv) for (b, h) in ((1, 1), (2, 8)) for sq in (1, 4, 16, 64, 512)
           for kv in (512, 2048, 8192, 32768)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("b,h,sq,kv", CONFIG3, ids=[f"B{b}H{h}_Q{sq}_KV{kv}" for b, h, sq, kv in CONFIG3])
def test_config3_split_sweep_points(b, h, sq, kv, dtype):
    # every split count of the reference's set that the table holds (general route: 32-token tiles), and auto
    from fgw_b200.operators.mha.current import mha_paged_decode
    page, dim = 128, 128
    width = kv // page
    gen = torch.Generator(device=DEV).manual_seed(31 + b + kv + sq)
    table = torch.randperm(b * width, device=DEV, generator=gen).reshape(b, width).to(torch.int32)
    q = torch.randn(b, sq, h, dim, generator=gen, device=DEV).to(dtype)
    k, v = _pool(b * width * page, h, dim, dtype, gen)
    lengths = torch.full((b,), kv, dtype=torch.int32, device=DEV)
    name = dtype_name(dtype)
    want = [_oracle_request(q, k, v, table, lengths.cpu(), page, False, r) for r in range(b)]
    runs = [dict(cube_mode="general", num_splits=s) for s in (1, 2, 8, 32) if s <= (kv + 31) // 32] + [{}]
    for kwargs in runs:
        out = mha_paged_decode(q, k, v, table, lengths, page, **kwargs).float().cpu().numpy()
        for r in range(b):
            _check_request(out[r], want[r], kv, sq, False, name)


CONFIG4 = [(d, p, sq) for d in (16, 32, 64, 96, 128, 192, 256) for p in (16, 64, 128) for sq in (1, 8, 128)]


@pytest.mark.parametrize("dim,page,sq", CONFIG4, ids=[f"D{d}_page{p}_Q{sq}" for d, p, sq in CONFIG4])
def test_config4_edge_grid(dim, page, sq):
    from fgw_b200.operators.mha.current import mha_paged_decode
    batch, heads, kv_max = 8, 16, 8192
    seed = 2026 + dim * 7 + page * 3 + sq
    dtype = torch.float16 if (dim // 16 + page + sq) % 2 else torch.bfloat16
    rng = np.random.default_rng(seed)
    lengths = rng.integers(0, kv_max + 1, size=batch)
    lengths[0] = 0                                  # an empty cache
    lengths[1] = (int(lengths[1]) // page) * page + page // 2 if page > 1 else int(lengths[1])  # partial tail page
    lengths = np.minimum(lengths, kv_max)
    width = kv_max // page
    pool_pages = batch * width + 1
    gen = torch.Generator(device=DEV).manual_seed(seed)
    table = torch.randperm(pool_pages, device=DEV, generator=gen)[: batch * width].reshape(batch, width).to(torch.int32)
    q = torch.randn(batch, sq, heads, dim, generator=gen, device=DEV).to(dtype)
    k, v = _pool(pool_pages * page, heads, dim, dtype, gen)
    big = torch.randperm(k.shape[0], device=DEV, generator=gen)[: k.shape[0] // 100]
    k[big] = (k[big].float() * 8).to(dtype)         # 1 % of K rows x8 stresses the running max
    lengths_t = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    _poison_unread(k, v, table, lengths_t.cpu(), page)
    name = dtype_name(dtype)
    want = [_oracle_request(q, k, v, table, lengths, page, True, b) for b in range(batch)]
    runs = [dict(), dict(path="decode"), dict(path="tensor")]
    if dim <= 128:
        runs.append(dict(path="tensor", tensor_kernel="halves"))
    for kwargs in runs:
        out = mha_paged_decode(q, k, v, table, lengths_t, page, True, **kwargs).float().cpu().numpy()
        for b in range(batch):
            _check_request(out[b], want[b], int(lengths[b]), sq, True, name, harness=False)


def test_config5_serving_decode_32_requests_every_head():
    import bench
    from fgw_b200.operators.mha.current import mha_paged_decode
    inp = bench.decode_inputs(4242, 0, 1, DEV, 256)
    out = mha_paged_decode(inp["q"], inp["k"], inp["v"], inp["table"], inp["lengths"], inp["page"],
                           cache_lengths=inp["host_lengths"])
    lengths = np.asarray(inp["host_lengths"])
    longest = list(np.argsort(-lengths, kind="stable")[:16])
    others = list(np.random.default_rng(5).choice([i for i in range(256) if i not in longest], 16, replace=False))
    _check_all(out, inp["q"], inp["k"], inp["v"], inp["table"], lengths, inp["page"], False,
               requests=sorted(int(x) for x in longest + others))
    del inp, out
    torch.cuda.empty_cache()
