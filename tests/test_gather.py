"""Paged-cache gather pre-pass: the oracle against the reference experiment's exact check (CPU), and the CUDA
gather bit for bit against the oracle plus gather-then-attend against direct attention (GPU).

Case matrix: FGW's cube/vector benchmark cases (benchmarks/mha/bench_cube_vector.py:14-26) plus the three
gather-specific cases of benchmarks/mha/bench_external_gather.py:10-13, each as
(name, batch, sq, heads, dim, page, width, lengths, causal).
"""
import numpy as np
import pytest

from oracle.gather import e4m3_to_f32, paged_cache_gather as oracle_gather, reference_packed_check

CASES = [(f"dim{d}_q16", 2, 16, 2, d, 128, 4, (512, 512), False) for d in (16, 48, 64, 80, 96, 128, 192, 256)]
CASES += [(f"d{d}_q{q}_kv2048", 2, q, 2, d, 128, 16, (2048, 2048), False) for d in (64, 128) for q in (1, 128, 512)]
CASES += [
    ("single_decode_kv8192", 1, 1, 1, 64, 256, 32, (8192,), False),
    ("page16_tail", 2, 4, 2, 16, 16, 8, (127, 113), False),
    ("page48_crossing", 2, 33, 2, 48, 48, 4, (191, 145), False),
    ("d128_q129_kv_tail", 2, 129, 2, 128, 128, 4, (511, 257), False),
    ("causal_d64_q16", 2, 16, 2, 64, 128, 4, (512, 512), True),
    ("causal_d128_q129", 2, 129, 2, 128, 128, 2, (256, 256), True),
    ("causal_empty_rows_d256", 2, 33, 2, 256, 128, 2, (17, 0), True),
    ("gather_fast_page16", 2, 17, 4, 256, 16, 16, (255, 129), False),
    ("gather_fast_page64", 2, 16, 3, 192, 64, 4, (256, 192), False),
    ("gather_zero_mixed", 2, 35, 2, 64, 128, 4, (0, 259), True),
]


def _packed(lengths, page):
    offsets = [0]
    for length in lengths:
        offsets.append(offsets[-1] + (length + page - 1) // page * page)
    return offsets


def _case_arrays(case, seed=7):
    _, b, _, h, d, page, width, lengths, _ = case
    rng = np.random.default_rng(seed)
    pages = b * width + 3
    cache = rng.integers(0, 1 << 16, size=(pages, page, h, d), dtype=np.uint16)
    table = rng.permutation(pages)[:b * width].reshape(b, width).astype(np.int32)
    return cache, table


# --- CPU: the oracle against the reference's own exact check ---------------------------------------------
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_packed_check(case):
    _, b, _, h, d, page, width, lengths, _ = case
    cache, table = _case_arrays(case)
    cu = _packed(lengths, page)
    got = oracle_gather(cache, table, cu)
    assert np.array_equal(got, reference_packed_check(cache, table, lengths, page))


def test_oracle_edges():
    rng = np.random.default_rng(3)
    cache = rng.integers(1, 1 << 16, size=(6, 16, 8), dtype=np.uint16)  # no zero words: zeros mean "not read"
    table = np.array([[5, 2, 9], [0, 1, 3]], dtype=np.int32)           # page 9 is outside the pool
    cu = [2, 20, 30]
    out = oracle_gather(cache, table, cu, total_rows=34, starts=[3, -2])
    flat = cache.reshape(-1, 8)
    assert not out[:2].any()                                            # before cu[0]
    for r in range(2, 20):                                              # request 0, positions 3..20
        pos = r - 2 + 3
        assert np.array_equal(out[r], flat[table[0, pos // 16] * 16 + pos % 16])
    assert not out[20:22].any()                                         # request 1, positions -2, -1
    for r in range(22, 30):
        pos = r - 20 - 2
        assert np.array_equal(out[r], flat[table[1, pos // 16] * 16 + pos % 16])
    assert not out[30:].any()                                           # past cu[batch]
    # page 9 does not exist: positions 32..47 of request 0 read nothing
    out = oracle_gather(cache, table, [0, 48, 48])
    assert not out[32:48].any() and out[:32].all()


def test_e4m3_known_answers():
    codes = np.array([0x00, 0x80, 0x38, 0xB8, 0x01, 0x08, 0x7E, 0xFE, 0x3C, 0x40, 0x7F, 0xFF], dtype=np.uint8)
    want = [0.0, -0.0, 1.0, -1.0, 2.0 ** -9, 2.0 ** -6, 448.0, -448.0, 1.5, 2.0]
    got = e4m3_to_f32(codes)
    assert list(got[:10]) == want and np.signbit(got[1])
    assert np.isnan(got[10]) and np.isnan(got[11])


# --- GPU: the CUDA gather and the gather-then-attend pipeline -------------------------------------------
def _torch():
    return pytest.importorskip("torch")


def _bits(torch, t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_gather_bit_exact(case, dtype):
    torch = _torch()
    from fgw_b200.operators.mha.paged_cache_gather import paged_cache_gather
    _, b, _, h, d, page, width, lengths, _ = case
    cache_bits, table = _case_arrays(case)
    dev = torch.device("cuda", 0)
    tdtype = getattr(torch, dtype)
    cache = torch.from_numpy(cache_bits.view(np.int16)).to(dev).view(tdtype)
    cu = _packed(lengths, page)
    dst = torch.full((cu[-1], h, d), float("nan"), dtype=tdtype, device=dev)
    paged_cache_gather(dst, cache, torch.from_numpy(table).to(dev), torch.tensor(cu, dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(torch, dst), oracle_gather(cache_bits, table, cu))


@pytest.mark.gpu
@pytest.mark.parametrize("row_width", [24, 20, 1024])  # 48 B rows (vector path), 40 B rows (scalar path), 2 KB
def test_gather_edges_starts_zero_rows_bad_pages(row_width):
    torch = _torch()
    from fgw_b200.operators.mha.paged_cache_gather import paged_cache_gather
    rng = np.random.default_rng(row_width)
    pages, page, b, width = 40, 16, 5, 6
    cache_bits = rng.integers(1, 1 << 16, size=(pages, page, row_width), dtype=np.uint16)
    table = rng.integers(0, pages, size=(b, width)).astype(np.int32)
    table[1, 2] = pages + 7          # outside the pool: zeros
    table[3, 0] = -1
    cu = [4, 40, 40, 71, 90, 100]    # rows 0..3 before the first request; request 1 empty
    starts = np.array([5, 0, -3, 90, 2], dtype=np.int32)  # request 3 runs past the table (6 pages x 16)
    total = 110                      # rows 100..109 past cu[batch]
    dev = torch.device("cuda", 0)
    dst = torch.full((total, row_width), float("nan"), dtype=torch.bfloat16, device=dev)
    paged_cache_gather(dst, torch.from_numpy(cache_bits.view(np.int16)).to(dev).view(torch.bfloat16),
                       torch.from_numpy(table).to(dev), torch.tensor(cu, dtype=torch.int32, device=dev),
                       seq_starts=torch.from_numpy(starts).to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(torch, dst), oracle_gather(cache_bits, table, cu, total_rows=total, starts=starts))


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("row_width", [576, 1024, 40])
def test_gather_fp8_dequantise(out_dtype, row_width):
    torch = _torch()
    if not hasattr(torch, "float8_e4m3fn"):
        pytest.skip("torch without float8_e4m3fn")
    from fgw_b200.operators.mha.paged_cache_gather import paged_cache_gather
    rng = np.random.default_rng(11)
    pages, page, b, width = 24, 64, 3, 5
    codes = rng.integers(0, 256, size=(pages, page, row_width), dtype=np.uint8)
    table = rng.permutation(pages)[:b * width].reshape(b, width).astype(np.int32)
    lengths = (300, 0, 129)
    cu = _packed(lengths, page)
    scale = np.float32(0.0371)
    dev = torch.device("cuda", 0)
    cache = torch.from_numpy(codes).to(dev).view(torch.float8_e4m3fn)
    dst = torch.empty((cu[-1], row_width), dtype=getattr(torch, out_dtype), device=dev)
    paged_cache_gather(dst, cache, torch.from_numpy(table).to(dev), torch.tensor(cu, dtype=torch.int32, device=dev),
                       scale=torch.tensor([scale], dtype=torch.float32, device=dev))
    torch.cuda.synchronize()
    want = oracle_gather(codes, table, cu, scale=scale, out_dtype=out_dtype)
    got = _bits(torch, dst)
    nan = np.isnan(e4m3_to_f32(reference_packed_check(codes, table, lengths, page)))  # NaN codes: any NaN
    fnan = np.isnan(got.view(np.float16).astype(np.float32)) if out_dtype == "float16" else \
        np.isnan((got.astype(np.uint32) << 16).view(np.float32))
    assert np.array_equal(fnan, nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.gpu
def test_gather_validation_errors():
    torch = _torch()
    from fgw_b200.operators.mha.paged_cache_gather import paged_cache_gather
    dev = torch.device("cuda", 0)
    cache = torch.zeros((4, 16, 2, 8), dtype=torch.float16, device=dev)
    table = torch.zeros((2, 4), dtype=torch.int32, device=dev)
    cu = torch.tensor([0, 16, 32], dtype=torch.int32, device=dev)
    dst = torch.empty((32, 2, 8), dtype=torch.float16, device=dev)
    bad = [dict(dst=dst.bfloat16()), dict(dst=torch.empty((32, 2, 4), dtype=torch.float16, device=dev)),
           dict(cu_seq_lens=cu[:2]), dict(block_table=table.long()), dict(cu_seq_lens=cu.cpu()),
           dict(scale=torch.ones(1, device=dev)), dict(seq_starts=torch.zeros(3, dtype=torch.int32, device=dev)),
           dict(dst=torch.empty((2, 32, 8), dtype=torch.float16, device=dev).transpose(0, 1))]
    for overrides in bad:
        args = dict(dst=dst, cache=cache, block_table=table, cu_seq_lens=cu)
        args.update(overrides)
        with pytest.raises(ValueError):
            paged_cache_gather(**args)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_gather_then_attend_equals_direct(case, dtype):
    torch = _torch()
    from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import build_kernel
    from fgw_b200.operators.mha.paged_cache_gather import build_gather_attention
    name, b, sq, h, d, page, width, lengths, causal = case
    dev = torch.device("cuda", 0)
    tdtype = getattr(torch, dtype)
    g = torch.Generator().manual_seed(42)
    pool_pages = b * width + 2
    q = torch.randn(b, sq, h, d, generator=g).to(tdtype).to(dev)
    k = torch.randn(pool_pages * page, h, d, generator=g).to(tdtype).to(dev)
    v = torch.randn(pool_pages * page, h, d, generator=g).to(tdtype).to(dev)
    table = torch.randperm(pool_pages, generator=g)[:b * width].reshape(b, width).int().to(dev)
    lens = torch.tensor(lengths, dtype=torch.int32, device=dev)
    direct = build_kernel(b, sq, h, d, pool_pages * page, width, page, causal, dtype, 0)
    run, info = build_gather_attention(b, sq, h, d, page, width, lengths, causal, dtype, 0)
    assert info["num_splits"] == direct.num_splits  # the split choice does not depend on the pool size
    want = direct(q, k, v, table, lens)
    got = run(q, k, v, table, lens)
    torch.cuda.synchronize()
    assert info["packed_rows"] == _packed(lengths, page)[-1]
    # same kernel, same splits, the same K/V values in the same logical order: identical bits
    assert torch.equal(got.view(torch.int16), want.view(torch.int16)), name
