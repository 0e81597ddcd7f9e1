"""Pins the NumPy oracle to FGW's own CPU reference through the committed golden outputs."""
import numpy as np
import pytest
import torch

from fixtures import build_case, dtype_name, input_digest, visible_counts
from golden_data import entry_params, expected_bits, flops_rows, output_index
from oracle import (algorithmic_bytes, dtype_bits_to_f32, f32_to_bf16_bits, f32_to_dtype_bits, lse_merge,
                    paged_attention, raw_state_merge, useful_flops)

ENTRIES = output_index()


def _oracle_bits(inputs):
    from fixtures import oracle_output
    return f32_to_dtype_bits(oracle_output(inputs), dtype_name(inputs["dtype"]))


@pytest.mark.parametrize("entry", ENTRIES, ids=[e["key"] for e in ENTRIES])
def test_oracle_matches_reference_outputs(entry):
    case, seed, dtype, causal, pattern = entry_params(entry)
    inputs = build_case(case, seed, dtype, causal, pattern)
    assert inputs["lengths"].tolist() == entry["lengths"]
    assert input_digest(inputs) == entry["input_sha256"], "fixture RNG stream drifted from the golden inputs"
    got = _oracle_bits(inputs)
    want = expected_bits(entry)
    name = dtype_name(dtype)
    got_f = dtype_bits_to_f32(got, name)
    want_f = dtype_bits_to_f32(want, name)
    assert np.isfinite(got_f).all()
    # Same FP32 algorithm, different summation order: allow one rounding step of the output dtype.
    ulp = 2.0 ** -7 if name == "bfloat16" else 2.0 ** -10
    np.testing.assert_allclose(got_f, want_f, rtol=ulp, atol=ulp * 2.0 ** -6)
    assert (got == want).mean() > 0.95
    vis = visible_counts(entry["lengths"], case[2], causal)
    assert not got_f[vis == 0].any(), "rows that see no key must be exactly zero"


def test_chunked_oracle_equals_unchunked():
    case = ("chunk", 2, 300, 2, 64, 32, 5)
    for causal in (False, True):
        inputs = build_case(case, 7, torch.bfloat16, causal, "mixed")
        from fixtures import oracle_output
        np.testing.assert_allclose(oracle_output(inputs, chunk=128), oracle_output(inputs), rtol=0, atol=1e-6)


@pytest.mark.parametrize("row", flops_rows()[:200])
def test_useful_flops_matches_reference(row):
    lengths, sq, heads, dim, causal, expected = row
    assert useful_flops(lengths, sq, heads, dim, causal) == expected


def test_algorithmic_bytes_config1():
    # B1 H1 D128 BF16, KV 2048, W 16: live K+V + Q+O + table + lengths.
    assert algorithmic_bytes([2048], 1, 1, 1, 128, 16, 2) == 2048 * 128 * 2 * 2 + 2 * 128 * 2 + 64 + 4


def test_bf16_rounding_ties_to_even_and_nan():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, np.nan], dtype=np.float32)
    bits = f32_to_bf16_bits(x)
    torch_bits = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert (bits[:5] == torch_bits[:5]).all()
    assert np.isnan(dtype_bits_to_f32(bits[5:], "bfloat16")).all()


def test_merge_oracles_match_dense_attention():
    # Independent dense attention vs split partials, with an empty partition
    # (mirrors FGW tests/mha/test_raw_partial_state.py:7-26).
    import math
    keys = [(1., 2.), (-3., 4.), (5., -6.), (2., -1.), (-4., -2.), (3., 5.)]
    values = [(2., -1.), (4., 3.), (-2., 5.), (7., -3.), (1., 6.), (-5., 8.)]
    for query in ((1., -2.), (-3., 4.), (100., -100.)):
        scores = [sum(a * b for a, b in zip(query, k)) / math.sqrt(2) for k in keys]
        peak = max(scores)
        w = [math.exp(x - peak) for x in scores]
        dense = [sum(wi * v[d] for wi, v in zip(w, values)) / sum(w) for d in range(2)]
        raw, lse = [], []
        for begin, end in ((0, 2), (2, 5), (5, 6)):
            m = max(scores[begin:end])
            e = [math.exp(x - m) for x in scores[begin:end]]
            acc = [sum(a * v[d] for a, v in zip(e, values[begin:end])) for d in range(2)]
            raw.append((acc, m, sum(e)))
            lse.append(([a / sum(e) for a in acc], m + math.log(sum(e))))
        raw.append(([0., 0.], -1e30, 0.))
        lse.append(([0., 0.], -1e30))
        for got in (raw_state_merge(raw), lse_merge(lse)):
            for a, b in zip(got, dense):
                assert abs(a - b) < 1e-12


def test_oracle_masks_nan_rows_and_empty_requests():
    q = np.ones((2, 3, 1, 16), np.float32)
    k = np.full((64, 1, 16), np.nan, np.float32)
    v = np.full((64, 1, 16), np.nan, np.float32)
    k[16:18] = 0.5
    v[16:18] = 2.0
    table = np.array([[1, 0], [2, 3]], np.int32)
    out = paged_attention(q, k, v, table, np.array([2, 0]), 16, causal=True)
    assert np.isfinite(out).all()
    assert (out[1] == 0).all()
    assert (out[0, 0] == 0).all()  # row 0 sees max(2 - 3 + 1, 0) = 0 keys
    np.testing.assert_allclose(out[0, 1:], 2.0)
