"""CUDA path vs FGW's reference outputs (golden) and vs the oracle, through the C ABI.

Tolerances are the reference harness's (test_mha_paged_accuracy.py:264): rtol/atol 1e-2/4e-3 for
BF16 and 2e-3/2e-3 for FP16, plus the north-star max-abs bound 2e-2 (BF16) / 5e-3 (FP16). Every
input pool is NaN-poisoned outside the live rows, and rows that see no key must be exactly zero.
"""
import numpy as np
import pytest
import torch

from fixtures import MAX_ABS, TOLERANCE, build_case, dtype_name, oracle_output, visible_counts
from golden_data import entry_params, expected_bits, output_index
from oracle import dtype_bits_to_f32

pytestmark = pytest.mark.gpu

ENTRIES = output_index()


def _run(inputs, **kwargs):
    from fgw_b200.operators.mha.current import mha_paged_decode
    dev = torch.device("cuda", 0)
    args = [inputs[k].to(dev) for k in ("q", "k", "v", "table", "lengths")]
    out = mha_paged_decode(*args, page_size=inputs["case"][5], is_causal=inputs["causal"], **kwargs)
    torch.cuda.synchronize()
    return out


def _check(out, expected_f32, inputs):
    name = dtype_name(inputs["dtype"])
    q = inputs["q"]
    assert out.shape == q.shape and out.dtype == q.dtype and out.is_contiguous()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "non-finite output"
    rtol, atol = TOLERANCE[name]
    err = np.abs(got - expected_f32)
    assert (err <= atol + rtol * np.abs(expected_f32)).all(), f"max err {err.max()}"
    assert err.max() <= MAX_ABS[name]
    vis = visible_counts(inputs["lengths"].tolist(), q.shape[1], inputs["causal"])
    assert not got[vis == 0].any(), "rows that see no key must be exactly zero"


@pytest.mark.parametrize("entry", ENTRIES, ids=[e["key"] for e in ENTRIES])
def test_matches_reference_golden(entry):
    case, seed, dtype, causal, pattern = entry_params(entry)
    inputs = build_case(case, seed, dtype, causal, pattern)
    expected = dtype_bits_to_f32(expected_bits(entry), dtype_name(dtype))
    out = _run(inputs)
    _check(out, expected, inputs)


SPLIT_CASES = [e for e in ENTRIES if e["seed"] == 7 and e["pattern"] != "empty"][::3]


@pytest.mark.parametrize("entry", SPLIT_CASES, ids=[e["key"] for e in SPLIT_CASES])
@pytest.mark.parametrize("splits", [2, 4, 32])
def test_explicit_splits_match_oracle(entry, splits):
    case, seed, dtype, causal, pattern = entry_params(entry)
    capacity_tiles = (case[5] * case[6] + 31) // 32
    if splits > capacity_tiles:
        pytest.skip("more splits than 32-token tiles in table capacity")
    inputs = build_case(case, seed, dtype, causal, pattern)
    out = _run(inputs, cube_mode="general", num_splits=splits)
    _check(out, oracle_output(inputs), inputs)


def test_native_library_is_loaded():
    from fgw_b200 import _native
    inputs = build_case(("tiny", 2, 2, 2, 16, 16, 2), 7, torch.bfloat16, False, "full")
    _run(inputs)
    assert _native._LIB is not None
    import pathlib
    maps = pathlib.Path("/proc/self/maps").read_text()
    assert "libfgw_mha.so" in maps


def test_config1_decode_parity():
    # B1 H1 D128 BF16, Q=1, KV=2048 in 128-token pages, 16 of 64 pages, split=1.
    gen = torch.Generator().manual_seed(7)
    table = torch.randperm(64, generator=gen)[:16].to(torch.int32).reshape(1, 16)
    q = torch.randn(1, 1, 1, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(64 * 128, 1, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(64 * 128, 1, 128, generator=gen).to(torch.bfloat16)
    inputs = {"case": ("config1", 1, 1, 1, 128, 128, 16), "q": q, "k": k, "v": v, "table": table,
              "lengths": torch.tensor([2048], dtype=torch.int32), "causal": False, "dtype": torch.bfloat16}
    out = _run(inputs, num_splits=1)
    _check(out, oracle_output(inputs), inputs)


def test_device_error_word_clean_after_call():
    from fgw_b200 import _native
    from fgw_b200.operators.mha.current import build_kernel
    inputs = build_case(("many_requests", 8, 2, 2, 64, 64, 4), 42, torch.float16, True, "mixed")
    dev = torch.device("cuda", 0)
    args = [inputs[k].to(dev) for k in ("q", "k", "v", "table", "lengths")]
    kernel = build_kernel(8, 2, 2, 64, args[1].shape[0], 4, 64, True, "float16", 0, cube_mode="general",
                          num_splits=4)
    ws = kernel.new_workspace(dev)
    kernel(*args, workspace=ws)
    status, site = _native.read_error(ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert (status, site) == (0, 0)


def test_bounded_wait_reports_timeout_and_context_survives():
    # A device wait on a phase nothing completes gives up after its budget and reports
    # FGW_ERR_DEVICE_TIMEOUT (site 99); the context stays usable for the next forward.
    import time
    from fgw_b200 import _native
    dev = torch.device("cuda", 0)
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    t0 = time.perf_counter()
    _native.selftest_wait(ws.data_ptr(), ws.numel(), 50, False, stream)
    assert _native.read_error(ws.data_ptr(), stream) == (_native.ERR_DEVICE_TIMEOUT, 99)
    assert 0.04 < time.perf_counter() - t0 < 5.0
    _native.selftest_wait(ws.data_ptr(), ws.numel(), 50, True, stream)
    assert _native.read_error(ws.data_ptr(), stream) == (_native.OK, 0)
    inputs = build_case(("after_timeout", 1, 130, 1, 128, 128, 2), 7, torch.bfloat16, False, "full")
    _check(_run(inputs), oracle_output(inputs), inputs)
