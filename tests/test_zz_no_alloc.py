"""The allocation-free entry point gives the same output as the ordinary one.

``fgw_mha_paged_fwd_static_ws`` exists for callers that cannot allocate device memory where they run
attention (allocator callbacks, allocation-free serving loops, plugins whose host owns all memory): it
uses the library's own static scratch array instead of a caller workspace. This file runs last
(``zz``) so a stop-at-first-failure run has already covered everything else; it also passes alone.
"""
import pytest
import torch

from fixtures import MAX_ABS, TOLERANCE, build_case, dtype_name

pytestmark = pytest.mark.gpu


def _params_for(kernel, args, out):
    from fgw_b200 import _native
    p = _native.Params.from_buffer_copy(kernel.params)
    q, k, v, table, lengths = args
    p.q, p.k_cache, p.v_cache = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.block_table, p.cache_seqlens, p.out = table.data_ptr(), lengths.data_ptr(), out.data_ptr()
    return p


# (case, path, splits, falls back): split-KV cases so the scratch holds partials as well as the plan, and
# a one-split tensor case whose AUTO schedule is the contiguous one: its partial slots (2 x 148 x 256 x D
# FP32) do not fit the array, so the entry point runs it on the strided schedule.
CASES = [
    (("nz_decode", 4, 1, 2, 128, 64, 8), "decode", 4, False),
    (("nz_tensor", 2, 160, 2, 64, 16, 12), "tensor", 2, False),
    (("nz_tensor_one_split", 2, 160, 2, 64, 16, 12), "tensor", 1, True),
]


@pytest.mark.parametrize("case,path,splits,falls_back", CASES, ids=[c[0][0] for c in CASES])
def test_static_workspace_matches_regular_entry_point_twice(case, path, splits, falls_back):
    from fgw_b200 import _native
    from fgw_b200.operators.mha.current import build_kernel
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, (seed, pattern, causal) in enumerate([(7, "mixed", False), (42, "full", True)]):
        inputs = build_case(case, seed, torch.bfloat16, causal, pattern)
        args = [inputs[key].to(dev) for key in ("q", "k", "v", "table", "lengths")]
        kernel = build_kernel(case[1], case[2], case[3], case[4], args[1].shape[0], case[6], case[5], causal,
                              "bfloat16", 0, cube_mode="general", num_splits=splits, path=path)
        assert (kernel.workspace_bytes > _native.STATIC_WORKSPACE_BYTES) == falls_back
        strided = _native.Params.from_buffer_copy(kernel.params)
        strided.schedule = _native.SCHEDULE_STRIDED
        assert _native.workspace_size(strided) <= _native.STATIC_WORKSPACE_BYTES
        expected = kernel(*args)
        got = torch.full_like(expected, float("nan"))
        _native.paged_fwd_static_ws(_params_for(kernel, args, got), stream)
        torch.cuda.synchronize()
        rtol, atol = TOLERANCE[dtype_name(torch.bfloat16)]
        torch.testing.assert_close(got, expected, rtol=rtol, atol=atol, msg=f"call {call}")
        assert (got.float() - expected.float()).abs().max().item() <= MAX_ABS["bfloat16"]
        # the device-side status lives in the library's array; this entry point reads it back
        assert _native.static_ws_read_error(stream) == (_native.OK, 0)


def test_static_workspace_rejects_requests_beyond_its_size():
    from fgw_b200 import _native
    p = _native.Params()
    for key, value in dict(pool_rows=1 << 16, batch=4096, q_len=1, heads=32, head_dim=256, table_width=64,
                           page_size=64, dtype=_native.DTYPE_BFLOAT16, num_splits=16).items():
        setattr(p, key, value)
    assert _native.workspace_size(p) > _native.STATIC_WORKSPACE_BYTES
    with pytest.raises(_native.FgwError) as err:
        _native.paged_fwd_static_ws(p, torch.cuda.current_stream().cuda_stream)
    assert err.value.status == _native.ERR_WORKSPACE_TOO_SMALL
