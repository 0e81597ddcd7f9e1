"""The C-ABI library loads, exports what include/fgw_mha.h declares, and rejects bad arguments.

These run without a GPU: no entry point that launches work is called with valid arguments.
"""
import ctypes
import pathlib
import re

import pytest

from fgw_b200 import _native

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "fgw_mha.h"


def declared_functions():
    text = HEADER.read_text(encoding="utf-8")
    return sorted(set(re.findall(r"FGW_API\s+[\w\s\*]*?\b(fgw_\w+)\s*\(", text)))


def test_header_declares_the_exported_set():
    assert declared_functions() == sorted(_native.EXPORTED)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert _native.abi_version() == _native.ABI_VERSION == 5


def test_status_strings():
    assert _native.status_string(0) == "ok"
    assert _native.status_string(5) == "device-side wait timed out"
    assert _native.status_string(99) == "unknown status"


def test_params_struct_layout_matches_header():
    # int64 pool_rows after six pointers; 14 int32 fields (schedule, then tensor_kernel) + 2 reserved.
    assert _native.Params.pool_rows.offset == 6 * 8
    assert _native.Params.schedule.offset == 6 * 8 + 8 + 12 * 4
    assert _native.Params.tensor_kernel.offset == 6 * 8 + 8 + 13 * 4
    assert ctypes.sizeof(_native.Params) == 6 * 8 + 8 + 16 * 4


def test_schedule_is_validated_and_sizes_the_workspace():
    # contiguous schedule (tensor path, one split, head_dim <= 128) adds the plan arrays and partial slots
    strided = _native.workspace_size(_params(q_len=4096, num_splits=1, path=_native.PATH_TENSOR,
                                             schedule=_native.SCHEDULE_STRIDED))
    contiguous = _native.workspace_size(_params(q_len=4096, num_splits=1, path=_native.PATH_TENSOR,
                                                schedule=_native.SCHEDULE_CONTIGUOUS))
    slots = 2 * 148 * 256 * (128 + 1) * 4
    assert contiguous >= strided + slots
    # AUTO: contiguous only with fewer than 2/3 x 148 work items (here 2 x 2 x 16 = 64)
    assert _native.workspace_size(_params(q_len=4096, num_splits=1, path=_native.PATH_TENSOR)) == contiguous
    many = dict(batch=8, heads=16, q_len=4096, num_splits=1, path=_native.PATH_TENSOR)  # 2048 items
    assert (_native.workspace_size(_params(**many))
            == _native.workspace_size(_params(schedule=_native.SCHEDULE_STRIDED, **many)))
    with pytest.raises(_native.FgwError):
        _native.check(_native.library().fgw_mha_paged_fwd(ctypes.byref(_params(schedule=4)), None, 0, None),
                      "fgw_mha_paged_fwd")
    # splits > 1 or the decode path keep the strided layout
    assert (_native.workspace_size(_params(q_len=4096, num_splits=2, path=_native.PATH_TENSOR))
            == _native.workspace_size(_params(q_len=4096, num_splits=2, path=_native.PATH_TENSOR,
                                              schedule=_native.SCHEDULE_STRIDED)))


def _params(**overrides):
    p = _native.Params()
    for key, value in dict(pool_rows=512, batch=2, q_len=1, heads=2, head_dim=128, table_width=4, page_size=128,
                           dtype=_native.DTYPE_BFLOAT16, num_splits=2).items():
        setattr(p, key, value)
    for key, value in overrides.items():
        setattr(p, key, value)
    return p


def test_workspace_size_grows_with_splits():
    one = _native.workspace_size(_params(num_splits=1, schedule=_native.SCHEDULE_STRIDED))
    four = _native.workspace_size(_params(num_splits=4))
    rows = 2 * 1 * 2
    assert four - one >= rows * 4 * (128 + 1) * 4
    with pytest.raises(_native.FgwError):
        _native.workspace_size(_params(batch=0))


def test_split_decode_workspace_holds_one_arrival_counter_per_row():
    # the decode path merges its splits in place: one int32 counter per output row group, upper-bounded by the
    # rows (a 256-byte aligned region after the partials); the tensor path keeps its merge launch, no counters
    rows = 8 * 3 * 4
    shape = dict(batch=8, q_len=3, heads=4, num_splits=4)
    decode = _native.workspace_size(_params(path=_native.PATH_DECODE, **shape))
    tensor = _native.workspace_size(_params(path=_native.PATH_TENSOR, **shape))
    assert decode - tensor == -(-rows * 4 // 256) * 256
    single = dict(shape, num_splits=1)
    strided = dict(single, schedule=_native.SCHEDULE_STRIDED)
    assert (_native.workspace_size(_params(path=_native.PATH_DECODE, **strided))
            == _native.workspace_size(_params(path=_native.PATH_TENSOR, **strided)))


@pytest.mark.parametrize("override", [dict(head_dim=24), dict(head_dim=272), dict(page_size=24),
                                      dict(pool_rows=500), dict(num_splits=0), dict(dtype=7), dict(causal=2),
                                      dict(path=9)])
def test_invalid_arguments_rejected_before_any_launch(override):
    p = _params(**override)
    buf = ctypes.create_string_buffer(1 << 16)
    status = _native.library().fgw_mha_paged_fwd(ctypes.byref(p), ctypes.addressof(buf), 1 << 16, None)
    assert status == _native.ERR_INVALID_ARGUMENT


def test_null_pointers_rejected():
    p = _params()
    status = _native.library().fgw_mha_paged_fwd(ctypes.byref(p), None, 0, None)
    assert status == _native.ERR_INVALID_ARGUMENT


def test_resolve_path_respects_explicit_choice():
    assert _native.resolve_path(_params(path=_native.PATH_DECODE)) == _native.PATH_DECODE
    assert _native.resolve_path(_params(path=_native.PATH_TENSOR)) == _native.PATH_TENSOR


def test_gather_params_layout_matches_header():
    # six pointers, int64 total_rows, seven int32 fields (the last is out_dtype) + 3 reserved
    assert _native.GatherParams.total_rows.offset == 6 * 8
    assert _native.GatherParams.out_dtype.offset == 6 * 8 + 8 + 6 * 4
    assert ctypes.sizeof(_native.GatherParams) == 6 * 8 + 8 + 10 * 4


def _gather(**overrides):
    g = _native.GatherParams()
    for key, value in dict(total_rows=0, batch=2, num_pages=8, page_size=16, table_width=4, row_width=256,
                           dtype=_native.DTYPE_BFLOAT16, out_dtype=_native.DTYPE_BFLOAT16).items():
        setattr(g, key, value)
    for key, value in overrides.items():
        setattr(g, key, value)
    return g


def _gather_status(g):
    return _native.library().fgw_paged_cache_gather(ctypes.byref(g), None)


def test_gather_argument_checks_without_a_device():
    # an empty gather is a no-op that never touches the device
    assert _gather_status(_gather()) == _native.OK
    bad = [dict(batch=0), dict(page_size=0), dict(row_width=0), dict(total_rows=-1),
           dict(out_dtype=_native.DTYPE_FLOAT16),                          # unquantized gather keeps the type
           dict(dtype=_native.DTYPE_FLOAT8_E4M3),                          # FP8 needs a scale
           dict(dtype=_native.DTYPE_FLOAT8_E4M3, out_dtype=_native.DTYPE_FLOAT8_E4M3, scale=8),
           dict(scale=8),                                                 # a scale only goes with FP8
           dict(page_size=1 << 20, table_width=1 << 12),                  # positions must fit int32
           dict(dtype=7), dict(total_rows=5)]                             # rows to write but no pointers
    for overrides in bad:
        g = _gather(**overrides)
        assert _gather_status(g) == _native.ERR_INVALID_ARGUMENT, overrides
    g = _gather()
    g.reserved[1] = 1
    assert _gather_status(g) == _native.ERR_INVALID_ARGUMENT


def test_resolved_schedule_per_path_and_kernel():
    # decode path with one split: the contiguous cut (slots of the decode kernel's query rows); with splits, or
    # when STRIDED is asked for, whole items
    decode = dict(batch=256, heads=32, q_len=1, num_splits=1, path=_native.PATH_DECODE)
    assert _native.resolve_schedule(_params(**decode)) == _native.SCHEDULE_STRIDED  # AUTO
    contiguous = dict(decode, schedule=_native.SCHEDULE_CONTIGUOUS)
    assert _native.resolve_schedule(_params(**contiguous)) == _native.SCHEDULE_CONTIGUOUS
    assert _native.resolve_schedule(_params(**dict(decode, num_splits=2))) == _native.SCHEDULE_STRIDED
    assert _native.resolve_schedule(_params(schedule=_native.SCHEDULE_STRIDED, **decode)) == _native.SCHEDULE_STRIDED
    assert _native.resolve_schedule(_params(schedule=_native.SCHEDULE_TAIL, **decode)) == _native.SCHEDULE_TAIL
    slots = 2 * 148 * 1 * (128 + 1) * 4  # D128 decode items carry one query row
    assert _native.workspace_size(_params(**contiguous)) >= _native.workspace_size(_params(**decode)) + slots
    # tensor path: the two-tile and key-halves kernels take the contiguous cut when asked for (with 256- and
    # 128-row slots), and on AUTO only when whole items would leave a third of the programs idle; the one-tile
    # kernel never does
    tensor = dict(q_len=4096, num_splits=1, path=_native.PATH_TENSOR, schedule=_native.SCHEDULE_CONTIGUOUS)
    assert _native.resolve_schedule(_params(**tensor)) == _native.SCHEDULE_CONTIGUOUS
    halves = dict(tensor, tensor_kernel=_native.TENSOR_KERNEL_HALVES, batch=8, heads=16)
    assert _native.resolve_schedule(_params(**halves)) == _native.SCHEDULE_CONTIGUOUS
    assert (_native.workspace_size(_params(**halves))
            >= _native.workspace_size(_params(**dict(halves, schedule=_native.SCHEDULE_STRIDED)))
            + 2 * 148 * 128 * (128 + 1) * 4)
    for kernel in (_native.TENSOR_KERNEL_PAIRS, _native.TENSOR_KERNEL_HALVES):
        auto = dict(tensor, schedule=_native.SCHEDULE_AUTO, tensor_kernel=kernel, batch=2, heads=8)  # config 2
        assert _native.resolve_schedule(_params(**auto)) == _native.SCHEDULE_STRIDED
        few = dict(auto, q_len=512, heads=4)  # 8 or 16 items: one partial wave
        assert _native.resolve_schedule(_params(**few)) == _native.SCHEDULE_CONTIGUOUS
    assert _native.resolve_schedule(_params(tensor_kernel=_native.TENSOR_KERNEL_SINGLE, **tensor)) == \
        _native.SCHEDULE_STRIDED
    with pytest.raises(_native.FgwError):
        _native.check(_native.library().fgw_mha_paged_fwd(ctypes.byref(_params(tensor_kernel=4)), None, 0, None),
                      "fgw_mha_paged_fwd")
