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
    return sorted(set(re.findall(r"FGW_API\s+[\w\s\*]*?\b(fgw_mha_\w+)\s*\(", text)))


def test_header_declares_the_exported_set():
    assert declared_functions() == sorted(_native.EXPORTED)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert _native.abi_version() == 1


def test_status_strings():
    assert _native.status_string(0) == "ok"
    assert _native.status_string(5) == "device-side wait timed out"
    assert _native.status_string(99) == "unknown status"


def test_params_struct_layout_matches_header():
    # int64 pool_rows after six pointers; 12 int32 fields + 4 reserved.
    assert _native.Params.pool_rows.offset == 6 * 8
    assert ctypes.sizeof(_native.Params) == 6 * 8 + 8 + 16 * 4


def _params(**overrides):
    p = _native.Params()
    for key, value in dict(pool_rows=512, batch=2, q_len=1, heads=2, head_dim=128, table_width=4, page_size=128,
                           dtype=_native.DTYPE_BFLOAT16, num_splits=2).items():
        setattr(p, key, value)
    for key, value in overrides.items():
        setattr(p, key, value)
    return p


def test_workspace_size_grows_with_splits():
    one = _native.workspace_size(_params(num_splits=1))
    four = _native.workspace_size(_params(num_splits=4))
    rows = 2 * 1 * 2
    assert four - one >= rows * 4 * (128 + 1) * 4
    with pytest.raises(_native.FgwError):
        _native.workspace_size(_params(batch=0))


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
