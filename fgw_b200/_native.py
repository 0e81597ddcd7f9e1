"""ctypes binding of libfgw_mha.so (the C ABI declared in include/fgw_mha.h).

The library is loaded from ``fgw_b200/_lib`` (built in-tree by ``python -m fgw_b200.build``).
There is no fallback: if the library is missing or cannot be loaded, every entry point raises
``NativeLibraryError`` naming the file, so a GPU box without the built extension fails loudly.
"""
import ctypes
import pathlib

import numpy as np

LIB_PATH = pathlib.Path(__file__).resolve().parent / "_lib" / "libfgw_mha.so"

# fgw_status codes
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE_TOO_SMALL = 3
ERR_CUDA = 4
ERR_DEVICE_TIMEOUT = 5
ERR_NO_DEVICE = 6

DTYPE_FLOAT16 = 0
DTYPE_BFLOAT16 = 1
DTYPE_FLOAT8_E4M3 = 2  # paged-cache gather only

PATH_AUTO = 0
PATH_DECODE = 1
PATH_TENSOR = 2

# fgw_schedule
SCHEDULE_AUTO = 0
SCHEDULE_STRIDED = 1
SCHEDULE_CONTIGUOUS = 2
SCHEDULE_TAIL = 3

# fgw_tensor_kernel
TENSOR_KERNEL_AUTO = 0
TENSOR_KERNEL_PAIRS = 1
TENSOR_KERNEL_SINGLE = 2
TENSOR_KERNEL_HALVES = 3

ABI_VERSION = 5  # FGW_MHA_ABI_VERSION the Params / GatherParams / SplitModel layouts below match

EXPORTED = (
    "fgw_mha_abi_version",
    "fgw_mha_status_string",
    "fgw_mha_device_sm_count",
    "fgw_mha_choose_splits",
    "fgw_mha_resolve_path",
    "fgw_mha_resolve_schedule",
    "fgw_mha_workspace_size",
    "fgw_mha_paged_fwd",
    "fgw_mha_plan",
    "fgw_mha_attend",
    "fgw_mha_partial",
    "fgw_mha_merge",
    "fgw_mha_read_error",
    "fgw_mha_paged_fwd_static_ws",
    "fgw_mha_static_ws_read_error",
    "fgw_mha_selftest_wait",
    "fgw_paged_cache_gather",
)

STATIC_WORKSPACE_BYTES = 16 << 20  # FGW_MHA_STATIC_WORKSPACE_BYTES


class NativeLibraryError(RuntimeError):
    """libfgw_mha.so is absent or unusable."""


class FgwError(RuntimeError):
    """A C-ABI call returned a non-zero fgw_status."""

    def __init__(self, status, where):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (fgw_status {status})")


class Params(ctypes.Structure):
    """Mirror of ``fgw_mha_params`` (include/fgw_mha.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("cache_seqlens", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("pool_rows", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("table_width", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("grid_cap", ctypes.c_int32),
        ("path", ctypes.c_int32),
        ("wait_budget_ms", ctypes.c_int32),
        ("schedule", ctypes.c_int32),
        ("tensor_kernel", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 2),
    ]


SPLIT_MODEL_FEATURES = 10  # FGW_SPLIT_MODEL_FEATURES


class SplitModel(ctypes.Structure):
    """Mirror of ``fgw_split_model`` (include/fgw_mha.h): the B200 split cost model's weights and selection rule."""

    _fields_ = [
        ("weights", ctypes.c_double * SPLIT_MODEL_FEATURES),
        ("floor_single_us", ctypes.c_double),
        ("floor_multi_us", ctypes.c_double),
        ("tolerance", ctypes.c_double),
        ("absolute_margin_us", ctypes.c_double),
    ]

    @classmethod
    def from_model(cls, model):
        """From the version-3 model dict (models/b200_general_split_cost_model.json)."""
        if model["version"] != 3 or len(model["weights"]) != SPLIT_MODEL_FEATURES:
            raise ValueError("the native split choice takes the version-3 model")
        m = cls()
        m.weights[:] = [float(w) for w in model["weights"]]
        m.floor_single_us = model["latency_floor_us"]["single"]
        m.floor_multi_us = model["latency_floor_us"]["multi"]
        m.tolerance = model["selection_tolerance"]
        m.absolute_margin_us = model.get("absolute_selection_margin_us", 0.0)
        return m


class SplitChoice(ctypes.Structure):
    """Mirror of ``fgw_split_choice``."""

    _fields_ = [
        ("splits", ctypes.c_int32),
        ("full_kv_cache", ctypes.c_int32),
        ("min_length", ctypes.c_int32),
        ("max_length", ctypes.c_int32),
    ]


class GatherParams(ctypes.Structure):
    """Mirror of ``fgw_gather_params`` (include/fgw_mha.h)."""

    _fields_ = [
        ("dst", ctypes.c_void_p),
        ("cache", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("cu_seq_lens", ctypes.c_void_p),
        ("seq_starts", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("total_rows", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("table_width", ctypes.c_int32),
        ("row_width", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 3),
    ]


_LIB = None


def library():
    """The loaded ``ctypes.CDLL``; raises ``NativeLibraryError`` if it cannot be loaded."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise NativeLibraryError(
            f"{LIB_PATH} is missing: build it with `python -m fgw_b200.build` (nvcc 12.9, sm_100a). "
            "There is no CPU fallback for the paged MHA forward.")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
    missing = [name for name in EXPORTED if not hasattr(lib, name)]
    if missing:
        raise NativeLibraryError(f"{LIB_PATH} lacks exported symbols {missing}")
    lib.fgw_mha_abi_version.restype = ctypes.c_int
    if lib.fgw_mha_abi_version() != ABI_VERSION:
        raise NativeLibraryError(f"{LIB_PATH} has ABI version {lib.fgw_mha_abi_version()}, this binding expects "
                                 f"{ABI_VERSION}: rebuild with `python -m fgw_b200.build`")
    p = ctypes.POINTER(Params)
    vp = ctypes.c_void_p
    lib.fgw_mha_abi_version.argtypes = []
    lib.fgw_mha_abi_version.restype = ctypes.c_int
    lib.fgw_mha_status_string.argtypes = [ctypes.c_int]
    lib.fgw_mha_status_string.restype = ctypes.c_char_p
    lib.fgw_mha_device_sm_count.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.fgw_mha_device_sm_count.restype = ctypes.c_int
    # fgw_mha_choose_splits runs on every serving call: no argtypes (their per-argument conversion costs more than
    # the call), so choose_splits passes ctypes pointers and Python ints (C int by default)
    lib.fgw_mha_choose_splits.restype = ctypes.c_int
    lib.fgw_mha_resolve_path.argtypes = [p, ctypes.POINTER(ctypes.c_int)]
    lib.fgw_mha_resolve_path.restype = ctypes.c_int
    lib.fgw_mha_resolve_schedule.argtypes = [p, ctypes.POINTER(ctypes.c_int)]
    lib.fgw_mha_resolve_schedule.restype = ctypes.c_int
    lib.fgw_mha_workspace_size.argtypes = [p, ctypes.POINTER(ctypes.c_size_t)]
    lib.fgw_mha_workspace_size.restype = ctypes.c_int
    for name in ("fgw_mha_paged_fwd", "fgw_mha_plan", "fgw_mha_attend", "fgw_mha_partial", "fgw_mha_merge"):
        fn = getattr(lib, name)
        fn.argtypes = [p, vp, ctypes.c_size_t, vp]
        fn.restype = ctypes.c_int
    lib.fgw_mha_read_error.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
    lib.fgw_mha_read_error.restype = ctypes.c_int
    lib.fgw_mha_selftest_wait.argtypes = [vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, vp]
    lib.fgw_mha_selftest_wait.restype = ctypes.c_int
    lib.fgw_mha_paged_fwd_static_ws.argtypes = [p, vp]
    lib.fgw_mha_paged_fwd_static_ws.restype = ctypes.c_int
    lib.fgw_mha_static_ws_read_error.argtypes = [vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
    lib.fgw_mha_static_ws_read_error.restype = ctypes.c_int
    lib.fgw_paged_cache_gather.argtypes = [ctypes.POINTER(GatherParams), vp]
    lib.fgw_paged_cache_gather.restype = ctypes.c_int
    _LIB = lib
    return lib


def status_string(status):
    try:
        return library().fgw_mha_status_string(int(status)).decode()
    except NativeLibraryError:
        return f"status {status}"


def check(status, where):
    if status != OK:
        raise FgwError(status, where)


def abi_version():
    return library().fgw_mha_abi_version()


def device_sm_count(device):
    out = ctypes.c_int(0)
    check(library().fgw_mha_device_sm_count(int(device), ctypes.byref(out)), "fgw_mha_device_sm_count")
    return out.value


_INT32 = np.dtype(np.int32)


def choose_splits(model, host_lengths, batch, q_len, heads, head_dim, page_size, table_width, sm_count):
    """``fgw_mha_choose_splits`` on a C-contiguous int32 NumPy array of host cache lengths: returns the filled
    ``SplitChoice`` and the status (FGW_ERR_INVALID_ARGUMENT when a length is outside the table capacity)."""
    if host_lengths.dtype is not _INT32 or host_lengths.shape != (batch,) or host_lengths.strides != (4,):
        raise ValueError("host_lengths must be a C-contiguous int32 array of the batch's lengths")
    choice = SplitChoice()
    status = library().fgw_mha_choose_splits(
        ctypes.byref(model), ctypes.c_void_p(host_lengths.__array_interface__["data"][0]), int(batch), int(q_len),
        int(heads), int(head_dim), int(page_size), int(table_width), int(sm_count), ctypes.byref(choice))
    return choice, status


def resolve_path(params):
    out = ctypes.c_int(0)
    check(library().fgw_mha_resolve_path(ctypes.byref(params), ctypes.byref(out)), "fgw_mha_resolve_path")
    return out.value


def resolve_schedule(params):
    """The schedule (SCHEDULE_STRIDED / _CONTIGUOUS / _TAIL) the main launch takes for ``params``."""
    out = ctypes.c_int(0)
    check(library().fgw_mha_resolve_schedule(ctypes.byref(params), ctypes.byref(out)), "fgw_mha_resolve_schedule")
    return out.value


def workspace_size(params):
    out = ctypes.c_size_t(0)
    check(library().fgw_mha_workspace_size(ctypes.byref(params), ctypes.byref(out)), "fgw_mha_workspace_size")
    return out.value


def paged_fwd(params, workspace_ptr, workspace_bytes, stream_ptr):
    check(library().fgw_mha_paged_fwd(ctypes.byref(params), workspace_ptr, workspace_bytes, stream_ptr),
          "fgw_mha_paged_fwd")


def plan(params, workspace_ptr, workspace_bytes, stream_ptr):
    check(library().fgw_mha_plan(ctypes.byref(params), workspace_ptr, workspace_bytes, stream_ptr), "fgw_mha_plan")


def attend(params, workspace_ptr, workspace_bytes, stream_ptr):
    check(library().fgw_mha_attend(ctypes.byref(params), workspace_ptr, workspace_bytes, stream_ptr),
          "fgw_mha_attend")


def partial(params, workspace_ptr, workspace_bytes, stream_ptr):
    check(library().fgw_mha_partial(ctypes.byref(params), workspace_ptr, workspace_bytes, stream_ptr),
          "fgw_mha_partial")


def merge(params, workspace_ptr, workspace_bytes, stream_ptr):
    check(library().fgw_mha_merge(ctypes.byref(params), workspace_ptr, workspace_bytes, stream_ptr),
          "fgw_mha_merge")


def read_error(workspace_ptr, stream_ptr):
    """(device_status, site) recorded in the workspace header; synchronises the stream."""
    status = ctypes.c_int(0)
    site = ctypes.c_int(0)
    check(library().fgw_mha_read_error(workspace_ptr, stream_ptr, ctypes.byref(status), ctypes.byref(site)),
          "fgw_mha_read_error")
    return status.value, site.value


def selftest_wait(workspace_ptr, workspace_bytes, budget_ms, complete, stream_ptr):
    """Bounded-wait self-test (see include/fgw_mha.h); read the outcome with read_error."""
    check(library().fgw_mha_selftest_wait(workspace_ptr, workspace_bytes, budget_ms, 1 if complete else 0,
                                          stream_ptr), "fgw_mha_selftest_wait")


def paged_fwd_static_ws(params, stream_ptr):
    """Forward with the library's own static scratch array: allocates nothing (see include/fgw_mha.h)."""
    check(library().fgw_mha_paged_fwd_static_ws(ctypes.byref(params), stream_ptr), "fgw_mha_paged_fwd_static_ws")


def static_ws_read_error(stream_ptr):
    """(device_status, site) of the last static-workspace forward on the current device; synchronises."""
    status = ctypes.c_int(0)
    site = ctypes.c_int(0)
    check(library().fgw_mha_static_ws_read_error(stream_ptr, ctypes.byref(status), ctypes.byref(site)),
          "fgw_mha_static_ws_read_error")
    return status.value, site.value


def paged_cache_gather(params, stream_ptr):
    """``fgw_paged_cache_gather``: pack the cache rows the requests reach into ``params.dst``."""
    check(library().fgw_paged_cache_gather(ctypes.byref(params), ctypes.c_void_p(stream_ptr)),
          "fgw_paged_cache_gather")
