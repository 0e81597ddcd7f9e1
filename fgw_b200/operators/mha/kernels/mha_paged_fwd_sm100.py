"""B200 (sm_100a) paged MHA forward behind FGW's ``operators/mha`` API.

Drop-in for ``operators.mha.current`` (FGW operators/mha/current.py:7, which re-exports
``mha_paged_decode_ascend_v7``) with the superset signature of
``mha_paged_decode_ascend_v7_experimental.py:858-897``:

* ``route`` reproduces the reference routing decision (v7_experimental.py:18-25) and is reported as
  ``launch.reference_route``; on B200 every route runs the same CUDA kernels, chosen by query length
  (``execution_path``: ``sm100_decode`` or ``sm100_tcgen05``);
* ``build_kernel`` validates like the reference (ValueError on the same conditions), selects the split
  count (explicit, the reference ``legacy`` rules, or the B200 cost models) and returns a launch callable
  carrying the reference's metadata attributes (v7.py:475-487, 500-513; cube_general.py:294-305);
* ``mha_paged_decode`` validates tensors like v7.py:529-544, reads the cache lengths once on the host
  (v7.py:548 does the same) to reject lengths outside table capacity and to feed the split model, and
  launches through the C ABI of ``libfgw_mha.so`` on the current CUDA stream.

Knobs of the Ascend pipeline (``pipeline_stages``, ``buffer_versions``, ``kv_versions``,
``q_resident``, ``schedule_mode``) are validated as in the reference and recorded on the launch
callable; the CUDA kernels size their own TMA rings, so they do not change the schedule.
``persistent_programs`` caps the persistent grid (default: the SM count; ``None`` uncapped).
"""
import collections
import functools
import threading

import numpy as np
import torch

from fgw_b200 import _native
from fgw_b200.operators.mha import general_split_cost_model as general_model
from fgw_b200.operators.mha import general_split_policy as general_policy
from fgw_b200.operators.mha import split_cost_model as v7_model

DEFAULT_PROGRAMS = "sm_count"
DECODE_MAX_QUERIES = 8  # query rows per request at or below which AUTO uses the decode kernel
BLOCK_Q_TENSOR = 128
BLOCK_KV = 128
# tcgen05 kernels of the tensor path (fgw_tensor_kernel): auto = pairs up to D128, single above
TENSOR_KERNELS = {"auto": _native.TENSOR_KERNEL_AUTO, "pairs": _native.TENSOR_KERNEL_PAIRS,
                  "single": _native.TENSOR_KERNEL_SINGLE, "halves": _native.TENSOR_KERNEL_HALVES}


def _decode_rows(dim):
    """Query rows per decode work item (DecodeShape<D>::kRows in fgw_decode.cu)."""
    chunks = dim // 8
    lanes = 8 if chunks >= 8 else (4 if chunks >= 4 else 2)
    per_lane = -(-chunks // lanes) * 8
    return 1 if per_lane >= 32 else (2 if per_lane >= 16 else 4)


def _probe_params(sq):
    p = _native.Params()
    p.q_len = sq
    p.path = _native.PATH_AUTO
    return p


def route(dtype, dim, page_size, sq=1, causal=False, cube_mode="stable"):
    """Reference routing decision (mha_paged_decode_ascend_v7_experimental.py:18-25)."""
    if cube_mode not in ("stable", "general"):
        raise ValueError("cube_mode must be stable or general")
    if cube_mode == "general":
        if (str(dtype) not in ("float16", "torch.float16", "bfloat16", "torch.bfloat16") or dim < 16 or dim > 256
                or dim % 16 or page_size <= 0 or page_size % 16):
            raise ValueError("General Cube supports FP16/BF16, D16..256 step16, page_size divisible by16")
        return "cube_general"
    restricted = (str(dtype) in ("bfloat16", "torch.bfloat16") and dim == 128 and (not causal or sq == 1)
                  and page_size > 0 and page_size % 128 == 0)
    return "cube_bf16_d128" if restricted else "fallback_v2"


@functools.lru_cache(maxsize=16)
def sm_count(device_index):
    return _native.device_sm_count(device_index)


def _device_index(device_index):
    if device_index is not None:
        return int(device_index)
    return torch.cuda.current_device()


def _dtype_code(dtype):
    return _native.DTYPE_BFLOAT16 if str(dtype) in ("bfloat16", "torch.bfloat16") else _native.DTYPE_FLOAT16


def _b200_model():
    return general_model.load_model(3)  # the B200 feature set fitted on B200 split sweeps


@functools.lru_cache(maxsize=1)
def _native_split_model():
    """The B200 model as the library's ``fgw_split_model`` (built once)."""
    return _native.SplitModel.from_model(_b200_model())


_route_cached = functools.lru_cache(maxsize=64)(route)

_KEPT_WORKSPACE_BYTES = 64 << 20  # workspaces up to this size are kept between eager calls
_KEPT_TOTAL_BYTES = 256 << 20     # all kept workspaces of the process together, least recently used dropped first


class _KeptWorkspaces:
    """Workspaces of eager launcher calls that pass none, kept per (launcher, device, stream) so that a serving loop
    saves an allocation per call. Calls on one stream run in order, so the next call on that stream may reuse its
    workspace (the plan launch re-initialises what the kernels read); a workspace is allocated on the stream it
    serves, so dropping one is ordered after the work that used it. One lock covers the lookup and the enqueue
    (ctypes releases the GIL during the call), so two threads never interleave their launches on one workspace."""

    def __init__(self, cap):
        self.cap = cap
        self.bytes = 0
        self.items = collections.OrderedDict()
        self.lock = threading.Lock()

    def get(self, key, nbytes, make):
        """The kept workspace for ``key`` (made by ``make()`` on a miss); the caller holds ``lock``."""
        ws = self.items.get(key)
        if ws is not None:
            self.items.move_to_end(key)
            return ws
        while self.items and self.bytes + nbytes > self.cap:
            _, old = self.items.popitem(last=False)
            self.bytes -= old.numel()
        ws = self.items[key] = make()
        self.bytes += ws.numel()
        return ws


_KEPT = _KeptWorkspaces(_KEPT_TOTAL_BYTES)


def _current_stream(device):
    """Raw handle of the current CUDA stream of device index ``device``."""
    return torch.cuda.current_stream(device).cuda_stream


if hasattr(torch._C, "_cuda_getCurrentRawStream"):
    def _current_stream(device):  # noqa: F811 -- the same handle without building a Stream object
        return torch._C._cuda_getCurrentRawStream(device)


def _host_lengths(lengths, batch, capacity):
    """Host cache lengths as a C-contiguous int32 array; values that int32 cannot hold are out of range."""
    host = np.asarray(lengths)
    if host.shape != (batch,):
        raise ValueError("metadata shape mismatch")
    if host.dtype != np.int32:
        if host.size and (int(host.min()) < 0 or int(host.max()) > capacity):
            raise ValueError("Cache lengths must be within table capacity")
        host = host.astype(np.int32)
    return np.ascontiguousarray(host)


def _select_auto_splits(batch, sq, heads, dim, width, page_size, lengths, cores, chosen=None):
    """B200 split choice from host-known lengths (or table capacity) with the fitted B200 model; ``chosen`` is
    that choice when the caller has already made it."""
    if chosen is not None:
        return chosen
    if lengths is None:
        lengths = (width * page_size,) * batch
    return general_model.select_model_splits(batch, sq, heads, dim, page_size, width, list(lengths),
                                             model=_b200_model(), cores=cores)


@functools.lru_cache(maxsize=128)
def build_kernel(batch, sq, heads, dim, pool_rows, width, page_size, causal, dtype, device_index=None,
                 pipeline_stages=2, buffer_versions=2, q_resident=True, kv_versions=None, dump_ir_dir=None,
                 schedule_mode="manual", num_splits=None, split_policy="auto", full_kv_cache=False,
                 persistent_programs=DEFAULT_PROGRAMS, cube_mode="stable", cache_lengths=None,
                 general_model_version=1, task_assignment=None, path="auto", tensor_kernel="auto",
                 _b200_splits=None, _auto_splits=None):
    """Validate a static shape, pick the split count and return a launch callable.

    ``_auto_splits`` is the B200 model's choice already made by the caller from the lengths' tile statistics
    (``mha_paged_decode`` does this, so launchers are cached per shape and split count, not per length list);
    it stands in for the model wherever the policy would run it.

    ``_b200_splits`` (B200-only, for measuring the split model's candidates) fixes the split count to one of
    ``general_split_cost_model.B200_SPLITS``, including the 64 and 128 that ``split_policy="auto"`` may pick but
    an explicit ``num_splits`` does not accept (the reference's set).
    """
    if str(dtype) not in ("float16", "torch.float16", "bfloat16", "torch.bfloat16"):
        raise ValueError("FP16 or BF16 required")
    if dim < 16 or dim > 256 or dim % 16:
        raise ValueError("D must be in [16, 256] and divisible by 16")
    if min(batch, sq, heads) <= 0:
        raise ValueError("Positive tensor extents required")
    if page_size <= 0 or pool_rows <= 0 or pool_rows % page_size or width <= 0:
        raise ValueError("positive page size, whole pool pages and positive table width required")
    if page_size % 16:
        raise ValueError("page_size must be a multiple of 16")
    if task_assignment not in (None, "strided", "contiguous", "tail"):
        raise ValueError("task_assignment must be None (route default), strided, contiguous or tail")
    if schedule_mode not in ("auto", "auto-offset", "manual", "nsa"):
        raise ValueError("schedule_mode must be auto, auto-offset, manual or nsa")
    if split_policy not in ("auto", "legacy", "cost_model"):
        raise ValueError("split_policy must be auto, legacy or cost_model")
    if path not in ("auto", "decode", "tensor"):
        raise ValueError("path must be auto, decode or tensor")
    if tensor_kernel not in TENSOR_KERNELS:
        raise ValueError("tensor_kernel must be one of " + ", ".join(TENSOR_KERNELS))
    selected_route = route(dtype, dim, page_size, sq, causal, cube_mode)
    if selected_route == "cube_general":
        if (pipeline_stages != 2 or buffer_versions != 2 or not q_resident or kv_versions is not None
                or dump_ir_dir is not None or schedule_mode != "manual"
                or persistent_programs not in (DEFAULT_PROGRAMS, 28)):
            raise ValueError("General Cube has its own untuned schedule; v7 tuning overrides are unsupported")
    else:
        if persistent_programs != DEFAULT_PROGRAMS and persistent_programs is not None and (
                type(persistent_programs) is not int or persistent_programs <= 0):
            raise ValueError("persistent_programs supports None (uncapped grid) or a positive program cap")
        effective_kv_versions = buffer_versions if kv_versions is None else kv_versions
        if effective_kv_versions not in (1, 2, 3):
            raise ValueError("K/V L1 versions must be 1, 2 or 3")
        if pipeline_stages not in (1, 2, 3) or buffer_versions not in (1, 2, 3):
            raise ValueError("Experimental pipeline stages and buffer versions must be 1, 2 or 3")
    if _b200_splits is not None:
        if num_splits is not None or type(_b200_splits) is not int or _b200_splits not in general_model.B200_SPLITS:
            raise ValueError("_b200_splits takes one of B200_SPLITS, and no num_splits")
        if _b200_splits > (width * page_size + general_model.KV_TILE - 1) // general_model.KV_TILE:
            raise ValueError("_b200_splits must not exceed the 128-token KV tiles in table capacity")
    dev = _device_index(device_index)
    cores = sm_count(dev)

    requested_policy = split_policy
    capacity_tokens = width * page_size
    if _b200_splits is not None:
        splits = _b200_splits
        policy_name = "explicit"
    elif selected_route == "cube_general":
        capacity_tiles = (capacity_tokens + 31) // 32
        tasks = batch * heads * ((sq + 31) // 32)
        if num_splits is None and split_policy == "cost_model":
            if cache_lengths is None and _auto_splits is None:
                raise ValueError("Experimental cost model requires host-known cache_lengths")
            splits = _select_auto_splits(batch, sq, heads, dim, width, page_size, cache_lengths, cores, _auto_splits)
            policy_name = "cost_model"
        elif num_splits is None and split_policy == "auto":
            # The reference's rule here fills the cores (fill_28); over 148 SMs that over-splits (the config-3
            # sweep measured it 1.2-2.4x slower than the best split), so "auto" takes the fitted B200 model,
            # over table capacity when the lengths are not known on the host.
            splits = _select_auto_splits(batch, sq, heads, dim, width, page_size, cache_lengths, cores, _auto_splits)
            policy_name = "cost_model"
        else:
            splits = general_policy.select_splits(tasks, capacity_tiles, num_splits, target_programs=cores)
            policy_name = "explicit" if num_splits is not None else "fill_sm"
    elif selected_route == "fallback_v2":
        if num_splits is not None or split_policy == "cost_model":
            raise ValueError("split override/policy requires the v7 Cube path")
        if split_policy == "legacy":
            splits = v7_model.vector_fallback_splits(batch, sq, heads, width, page_size)
            policy_name = "legacy"
        else:
            splits = _select_auto_splits(batch, sq, heads, dim, width, page_size, cache_lengths, cores, _auto_splits)
            policy_name = "cost_model"
    else:
        if num_splits is not None and (type(num_splits) is not int or num_splits not in (1, 2, 4, 8, 16)):
            raise ValueError("num_splits supports None (automatic) or 1/2/4/8/16")
        if num_splits is not None:
            if num_splits > capacity_tokens // BLOCK_KV:
                raise ValueError("num_splits must not exceed the number of KV tiles in table capacity")
            splits = num_splits
            policy_name = "explicit"
        elif split_policy == "legacy":
            splits = v7_model.legacy_splits(batch, sq, heads, width, page_size)
            policy_name = "legacy"
        else:
            splits = _select_auto_splits(batch, sq, heads, dim, width, page_size, cache_lengths, cores, _auto_splits)
            policy_name = "cost_model"

    kernel_path = {"auto": _native.PATH_AUTO, "decode": _native.PATH_DECODE, "tensor": _native.PATH_TENSOR}[path]
    if kernel_path == _native.PATH_AUTO:
        kernel_path = _native.resolve_path(_probe_params(sq))
    if kernel_path == _native.PATH_DECODE:
        rows = _decode_rows(dim)
        query_blocks = (sq + rows - 1) // rows
        block_q = rows
    else:
        query_blocks = (sq + BLOCK_Q_TENSOR - 1) // BLOCK_Q_TENSOR
        block_q = BLOCK_Q_TENSOR
    tasks = batch * heads * query_blocks
    compute_work = tasks * splits
    if persistent_programs is None:
        grid_cap = 0
        compute_grid = compute_work
        programs = None
    else:
        programs = cores if persistent_programs == DEFAULT_PROGRAMS else int(persistent_programs)
        grid_cap = programs
        compute_grid = min(compute_work, programs)

    params = _native.Params()
    params.pool_rows = pool_rows
    params.batch = batch
    params.q_len = sq
    params.heads = heads
    params.head_dim = dim
    params.table_width = width
    params.page_size = page_size
    params.dtype = _dtype_code(dtype)
    params.causal = 1 if causal else 0
    params.num_splits = splits
    params.grid_cap = grid_cap
    params.path = kernel_path
    params.schedule = {None: _native.SCHEDULE_AUTO, "strided": _native.SCHEDULE_STRIDED,
                       "contiguous": _native.SCHEDULE_CONTIGUOUS, "tail": _native.SCHEDULE_TAIL}[task_assignment]
    params.tensor_kernel = TENSOR_KERNELS[tensor_kernel]
    workspace_bytes = _native.workspace_size(params)
    # The library resolves the schedule (fgw_schedule in include/fgw_mha.h): the contiguous cut where it applies,
    # otherwise whole work items dealt out strided in longest-request-first order.
    schedule = _native.resolve_schedule(params)
    contiguous = schedule != _native.SCHEDULE_STRIDED

    def _bind(q, k, v, table, lengths, out):
        p = _native.Params.from_buffer_copy(params)
        p.q, p.k_cache, p.v_cache = q.data_ptr(), k.data_ptr(), v.data_ptr()
        p.block_table, p.cache_seqlens, p.out = table.data_ptr(), lengths.data_ptr(), out.data_ptr()
        return p

    def _workspace(device):
        return torch.empty(max(workspace_bytes, 256), dtype=torch.uint8, device=device)

    # Eager calls that pass no workspace reuse one kept for this launcher, device and stream (_KeptWorkspaces);
    # a call being captured into a CUDA graph gets a workspace of its own (the graph keeps it), and large
    # workspaces (many splits) are not kept.
    keep = workspace_bytes <= _KEPT_WORKSPACE_BYTES
    launcher_id = object()

    def launch(q, k, v, table, lengths, out=None, workspace=None):
        out = torch.empty_like(q) if out is None else out
        device = q.get_device()
        stream = _current_stream(device)
        if workspace is not None or not keep or torch.cuda.is_current_stream_capturing():
            ws = _workspace(q.device) if workspace is None else workspace
            _native.paged_fwd(_bind(q, k, v, table, lengths, out), ws.data_ptr(), ws.numel(), stream)
            return out
        with _KEPT.lock:
            ws = _KEPT.get((launcher_id, device, stream), max(workspace_bytes, 256), lambda: _workspace(q.device))
            _native.paged_fwd(_bind(q, k, v, table, lengths, out), ws.data_ptr(), ws.numel(), stream)
        return out

    def plan_kernel(q, k, v, table, lengths, workspace):
        _native.plan(_bind(q, k, v, table, lengths, q), workspace.data_ptr(), workspace.numel(),
                     torch.cuda.current_stream(q.device).cuda_stream)
        return workspace

    def attend_kernel(q, k, v, table, lengths, workspace, out):
        _native.attend(_bind(q, k, v, table, lengths, out), workspace.data_ptr(), workspace.numel(),
                       torch.cuda.current_stream(q.device).cuda_stream)
        return out

    def partial_kernel(q, k, v, table, lengths, workspace):
        out = torch.empty_like(q)
        _native.partial(_bind(q, k, v, table, lengths, out), workspace.data_ptr(), workspace.numel(),
                        torch.cuda.current_stream(q.device).cuda_stream)
        return workspace

    def merge_kernel(q, k, v, table, lengths, workspace, out=None):
        out = torch.empty_like(q) if out is None else out
        _native.merge(_bind(q, k, v, table, lengths, out), workspace.data_ptr(), workspace.numel(),
                      torch.cuda.current_stream(q.device).cuda_stream)
        return out

    launch.block_q = block_q
    launch.compute_grid = compute_grid
    launch.task_assignment = {_native.SCHEDULE_STRIDED: "strided", _native.SCHEDULE_CONTIGUOUS: "contiguous",
                              _native.SCHEDULE_TAIL: "tail"}[schedule]
    if contiguous:
        # one program per persistent CTA, at most the library's contiguous-schedule limit
        compute_grid = min(cores if grid_cap == 0 else min(grid_cap, cores), general_model.STREAM_MAX_PROGRAMS)
        launch.compute_grid = compute_grid
    launch.compute_work = compute_work
    launch.persistent_programs = programs
    launch.requested_split_policy = requested_policy
    launch.split_policy = policy_name
    launch.num_splits = splits
    launch.requested_num_splits = num_splits
    launch.query_tile_tasks = tasks
    launch.execution_mode = "direct_single_split" if splits == 1 else "split_and_merge"
    launch.execution_path = "sm100_decode" if kernel_path == _native.PATH_DECODE else "sm100_tcgen05"
    launch.tensor_kernel = tensor_kernel
    launch.reference_route = selected_route
    launch.workspace_bytes = workspace_bytes
    launch.schedule = {"schedule_mode": schedule_mode, "pipeline_stages": pipeline_stages,
                       "buffer_versions": buffer_versions, "kv_versions": kv_versions, "q_resident": q_resident}
    launch.general_model_version = general_model_version if policy_name == "cost_model" else None
    launch.prepare_q = lambda q: q  # Q is read in place through a 4-D TMA map; no head-major copy
    launch.new_workspace = _workspace
    launch.plan_kernel = plan_kernel
    launch.attend_kernel = attend_kernel
    launch.merge_only = merge_kernel
    launch.params = params
    if splits == 1:
        launch.direct_kernel = launch
    else:
        launch.partial_kernel = partial_kernel
        launch.merge_kernel = merge_kernel
    return launch


def _check_inputs(q, k_cache, v_cache, block_table, cache_seqlens):
    """Tensor preconditions with the reference's messages (v7.py:529-544)."""
    if q.ndim != 4 or k_cache.ndim != 3:
        raise ValueError("expected Q[B,Sq,H,D], K/V[N,H,D]")
    b, sq, h, d = q.shape
    if min(b, sq, h, d) <= 0 or block_table.ndim != 2:
        raise ValueError("positive Q extents and rank-2 table required")
    if k_cache.shape[1:] != (h, d) or v_cache.shape != k_cache.shape:
        raise ValueError("K/V shape mismatch")
    if block_table.shape[0] != b or block_table.shape[1] <= 0 or cache_seqlens.shape != (b,):
        raise ValueError("metadata shape mismatch")
    if q.dtype not in (torch.float16, torch.bfloat16) or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError("matching FP16/BF16 Q/K/V required")
    if block_table.dtype != torch.int32 or cache_seqlens.dtype != torch.int32:
        raise ValueError("int32 metadata required")
    dev = q.get_device() if q.is_cuda else -1
    if (dev < 0 or k_cache.get_device() != dev or v_cache.get_device() != dev or block_table.get_device() != dev
            or cache_seqlens.get_device() != dev or not q.is_contiguous() or not k_cache.is_contiguous()
            or not v_cache.is_contiguous() or not block_table.is_contiguous() or not cache_seqlens.is_contiguous()):
        raise ValueError("contiguous inputs on the same CUDA device required")
    return b, sq, h, d


def mha_paged_decode(q, k_cache, v_cache, block_table, cache_seqlens, page_size, is_causal=False, *,
                     pipeline_stages=2, buffer_versions=2, q_resident=True, kv_versions=None,
                     schedule_mode="manual", num_splits=None, split_policy="auto",
                     persistent_programs=DEFAULT_PROGRAMS, cube_mode="stable", general_model_version=1,
                     path="auto", cache_lengths=None, out=None, task_assignment=None, tensor_kernel="auto"):
    """Paged MHA forward: O[B,Sq,H,D] = softmax(Q K^T / sqrt(D)) V over each request's live pages.

    ``cache_lengths`` may pass the host copy of ``cache_seqlens`` (a sequence or a NumPy array) when the caller
    already has it; otherwise it is read once from the device, as the reference does. Launchers are cached per
    shape and split count, so a serving loop whose lengths change every call reuses them.
    """
    b, sq, h, d = _check_inputs(q, k_cache, v_cache, block_table, cache_seqlens)
    width = block_table.shape[1]
    capacity = width * page_size
    _route_cached(q.dtype, d, page_size, sq, bool(is_causal), cube_mode)  # the reference's route checks
    host = _host_lengths(cache_lengths if cache_lengths is not None else cache_seqlens.cpu().numpy(), b, capacity)
    # One pass over the host lengths in the library: their range check, whether every cache is full, and the
    # B200 model's split choice (it reads the lengths only through their KV-tile sum and maximum), so the
    # launcher below is cached per shape and split count and a new length list costs no rebuild.
    device = q.get_device()
    choice, status = _native.choose_splits(_native_split_model(), host, b, sq, h, d, page_size, width,
                                           sm_count(device))
    if status != _native.OK:
        raise ValueError("Cache lengths must be within table capacity")
    full_kv_cache = bool(choice.full_kv_cache)
    dtype_name = "float16" if q.dtype == torch.float16 else "bfloat16"
    auto = choice.splits if num_splits is None and split_policy != "legacy" else None
    kernel = build_kernel(b, sq, h, d, k_cache.shape[0], width, page_size, bool(is_causal), dtype_name,
                          device, pipeline_stages=pipeline_stages, buffer_versions=buffer_versions,
                          q_resident=q_resident, kv_versions=kv_versions, schedule_mode=schedule_mode,
                          num_splits=num_splits, split_policy=split_policy, full_kv_cache=full_kv_cache,
                          persistent_programs=persistent_programs, cube_mode=cube_mode, cache_lengths=None,
                          general_model_version=general_model_version, path=path, task_assignment=task_assignment,
                          tensor_kernel=tensor_kernel, _auto_splits=auto)
    return kernel(q, k_cache, v_cache, block_table, cache_seqlens, out=out)
