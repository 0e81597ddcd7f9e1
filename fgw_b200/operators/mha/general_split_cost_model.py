"""Latency model used to pick the split count of the general route, generalised over core count.

Restates ``operators/mha/general_split_cost_model.py:44-91`` of FGW:

* features over 32-token tiles with the head dimension padded to max(32, pow2(D)) / 64, waves over
  the core count, mean live tiles per request, merge work and partial traffic (:109-132); version 2
  adds the longest partition's excess over the mean (:128-131);
* ``predict_us`` = max(linear model, latency floor of single- or multi-split launches) (:135-139);
* ``select_model_splits`` keeps every split within tolerance of the best prediction and returns the
  smallest (version 1: 2 % relative; version 2: max(2 %, absolute margin)) (:142-156).

``cores=28`` with the reference coefficients (``models/reference_general_split_cost_model_v*.json``)
reproduces the reference bit for bit; the reference's constants 28 and 56 are ``cores`` and
``2 * cores``.

Version 3 is the B200 feature set (no reference counterpart), fitted on B200 split sweeps with the
reference fitter's loss (``fit_split_cost_model.py``) into ``models/b200_general_split_cost_model.json``. It
describes the B200 kernels instead of the Ascend ones: query rows per work item are the decode kernel's
(``decode_rows``) for up to 8 query rows and 256-row pairs above, KV tiles have 128 tokens, serial work
per program is counted separately for the two kernels, and with one split a tensor-path launch whose items
fill fewer than 2/3 of the programs runs the contiguous schedule (KV tiles spread evenly over the
programs). Its candidates are ``B200_SPLITS``: the reference's counts plus 64 and 128, since one request
and head over a long cache fills only ``splits`` of the 148 SMs (B1 H1 Q1 KV131072 measured 58 us at 32
splits, 33 us at 128). Explicit ``num_splits`` keeps the reference's accepted set.
"""
import functools
import json
import math
import pathlib

from fgw_b200.operators.mha.general_split_policy import SPLITS

B200_SPLITS = SPLITS + (64, 128)  # candidates of the version-3 (B200) model

MODEL_DIR = pathlib.Path(__file__).with_name("models")
FEATURE_NAMES = (
    "constant", "wave_tiles_times_padded_d", "wave_tiles", "waves_times_padded_d",
    "waves", "has_merge", "merge_rows_times_splits_times_padded_d",
    "partial_tasks_times_splits_times_padded_d",
)
FEATURE_NAMES_V2 = FEATURE_NAMES + ("longest_partition_excess_times_padded_d", "longest_partition_excess")
FEATURE_NAMES_V3 = (
    "constant", "decode_serial_tiles", "tensor_serial_tiles", "decode_waves", "tensor_waves", "has_merge",
    "splits", "merge_rows_times_splits", "longest_partition_excess", "contiguous_pieces_per_item",
)
DECODE_MAX_QUERIES = 8  # query rows per request at or below which the decode kernel runs
PAIR_ROWS = 256         # query rows per tensor-path work item (two 128-row tiles)
KV_TILE = 128
STREAM_MAX_PROGRAMS = 148  # programs of the contiguous schedule at most (kStreamMaxPrograms in the library)


def model_path(version=1):
    if type(version) is not int or version not in (1, 2, 3):
        raise ValueError("General model version must be 1, 2 or 3")
    if version == 3:
        return MODEL_DIR / "b200_general_split_cost_model.json"
    return MODEL_DIR / f"reference_general_split_cost_model_v{version}.json"


def feature_names(version=1):
    model_path(version)
    return {1: FEATURE_NAMES, 2: FEATURE_NAMES_V2, 3: FEATURE_NAMES_V3}[version]


def decode_rows(dim):
    """Query rows per decode work item (DecodeShape<D>::kRows of the decode kernel)."""
    chunks = dim // 8
    lanes = 8 if chunks >= 8 else (4 if chunks >= 4 else 2)
    per_lane = -(-chunks // lanes) * 8
    return 1 if per_lane >= 32 else (2 if per_lane >= 16 else 4)


def tile_stats(lengths):
    """(sum, max) over the requests of their caches' 128-token KV tiles: all the version-3 model reads of the
    lengths, so a serving loop whose lengths change every step computes these once per call."""
    if len(lengths) > 64:
        import numpy as np
        tiles = (np.asarray(lengths, dtype=np.int64) + (KV_TILE - 1)) // KV_TILE
        return int(tiles.sum()), int(tiles.max())
    tiles = [(n + KV_TILE - 1) // KV_TILE for n in lengths]
    return sum(tiles), max(tiles)


def _features_b200(batch, sq, heads, dim, lengths, splits, cores):
    return _features_b200_stats(batch, sq, heads, dim, *tile_stats(lengths), splits, cores)


def _features_b200_stats(batch, sq, heads, dim, tiles_sum, tiles_max, splits, cores):
    mean_tiles = tiles_sum / batch
    decode = sq <= DECODE_MAX_QUERIES
    rows = decode_rows(dim) if decode else PAIR_ROWS
    items = batch * heads * ((sq + rows - 1) // rows) * splits
    pieces = 0.0
    if not decode and splits == 1 and 3 * items < 2 * STREAM_MAX_PROGRAMS:
        programs = min(cores, STREAM_MAX_PROGRAMS)
        serial = math.ceil(items * max(mean_tiles, 1.0) / programs)
        waves = 1
        # an item cut into this many pieces is merged by one CTA (it reads every other piece's partial rows)
        pieces = min(programs / items, max(mean_tiles, 1.0))
    else:
        waves = (items + cores - 1) // cores
        serial = waves * math.ceil(mean_tiles / splits)
    longest = (tiles_max + splits - 1) // splits
    multi = 1 if splits > 1 else 0
    return [1.0,
            float(serial) if decode else 0.0,
            0.0 if decode else float(serial),
            float(waves) if decode else 0.0,
            0.0 if decode else float(waves),
            float(multi),
            float(splits),
            multi * batch * heads * sq * splits / cores,
            max(0.0, longest - mean_tiles / splits),
            pieces]


@functools.lru_cache(maxsize=8)
def load_model(version=1, path=None):
    model = json.loads(pathlib.Path(path or model_path(version)).read_text(encoding="utf-8"))
    names = feature_names(model["version"])
    if model["version"] != version or list(model["feature_names"]) != list(names) \
            or len(model["weights"]) != len(names):
        raise ValueError("General split model feature mismatch")
    if any(not math.isfinite(v) or v < 0 for v in model["weights"]):
        raise ValueError("General split model requires finite nonnegative weights")
    return model


def features(batch, sq, heads, dim, lengths, splits, version=1, cores=28):
    feature_names(version)
    if min(batch, sq, heads) <= 0 or not 16 <= dim <= 256 or dim % 16:
        raise ValueError("Positive B/Q/H and D16..256 step16 required")
    if len(lengths) != batch or any(type(n) is not int or n < 0 for n in lengths):
        raise ValueError("One nonnegative integer cache length per request required")
    if type(splits) is not int or splits not in (B200_SPLITS if version == 3 else SPLITS):
        raise ValueError("Unsupported split count")
    if version == 3:
        return _features_b200(batch, sq, heads, dim, lengths, splits, cores)
    padded_d = max(32, 1 << (dim - 1).bit_length()) / 64
    tasks = batch * heads * ((sq + 31) // 32)
    waves = (tasks * splits + cores - 1) // cores
    mean_tiles = sum((n + 31) // 32 for n in lengths) / batch
    merge_rows = min(8, 1 << (sq - 1).bit_length())
    merge_work = batch * heads * ((sq + merge_rows - 1) // merge_rows)
    multi = 1 if splits > 1 else 0
    values = [1.0,
              waves * mean_tiles / splits * padded_d,
              waves * mean_tiles / splits,
              waves * padded_d,
              float(waves),
              float(multi),
              multi * merge_work * splits * padded_d / (2 * cores),
              multi * tasks * splits * padded_d / cores]
    if version == 2:
        longest = (max((n + 31) // 32 for n in lengths) + splits - 1) // splits
        excess = max(0.0, longest - mean_tiles / splits)
        values += [excess * padded_d, excess]
    return values


def predict_us(batch, sq, heads, dim, lengths, splits, model=None, version=1, cores=None):
    model = load_model(version) if model is None else model
    cores = model.get("cores", 28) if cores is None else cores
    # The builtin sum (compensated on CPython >= 3.12), exactly as the reference accumulates.
    raw = sum(a * b for a, b in zip(features(batch, sq, heads, dim, lengths, splits, model["version"], cores),
                                    model["weights"]))
    floor = model["latency_floor_us"]["multi" if splits > 1 else "single"]
    return max(raw, floor)


def select_model_splits(batch, sq, heads, dim, page_size, width, lengths, model=None, version=1, cores=None):
    if page_size <= 0 or page_size % 16 or width <= 0:
        raise ValueError("Positive page16-multiple and table width required")
    if lengths is None:
        raise ValueError("Experimental cost model requires host-known cache_lengths")
    if len(lengths) != batch or any(n > page_size * width for n in lengths):
        raise ValueError("cache_lengths must match batch and page-table capacity")
    model = load_model(version) if model is None else model
    # KV tiles of table capacity: 32-token tiles of the reference's general kernel; 128 on B200 (version 3)
    tile = KV_TILE if model["version"] == 3 else 32
    capacity_tiles = (page_size * width + tile - 1) // tile
    costs = {}
    for s in (B200_SPLITS if model["version"] == 3 else SPLITS):
        if s <= capacity_tiles:
            costs[s] = predict_us(batch, sq, heads, dim, lengths, s, model, cores=cores)
    return pick_within_tolerance(costs, model)


def pick_within_tolerance(costs, model):
    """Smallest split count whose predicted latency is within the model's tolerance of the best prediction
    (version 1: 2 % relative; later versions: max(2 %, the absolute margin)); ``costs`` maps split -> us."""
    best = min(costs.values())
    tolerance = model["selection_tolerance"]
    if model["version"] == 1:
        limit = best * (1 + tolerance)
    else:
        limit = best + max(best * tolerance, model.get("absolute_selection_margin_us", 0.0))
    return min(s for s, value in costs.items() if value <= limit)


def select_b200_splits(batch, sq, heads, dim, page_size, width, tiles_sum, tiles_max, model=None, cores=None):
    """``select_model_splits`` of the version-3 (B200) model from ``tile_stats`` of the lengths instead of the
    lengths themselves (the same choice; the caller has checked the lengths against the table)."""
    model = load_model(3) if model is None else model
    if model["version"] != 3:
        raise ValueError("select_b200_splits takes the version-3 model")
    cores = model.get("cores", 28) if cores is None else cores
    capacity_tiles = (page_size * width + KV_TILE - 1) // KV_TILE
    floor = model["latency_floor_us"]
    costs = {}
    for s in B200_SPLITS:
        if s <= capacity_tiles:
            raw = sum(a * b for a, b in zip(_features_b200_stats(batch, sq, heads, dim, tiles_sum, tiles_max, s,
                                                                 cores), model["weights"]))
            costs[s] = max(raw, floor["multi" if s > 1 else "single"])
    return pick_within_tolerance(costs, model)
