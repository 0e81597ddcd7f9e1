"""Split selector of the restricted (BF16, D128, page%128) route, generalised over core count.

Restates ``operators/mha/split_cost_model.py`` of FGW: six features per candidate split count,
a non-negative linear score, argmin with ties going to the smaller split (:13-31), and the
promotion guard ``eligible_config`` (:34-44). With the reference coefficients
(``models/reference_split_cost_model.json``) and ``cores=28`` every selection is bit-identical
to the reference's; ``tests/test_split_models.py`` checks that against tables generated from the
reference itself. The B200 routes choose their split counts with the version-3 model of
``general_split_cost_model`` instead; this selector is kept for the reference's ``cost_model`` parity.
"""
import functools
import json
import pathlib

SPLITS = (1, 2, 4, 8, 16)
MODEL_DIR = pathlib.Path(__file__).with_name("models")
REFERENCE_MODEL = MODEL_DIR / "reference_split_cost_model.json"


@functools.lru_cache(maxsize=8)
def load_model(path=REFERENCE_MODEL):
    """{'weights': [...6 floats], 'cores': int, ...} from a JSON coefficient file."""
    model = json.loads(pathlib.Path(path).read_text(encoding="utf-8"))
    if len(model["weights"]) != 6 or any(w < 0 for w in model["weights"]):
        raise ValueError("split cost model needs six non-negative weights")
    return model


def _next_pow2(n):
    return 1 << (n - 1).bit_length()


def features(batch, sq, heads, kv_tiles, splits, cube_cores=28):
    """(wave_tiles, waves, extra_launch, partial_elements, merge_work*splits, multi*wave_tiles)."""
    query_tiles = (sq + 127) // 128
    tasks = batch * query_tiles * heads
    waves = (tasks * splits + cube_cores - 1) // cube_cores
    tiles_per_split = (kv_tiles + splits - 1) // splits
    merge_rows = min(8, _next_pow2(sq))
    merge_work = batch * heads * ((sq + merge_rows - 1) // merge_rows)
    multi = 1 if splits > 1 else 0
    return (waves * tiles_per_split, waves, multi, multi * tasks * splits, multi * merge_work * splits,
            multi * waves * tiles_per_split)


def score(weights, values):
    # The builtin sum (compensated on CPython >= 3.12), exactly as the reference accumulates.
    return sum(w * x for w, x in zip(weights, values))


def select_splits(batch, sq, heads, kv_tiles, *, weights=None, cores=None, model=None):
    """Split count in SPLITS minimising the model score; ties go to the smaller split."""
    if min(batch, sq, heads, kv_tiles) <= 0:
        raise ValueError("positive extents required")
    if model is None:
        model = load_model()
    weights = model["weights"] if weights is None else weights
    cores = model.get("cores", 28) if cores is None else cores
    scores = {}
    for s in SPLITS:
        if s <= kv_tiles:
            scores[s] = score(weights, features(batch, sq, heads, kv_tiles, s, cores))
    return min(scores, key=lambda s: (scores[s], s))


def eligible_config(batch, sq, heads, kv_tokens, *, dtype, dim, page_size, causal, pipeline_stages,
                    buffer_versions, kv_versions, q_resident, schedule_mode, full_kv_cache, cube_cores,
                    expected_cores=28):
    """Whether the automatic policy may use the cost model (split_cost_model.py:34-44).

    ``expected_cores`` is the core count the coefficients were fitted for (28 for the reference
    model, the SM count for the B200 refit).
    """
    return (full_kv_cache is True and cube_cores == expected_cores
            and str(dtype) in ("bfloat16", "torch.bfloat16") and dim == 128
            and page_size == 128 and not causal and pipeline_stages == 2
            and buffer_versions == 2 and kv_versions == 2 and q_resident
            and schedule_mode == "manual" and 1 <= batch <= 4 and 1 <= heads <= 16
            and batch * heads <= 32 and 1 <= sq <= 8192
            and 512 <= kv_tokens <= 32768 and kv_tokens % 128 == 0)


def legacy_splits(batch, sq, heads, width, page_size, block_q=128, block_kv=128):
    """The reference's fallback doubling rule for the restricted route (v7.py:91-96).

    Doubles while fewer than 16 splits, at least two KV tiles per split remain in table capacity,
    and query-tile tasks times splits stay below 128.
    """
    tasks = batch * ((sq + block_q - 1) // block_q) * heads
    splits = 1
    while splits < 16 and splits * 2 <= width * page_size // block_kv and tasks * splits < 128:
        splits *= 2
    return splits


def vector_fallback_splits(batch, sq, heads, width, page_size):
    """The reference's SIMT fallback rule (v2.py:21-29): 32- or 16-token tiles, tasks = B*Sq*H."""
    tile = 32 if page_size % 32 == 0 else 16
    tasks = batch * sq * heads
    capacity_tiles = width * page_size // tile
    splits = 1
    while splits < 16 and splits * 2 <= capacity_tiles and tasks * splits < 128:
        splits *= 2
    return splits
