"""The host side of a call: the library's split choice (fgw_mha_choose_splits) against the Python restatement of
the B200 model, and the workspaces kept between eager launcher calls.

The serving path hands the host copy of its cache lengths to the library, which range-checks them and picks the
split count in one pass (no CUDA call, so this runs on CPU). It must pick exactly what
``general_split_cost_model.select_b200_splits`` picks from the same lengths, ties included.
"""
import numpy as np
import pytest

from fgw_b200 import _native
from fgw_b200.operators.mha import general_split_cost_model as general_model

MODEL = general_model.load_model(3)


def _native_model():
    return _native.SplitModel.from_model(MODEL)


def _python_choice(lengths, batch, sq, heads, dim, page, width, cores):
    stats = general_model.tile_stats(lengths.tolist())
    return general_model.select_b200_splits(batch, sq, heads, dim, page, width, *stats, model=MODEL, cores=cores)


def _random_case(rng):
    batch = int(rng.choice([1, 2, 3, 8, 16, 64, 65, 256, 300]))
    sq = int(rng.choice([1, 2, 3, 4, 8, 9, 16, 64, 128, 255, 256, 257, 512, 1000, 4096, 8192]))
    heads = int(rng.choice([1, 2, 4, 8, 16, 32, 40, 64]))
    dim = int(rng.choice(np.arange(16, 257, 16)))
    page = int(rng.choice([16, 32, 48, 64, 128]))
    width = int(rng.integers(1, 600))
    capacity = page * width
    kind = rng.integers(0, 5)
    if kind == 0:
        lengths = rng.integers(0, capacity + 1, size=batch)
    elif kind == 1:
        lengths = np.full(batch, capacity)
    elif kind == 2:
        lengths = np.exp(rng.uniform(0, np.log(capacity + 1), size=batch)).astype(np.int64)
    elif kind == 3:
        lengths = np.zeros(batch, dtype=np.int64)
    else:
        lengths = rng.integers(0, capacity + 1, size=batch)
        lengths[rng.integers(0, batch)] = capacity
    cores = int(rng.choice([148, 132, 28, 16, 200]))
    return np.minimum(lengths, capacity).astype(np.int32), batch, sq, heads, dim, page, width, cores


def test_native_choice_equals_the_python_model_on_random_shapes():
    rng = np.random.default_rng(2027)
    model = _native_model()
    seen = set()
    for _ in range(4000):
        lengths, batch, sq, heads, dim, page, width, cores = _random_case(rng)
        choice, status = _native.choose_splits(model, lengths, batch, sq, heads, dim, page, width, cores)
        assert status == _native.OK
        want = _python_choice(lengths, batch, sq, heads, dim, page, width, cores)
        assert choice.splits == want, (batch, sq, heads, dim, page, width, cores)
        assert choice.full_kv_cache == int(int(lengths.min()) == page * width)
        assert (choice.min_length, choice.max_length) == (int(lengths.min()), int(lengths.max()))
        seen.add(want)
    assert len(seen) >= 5  # the random shapes reach most candidates


@pytest.mark.parametrize("bad", [-1, 10 * 64 + 1])
def test_native_choice_rejects_lengths_outside_the_table(bad):
    lengths = np.array([5, bad, 7], dtype=np.int32)
    choice, status = _native.choose_splits(_native_model(), lengths, 3, 1, 8, 128, 64, 10, 148)
    assert status == _native.ERR_INVALID_ARGUMENT
    assert choice.splits == 0
    assert choice.min_length == min(5, bad) and choice.max_length == max(7, bad)


def test_native_choice_rejects_non_positive_extents():
    import ctypes
    lengths = np.array([5], dtype=np.int32)
    model = _native_model()
    fn = _native.library().fgw_mha_choose_splits
    for args in [(0, 1, 8, 128, 64, 10, 148), (1, 0, 8, 128, 64, 10, 148), (1, 1, 8, 128, 64, 0, 148),
                 (1, 1, 8, 128, 64, 10, 0)]:
        choice = _native.SplitChoice()
        status = fn(ctypes.byref(model), ctypes.c_void_p(lengths.ctypes.data), *args, ctypes.byref(choice))
        assert status == _native.ERR_INVALID_ARGUMENT


def test_binding_takes_only_the_batch_int32_lengths():
    model = _native_model()
    for bad in (np.array([5, 6], dtype=np.int64), np.array([5, 6, 7], dtype=np.int32),
                np.array([5, 0, 6, 0], dtype=np.int32)[::2]):
        with pytest.raises(ValueError):
            _native.choose_splits(model, bad, 2, 1, 8, 128, 64, 10, 148)


def test_kept_workspaces_stay_under_their_byte_cap_least_recently_used_first():
    # Eager launcher calls without a workspace reuse one kept per (launcher, device, stream); the process-wide pool
    # drops the least recently used workspace once the total would pass its cap.
    from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import _KeptWorkspaces

    class Buffer:
        def __init__(self, nbytes):
            self.nbytes = nbytes

        def numel(self):
            return self.nbytes

    pool = _KeptWorkspaces(100)
    with pool.lock:
        a = pool.get(("x", 0, 1), 40, lambda: Buffer(40))
        pool.get(("y", 0, 1), 40, lambda: Buffer(40))
        assert pool.get(("x", 0, 1), 40, lambda: Buffer(40)) is a  # a hit; x is now the most recent
        pool.get(("z", 0, 1), 40, lambda: Buffer(40))             # drops y
        assert set(pool.items) == {("x", 0, 1), ("z", 0, 1)} and pool.bytes == 80
        pool.get(("w", 0, 2), 90, lambda: Buffer(90))             # drops both
        assert set(pool.items) == {("w", 0, 2)} and pool.bytes == 90
