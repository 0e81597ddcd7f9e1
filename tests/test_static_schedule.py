"""Host static schedules against the known answers of FGW's schedule tests (tests/mha/test_static_schedule.py).

The expected plan shapes below (partial counts, merge counts, loads, task counts) are the reference test's
assertions; the attention check restates its independent CPU oracle for split states.
"""
import math
import random
from collections import Counter

import pytest

from fgw_b200.operators.mha.static_schedule import (choose_plan, choose_stream_plan, make_block_merge_tasks,
                                                     make_merge_tasks, make_plan, make_q_plan, make_stream_plan,
                                                     make_tail_plan, validate_plan)

# the reference benchmark grid (benchmarks/mha/summarize_clean_grid.py:7-8)
QS = (64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768)
KVS = (512, 1024, 2048, 4096, 8192, 16384, 24576, 32768)


def test_whole_q_assignment_and_cost_selection():
    for q in (1, 17, 129, 3712, 32768):
        plan = make_q_plan(q, 512)
        assert not plan.merges and plan.partial_count == 0
        assert [tile for program in plan.programs for tile, *_ in program] == list(range((q + 127) // 128))
        assert all(first == 0 and count == 4 and slot == -1 for program in plan.programs
                   for _, first, count, slot in program)
    assert not choose_plan(128, 512).merges
    assert choose_plan(8192, 32768).merges
    assert len(choose_plan(8192, 32768).programs) == 28


def test_target_shapes_and_balanced_no_merge():
    plan = make_plan(8192, 32768)
    assert (plan.partial_count, len(plan.merges)) == (54, 27)
    assert (plan.describe()["min_kv_blocks"], plan.describe()["max_kv_blocks"]) == (585, 586)
    for q in (3584, 7168, 17920, 28672):
        plan = make_plan(q, 32768)
        assert (plan.partial_count, len(plan.merges)) == (0, 0)
        assert plan.describe()["min_kv_blocks"] == plan.describe()["max_kv_blocks"]


def test_tail_wave_coverage_and_fragment_count():
    for kv in (4096, 8192):
        plan = make_tail_plan(32768, kv)
        validate_plan(plan)
        assert (len(plan.merges), plan.partial_count) == (4, 28)
        assert {tile for tile, _, _ in plan.merges} == set(range(252, 256))
        assert plan.describe()["direct_q_tiles"] == 252
        assert plan.describe()["max_kv_blocks"] - plan.describe()["min_kv_blocks"] <= 1
    for q in (1, 129, 3584, 3712, 4096, 8192, 32768):
        for kv in (128, 256, 512, 4096, 8192):
            for pieces in (None, 2, 4, 7):
                validate_plan(make_tail_plan(q, kv, pieces=pieces))


def test_coverage_and_unique_ownership():
    for q in (1, 17, 128, 129, 257):
        for kv in (128, 256, 512, 1024):
            for cores in (1, 2, 7, 28):
                plan = make_plan(q, kv, cores)
                seen = Counter((tile, k) for program in plan.programs for tile, first, count, _ in program
                               for k in range(first, first + count))
                assert set(seen) == {(t, k) for t in range((q + 127) // 128) for k in range(kv // 128)}
                assert all(n == 1 for n in seen.values())
                validate_plan(plan)


@pytest.mark.parametrize("q", (*QS, 17, 129, 3712))
def test_selected_grid_coverage(q):
    for kv in KVS:
        plan = choose_plan(q, kv)
        validate_plan(plan)
        assert len(plan.programs) <= 28


def test_stream_policy_coverage_and_parallelism():
    for q in (*QS, 1, 17, 129, 3712):
        for kv in KVS:
            validate_plan(choose_stream_plan(q, kv))
            for cores in (1, 2, 7, 27, 28):
                validate_plan(make_stream_plan(q, kv, cores))
    assert len(choose_stream_plan(64, 32768).programs) > 1
    assert not choose_stream_plan(16384, 1024).merges
    assert not choose_stream_plan(128, 512).merges


def test_weighted_merge_exact_row_ownership():
    for q in (*QS, 1, 129, 3712):
        for kv in KVS:
            plan = choose_stream_plan(q, kv)
            tasks = make_merge_tasks(plan)
            assert len(tasks) <= 56
            expected = {(tile, r) for tile, _, _ in plan.merges for r in range(min(128, q - tile * 128))}
            seen = Counter((tile, r) for tile, _, _, begin, rows in tasks for r in range(begin, begin + rows))
            assert set(seen) == expected and all(n == 1 for n in seen.values())
            groups = {tile: (first, count) for tile, first, count in plan.merges}
            for tile, first, count, begin, rows in tasks:
                assert groups[tile] == (first, count) and rows > 0 and begin + rows <= min(128, q - tile * 128)
    tasks = make_merge_tasks(make_tail_plan(32768, 4096, pieces=7))
    assert len(tasks) == 52
    assert max(task[4] for task in tasks) == 10


def test_grouped_dma_chunk_ownership():
    for q in (*QS, 129, 3712):
        for kv in KVS:
            plan = choose_stream_plan(q, kv)
            expected = {(t, r) for t, _, _ in plan.merges for r in range(min(128, q - t * 128))}
            for budget in (28, 56):
                workers = make_block_merge_tasks(plan, budget)
                seen = Counter((t, r) for worker in workers for t, _, _, begin, rows in worker
                               for r in range(begin, begin + rows))
                assert set(seen) == expected and all(n == 1 for n in seen.values())
                assert len(workers) <= budget and all(workers)
                assert all(begin % 8 == 0 and 0 < rows <= 8 for worker in workers for *_, begin, rows in worker)


def test_device_cut_arithmetic():
    # The device's contiguous schedule cuts units the way make_plan does (program p starts at
    # p * (T // G) + min(p, T % G)).
    for total, programs in ((4096, 148), (16, 148), (148, 148), (27, 7)):
        starts = [p * (total // programs) + min(p, total % programs) for p in range(programs + 1)]
        loads = [b - a for a, b in zip(starts, starts[1:])]
        assert starts[-1] == total and max(loads) - min(loads) <= 1
    plan = make_plan(4096 * 128, 128, 148)
    starts = [p * (4096 // 148) + min(p, 4096 % 148) for p in range(149)]
    assert [sum(seg[2] for seg in program) for program in plan.programs] == \
        [b - a for a, b in zip(starts, starts[1:])]


@pytest.mark.parametrize("maker", [lambda: make_plan(257, 512, 2), lambda: make_tail_plan(257, 512, 2),
                                   lambda: make_stream_plan(257, 512, 2)])
def test_split_state_merge_matches_dense_attention(maker):
    # Three Q tiles on two cores: a whole tile and a piece in each, only the middle tile merges.
    plan = maker()
    assert len(plan.merges) == 1
    for weighted in (False, True, "grouped"):
        _check_attention(plan, weighted)


def _check_attention(plan, weighted):
    qlen, kv = plan.q, plan.kv
    rng = random.Random(7)
    q = [[rng.uniform(-1, 1) for _ in range(2)] for _ in range(qlen)]
    k = [[rng.uniform(-1, 1) for _ in range(2)] for _ in range(kv)]
    v = [[rng.uniform(-1, 1) for _ in range(2)] for _ in range(kv)]

    def attention(query, first, count):
        scores = [sum(a * b for a, b in zip(query, key)) / math.sqrt(2) for key in k[first:first + count]]
        top = max(scores)
        weights = [math.exp(x - top) for x in scores]
        total = sum(weights)
        return [sum(w * value[d] for w, value in zip(weights, v[first:first + count])) / total
                for d in range(2)], top + math.log(total)

    outputs, partials = {}, {}
    for program in plan.programs:
        for tile, first, count, slot in program:
            values = [attention(qi, first * 128, count * 128) for qi in q[tile * 128:min((tile + 1) * 128, qlen)]]
            if slot < 0:
                for row, (value, _) in enumerate(values):
                    outputs[tile * 128 + row] = value
            else:
                partials[slot] = values
    if weighted == "grouped":
        tasks = tuple(task for worker in make_block_merge_tasks(plan) for task in worker)
    elif weighted:
        tasks = make_merge_tasks(plan)
    else:
        tasks = tuple((tile, first, count, 0, min(128, qlen - tile * 128)) for tile, first, count in plan.merges)
    for tile, first, count, begin, rows in tasks:
        for row in range(begin, begin + rows):
            fragments = [partials[s][row] for s in range(first, first + count)]
            top = max(lse for _, lse in fragments)
            weights = [math.exp(lse - top) for _, lse in fragments]
            outputs[tile * 128 + row] = [sum(w * value[d] for w, (value, _) in zip(weights, fragments))
                                         / sum(weights) for d in range(2)]
    for row in range(qlen):
        expected, _ = attention(q[row], 0, kv)
        for got, ref in zip(outputs[row], expected):
            assert got == pytest.approx(ref, abs=1e-12)


# --- exact parity with the reference's plans (tests/golden/make_schedule_golden.py) -----------------------
def _golden():
    import json
    import pathlib
    return json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "static_schedule.json").read_text())


def _digest(value):
    import hashlib
    import json
    return hashlib.sha256(json.dumps(value, separators=(",", ":")).encode()).hexdigest()[:16]


def _record(plan):
    return _digest({"programs": [[list(s) for s in program] for program in plan.programs],
                    "merges": [list(m) for m in plan.merges], "partial_count": plan.partial_count,
                    "strategy": plan.strategy})


def test_plans_identical_to_reference_over_grid():
    golden = _golden()
    makers = {"make_plan": make_plan, "make_q_plan": make_q_plan, "make_stream_plan": make_stream_plan}
    for name, fn in makers.items():
        for key, expected in golden[name].items():
            q, kv, cores = map(int, key.split(","))
            assert _record(fn(q, kv, cores)) == expected, (name, key)
    for key, expected in golden["make_tail_plan"].items():
        q, kv, cores, pieces = key.split(",")
        plan = make_tail_plan(int(q), int(kv), int(cores), None if pieces == "None" else int(pieces))
        assert _record(plan) == expected, ("make_tail_plan", key)


def test_selection_and_merge_tasks_identical_to_reference():
    golden = _golden()
    for key, expected in golden["choose_plan"].items():
        q, kv = map(int, key.split(","))
        assert _record(choose_plan(q, kv)) == expected, key
    for key, expected in golden["choose_stream_plan"].items():
        q, kv = map(int, key.split(","))
        plan = choose_stream_plan(q, kv)
        assert _record(plan) == expected, key
        assert _digest([list(t) for t in make_merge_tasks(plan)]) == golden["make_merge_tasks"][key], key
        assert (_digest([[list(t) for t in w] for w in make_block_merge_tasks(plan)])
                == golden["make_block_merge_tasks"][key]), key


def test_b200_sized_plans_keep_every_invariant():
    # The planner takes the B200 SM count (the reference stops at its 28 Ascend cores): every plan kind at
    # 148 programs passes validate_plan (each (Q tile, KV block) exactly once, balanced loads within one block,
    # consistent slots and merges).
    for q in (128, 1000, 4096, 8192, 32768):
        for kv in (512, 2048, 8192, 32768):
            for make in (make_plan, make_q_plan, make_stream_plan, make_tail_plan):
                plan = make(q, kv, 148)
                validate_plan(plan)
                assert len(plan.programs) <= 148
    plan = make_plan(8192, 32768, 148)
    loads = [sum(seg[2] for seg in program) for program in plan.programs]
    assert len(loads) == 148 and max(loads) - min(loads) <= 1 and sum(loads) == 64 * 256
    # the search over program counts widens with max_cores; the reference's default stays 1..28
    assert len(choose_plan(8192, 32768).programs) == 28
    assert len(choose_plan(8192, 32768, max_cores=148).programs) > 28
    validate_plan(choose_stream_plan(4096, 2048, max_cores=148))
    with pytest.raises(ValueError):
        make_plan(128, 512, 0)
