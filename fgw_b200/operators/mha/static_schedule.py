"""Host-side static KV-block schedules for one (request, head) with 128x128 dense tiles.

Restates FGW's pure-host planner (operators/mha/static_schedule.py) with the same public API and the same
plans, so callers and tests written against it run unchanged:

* ``Plan``: per program a tuple of segments ``(q_tile, first_kv_block, kv_blocks, slot)``; ``slot == -1`` is
  a whole Q tile written directly, otherwise the partial slot the segment writes; ``merges`` lists
  ``(q_tile, first_slot, slot_count)`` for the Q tiles computed in pieces (static_schedule.py:7-45).
* ``make_plan``: every (Q tile, KV block) unit laid end to end and cut into equal contiguous ranges
  (loads differ by at most one block; static_schedule.py:48-80).
* ``make_q_plan``: whole consecutive Q tiles only (static_schedule.py:153-167).
* ``make_tail_plan``: whole Q tiles in the full waves, only the final wave's tiles split into pieces
  (static_schedule.py:118-150).
* ``make_stream_plan``: whole-Q-first greedy assignment against the remaining work per core with a
  half-block tolerance (static_schedule.py:194-247).
* ``estimate_cost`` / ``choose_plan`` / ``choose_stream_plan``: the reference's fixed stage-cost estimate
  and its selection rules (static_schedule.py:170-262).
* ``make_merge_tasks`` / ``make_block_merge_tasks``: merge work split over vector workers by rows x pieces
  and as fixed 8-row chunks (static_schedule.py:265-310).

The device counterpart on B200 is the contiguous schedule of the two-tile kernel (fgw_schedule in
include/fgw_mha.h): the same balanced cut of ``make_plan`` over (query-tile pair, KV tile) units of every
request and head, planned on the GPU from the device-resident lengths, with the pieces merged in the same
launch. ``cores`` defaults to the reference's 28 so its plans (and tests) reproduce; any program count up to
``MAX_CORES`` is accepted (the reference stops at its 28 Ascend cores), so ``make_plan(q, kv, 148)`` is a plan
for one B200. ``choose_plan`` / ``choose_stream_plan`` search 1..``max_cores`` programs (default 28, the
reference's search; pass the SM count for B200).
"""
from dataclasses import dataclass
from functools import lru_cache

BLOCK = 128  # rows of a Q tile and of a KV block
REFERENCE_CORES = 28
MAX_CORES = 4096  # programs a plan may have (one B200 has 148 SMs)


@dataclass(frozen=True)
class Plan:
    q: int
    kv: int
    programs: tuple
    merges: tuple
    partial_count: int
    strategy: str = "balanced"

    @property
    def max_segments(self):
        return max(len(program) for program in self.programs)

    @property
    def max_parts(self):
        return max((count for _, _, count in self.merges), default=0)

    def describe(self):
        loads = [sum(seg[2] for seg in program) for program in self.programs]
        q_tiles = _ceil(self.q, BLOCK)
        return dict(strategy=self.strategy, Q=self.q, KV=self.kv, programs=len(loads), q_tiles=q_tiles,
                    min_kv_blocks=min(loads), max_kv_blocks=max(loads),
                    segments=sum(len(program) for program in self.programs), max_segments=self.max_segments,
                    partial_count=self.partial_count, merge_q_tiles=len(self.merges),
                    direct_q_tiles=q_tiles - len(self.merges), max_parts=self.max_parts,
                    partial_bytes=self.partial_count * BLOCK * BLOCK * 4, lse_bytes=self.partial_count * BLOCK * 4)


def _ceil(a, b):
    return -(-a // b)


def _check_shape(q, kv, cores):
    if type(q) is not int or type(kv) is not int or q <= 0 or kv <= 0 or kv % BLOCK:
        raise ValueError("positive integer Q and positive 128-aligned KV required")
    if type(cores) is not int or not 1 <= cores <= MAX_CORES:
        raise ValueError(f"cores must be 1..{MAX_CORES}")
    tiles, blocks = _ceil(q, BLOCK), kv // BLOCK
    if tiles * blocks > 2**31 - 1:
        raise ValueError("int32 scheduling range exceeded")
    return tiles, blocks


def _assign_slots(programs):
    """Give every segment of a Q tile held by more than one program a partial slot, tile by tile."""
    holders = {}
    for pid, program in enumerate(programs):
        for index, segment in enumerate(program):
            holders.setdefault(segment[0], []).append((pid, index))
    merges, slot = [], 0
    for tile in sorted(holders):
        owners = holders[tile]
        if len(owners) < 2:
            continue
        merges.append((tile, slot, len(owners)))
        for pid, index in owners:
            programs[pid][index][3] = slot
            slot += 1
    return merges, slot


def _freeze(programs):
    return tuple(tuple(tuple(segment) for segment in program) for program in programs)


@lru_cache(maxsize=128)
def make_plan(q, kv, cores=REFERENCE_CORES):
    tiles, blocks = _check_shape(q, kv, cores)
    total = tiles * blocks
    cores = min(cores, total)
    base, extra = divmod(total, cores)
    programs = []
    for pid in range(cores):
        unit = pid * base + min(pid, extra)
        end = unit + base + (1 if pid < extra else 0)
        program = []
        while unit < end:
            tile, first = divmod(unit, blocks)
            take = min(end, (tile + 1) * blocks) - unit
            program.append([tile, first, take, -1])
            unit += take
        programs.append(program)
    merges, slots = _assign_slots(programs)
    plan = Plan(q, kv, _freeze(programs), tuple(merges), slots)
    validate_plan(plan)
    return plan


def validate_plan(plan):
    """Every (Q tile, KV block) exactly once; slots, merges and loads consistent (raises AssertionError)."""
    blocks, tiles = plan.kv // BLOCK, _ceil(plan.q, BLOCK)
    spans, direct, pieces, loads, slots = {}, set(), {}, [], []
    for program in plan.programs:
        assert program, "empty program"
        loads.append(sum(segment[2] for segment in program))
        for tile, first, count, slot in program:
            assert 0 <= tile < tiles and 0 <= first < blocks and 0 < count <= blocks - first
            spans.setdefault(tile, []).append((first, first + count))
            if slot < 0:
                assert first == 0 and count == blocks and tile not in direct
                direct.add(tile)
            else:
                slots.append(slot)
                pieces.setdefault(tile, []).append(slot)
    assert set(spans) == set(range(tiles))
    for ranges in spans.values():
        cursor = 0
        for first, end in sorted(ranges):
            assert first == cursor
            cursor = end
        assert cursor == blocks
    spread = max(loads) - min(loads)
    assert spread <= (1 if plan.strategy == "balanced" else blocks)
    assert sorted(slots) == list(range(plan.partial_count))
    assert not (set(pieces) & direct) and len(pieces) + len(direct) == tiles
    assert len(plan.merges) <= len(plan.programs) - 1
    merged = [tile for tile, _, _ in plan.merges]
    assert len(set(merged)) == len(merged) and set(merged) == set(pieces)
    for tile, first, count in plan.merges:
        assert count >= 2 and sorted(pieces[tile]) == list(range(first, first + count))
    return True


@lru_cache(maxsize=128)
def make_q_plan(q, kv, cores=REFERENCE_CORES):
    """Whole consecutive Q tiles per program; no partial KV states."""
    make_plan(q, kv, cores)
    tiles, blocks = _ceil(q, BLOCK), kv // BLOCK
    cores = min(cores, tiles)
    base, extra = divmod(tiles, cores)
    programs = []
    for pid in range(cores):
        first = pid * base + min(pid, extra)
        count = base + (1 if pid < extra else 0)
        programs.append(tuple((tile, 0, blocks, -1) for tile in range(first, first + count)))
    plan = Plan(q, kv, tuple(programs), (), 0, "q_only")
    validate_plan(plan)
    return plan


@lru_cache(maxsize=128)
def make_tail_plan(q, kv, cores=REFERENCE_CORES, pieces=None):
    """Whole Q tiles in the full waves; only the final wave's Q tiles are split into KV pieces."""
    make_plan(q, kv, cores)
    if pieces is not None and (type(pieces) is not int or pieces < 2):
        raise ValueError("pieces must be None or an integer >=2")
    tiles, blocks = _ceil(q, BLOCK), kv // BLOCK
    waves, tail = divmod(tiles, cores)
    if not waves or not tail or blocks < 2:
        return make_q_plan(q, kv, cores)
    programs = [[(tile, 0, blocks, -1) for tile in range(pid * waves, (pid + 1) * waves)] for pid in range(cores)]
    merges, slot, turn = [], 0, 0
    for extra in range(tail):
        tile = waves * cores + extra
        parts = min(blocks, pieces or (cores // tail + (1 if extra < cores % tail else 0)))
        if parts == 1:
            programs[turn % cores].append((tile, 0, blocks, -1))
            turn += 1
            continue
        merges.append((tile, slot, parts))
        base, rem = divmod(blocks, parts)
        for part in range(parts):
            first = part * base + min(part, rem)
            programs[turn % cores].append((tile, first, base + (1 if part < rem else 0), slot))
            turn += 1
            slot += 1
    if not merges:
        return make_q_plan(q, kv, cores)
    plan = Plan(q, kv, tuple(tuple(program) for program in programs), tuple(merges), slot, "tail")
    validate_plan(plan)
    return plan


# The reference's fixed per-stage estimates in microseconds (not fitted): KV block, segment start, merge
# launch, partial write and merged Q tile (static_schedule.py:170-173).
COST_MODEL = dict(block_us=0.72, segment_us=2.0, merge_launch_us=12.0, partial_us=0.20, merge_tile_us=0.15)


def estimate_cost(plan):
    """Busiest program's blocks and segments plus the merge launch (when there is one)."""
    c = COST_MODEL
    local = max(sum(seg[2] for seg in program) * c["block_us"] + len(program) * c["segment_us"]
                for program in plan.programs)
    merge = 0.0
    if plan.merges:
        merge = c["merge_launch_us"] + plan.partial_count * c["partial_us"] + len(plan.merges) * c["merge_tile_us"]
    return dict(local_us=local, merge_us=merge, total_us=local + merge)


@lru_cache(maxsize=128)
def choose_plan(q, kv, max_cores=REFERENCE_CORES):
    """Cheapest of the whole-Q plan and the balanced plans on 1..max_cores programs (ties: fewer partials, more
    programs)."""
    candidates = [make_q_plan(q, kv, max_cores)] + [make_plan(q, kv, cores) for cores in range(1, max_cores + 1)]
    return min(candidates, key=lambda p: (estimate_cost(p)["total_us"], p.partial_count, -len(p.programs)))


@lru_cache(maxsize=128)
def make_stream_plan(q, kv, cores=REFERENCE_CORES):
    """Whole-Q-first assignment: each program takes units up to the remaining work per remaining program,
    finishing the current Q tile when that stays within half a block of the target."""
    make_plan(q, kv, cores)
    tiles, blocks = _ceil(q, BLOCK), kv // BLOCK
    total = tiles * blocks
    cores = min(cores, total)
    programs, cursor = [], 0
    for pid in range(cores):
        if cursor == total:
            break
        target = (total - cursor) / (cores - pid)
        taken, program = 0, []
        while cursor < total:
            tile, first = divmod(cursor, blocks)
            left = blocks - first
            if taken + left <= target + 0.5 or pid == cores - 1:
                take = left
            else:
                take = min(left, max(0, int(target + 0.5 - taken)))
                if not program:
                    take = max(1, take)
                if take == 0:
                    break
            program.append([tile, first, take, -1])
            cursor += take
            taken += take
            if taken >= target - 0.5:
                break
        programs.append(program)
    assert cursor == total
    merges, slots = _assign_slots(programs)
    if not merges:
        return make_q_plan(q, kv, len(programs))
    plan = Plan(q, kv, _freeze(programs), tuple(merges), slots, "stream")
    validate_plan(plan)
    return plan


@lru_cache(maxsize=128)
def choose_stream_plan(q, kv, max_cores=REFERENCE_CORES):
    """Best stream or tail plan over 1..max_cores programs, taken only if it beats whole-Q tiles by more than
    one block's cost."""
    direct = make_q_plan(q, kv, max_cores)
    candidates = [make_stream_plan(q, kv, cores) for cores in range(1, max_cores + 1)]
    candidates += [make_tail_plan(q, kv, cores) for cores in range(1, max_cores + 1)]
    split = min(candidates, key=lambda p: (estimate_cost(p)["total_us"], p.partial_count))
    if estimate_cost(direct)["total_us"] - estimate_cost(split)["total_us"] > COST_MODEL["block_us"]:
        return split
    return direct


@lru_cache(maxsize=128)
def make_merge_tasks(plan, vectors=56):
    """Merge records ``(q_tile, first_slot, pieces, first_row, rows)``: each merged Q tile's valid rows cut into
    row ranges in proportion to rows x pieces over at most ``vectors`` workers."""
    if type(vectors) is not int or vectors <= 0 or vectors < len(plan.merges):
        raise ValueError("positive vector budget, at least one per merge group required")
    if not plan.merges:
        return ()
    groups = [(tile, first, count, min(BLOCK, plan.q - tile * BLOCK)) for tile, first, count in plan.merges]
    budget = min(vectors, sum(rows for *_, rows in groups))
    average = _ceil(sum(rows * count for _, _, count, rows in groups), budget)
    spare = budget - len(groups)
    tasks = []
    for tile, first, count, rows in groups:
        parts = min(rows, spare + 1, max(1, rows * count // average))
        stride = _ceil(rows, parts)
        parts = _ceil(rows, stride)
        spare -= parts - 1
        tasks.extend((tile, first, count, begin, min(stride, rows - begin)) for begin in range(0, rows, stride))
    assert len(tasks) <= vectors
    return tuple(tasks)


@lru_cache(maxsize=128)
def make_block_merge_tasks(plan, vectors=56, rows=8):
    """8-row merge chunks dealt to the least-loaded of ``vectors`` workers, heaviest (pieces x rows) first."""
    if type(vectors) is not int or vectors <= 0 or rows != 8:
        raise ValueError("positive vector budget and rows=8 required")
    chunks = [(tile, first, count, begin, min(rows, plan.q - tile * BLOCK - begin))
              for tile, first, count in plan.merges
              for begin in range(0, min(BLOCK, plan.q - tile * BLOCK), rows)]
    if not chunks:
        return ()
    workers = [[] for _ in range(min(vectors, len(chunks)))]
    loads = [0] * len(workers)
    for chunk in sorted(chunks, key=lambda c: (-c[2] * c[4], c[0], c[3])):
        w = min(range(len(workers)), key=lambda i: (loads[i], len(workers[i]), i))
        workers[w].append(chunk)
        loads[w] += chunk[2] * chunk[4]
    return tuple(tuple(worker) for worker in workers)
