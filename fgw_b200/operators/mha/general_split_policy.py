"""Task-filling split policy of the general route ("fill28" in the reference).

Restates ``operators/mha/general_split_policy.py:6-21``: double the split count while
``tasks * splits < target_programs``, fewer than 32 splits, and two splits still fit in the
table's 32-token tile capacity. The reference fills 28 Cube cores; on B200 the target is the SM
count (148), passed as ``target_programs``.
"""
SPLITS = (1, 2, 4, 8, 16, 32)


def select_splits(tasks, capacity_tiles, num_splits=None, target_programs=28):
    if min(tasks, capacity_tiles, target_programs) <= 0:
        raise ValueError("Positive tasks, capacity tiles and target programs required")
    if num_splits is not None:
        if type(num_splits) is not int or num_splits not in SPLITS:
            raise ValueError("General Cube num_splits supports None or 1/2/4/8/16/32")
        if num_splits > capacity_tiles:
            raise ValueError("num_splits must not exceed KV tiles in page-table capacity")
        return num_splits
    splits = 1
    while splits < SPLITS[-1] and tasks * splits < target_programs and splits * 2 <= capacity_tiles:
        splits *= 2
    return splits
