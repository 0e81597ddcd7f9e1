"""Generate ``static_schedule.json``: FGW's host static schedules over a shape grid, for parity tests.

Run once, pointing ``--reference`` at a checkout of FGW:

    python tests/golden/make_schedule_golden.py --reference <FGW checkout>

``operators/mha/static_schedule.py`` of the reference is stdlib-only and is imported directly. Every plan
(programs of segments ``[q_tile, first_kv_block, kv_blocks, slot]``, merges, partial count, strategy) and
every merge-task list is stored as the first 16 hex digits of the SHA-256 of its canonical JSON
(``digest`` below), which keeps the fixture small while pinning each plan exactly.
"""
import argparse
import hashlib
import importlib.util
import json
import pathlib

HERE = pathlib.Path(__file__).resolve().parent

QS = (1, 17, 64, 128, 129, 256, 257, 512, 1024, 2048, 3712, 4096, 8192, 16384, 32768)
KVS = (128, 512, 1024, 2048, 4096, 8192, 16384, 24576, 32768)
CORES = (1, 2, 7, 27, 28)


def load(reference):
    path = pathlib.Path(reference) / "operators" / "mha" / "static_schedule.py"
    spec = importlib.util.spec_from_file_location("reference_static_schedule", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def digest(value):
    return hashlib.sha256(json.dumps(value, separators=(",", ":")).encode()).hexdigest()[:16]


def plan_record(plan):
    return digest({"programs": [[list(s) for s in program] for program in plan.programs],
                   "merges": [list(m) for m in plan.merges], "partial_count": plan.partial_count,
                   "strategy": plan.strategy})


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of an FGW checkout")
    args = parser.parse_args()
    ref = load(args.reference)
    out = {"make_plan": {}, "make_q_plan": {}, "make_tail_plan": {}, "make_stream_plan": {}, "choose_plan": {},
           "choose_stream_plan": {}, "make_merge_tasks": {}, "make_block_merge_tasks": {}}
    for q in QS:
        for kv in KVS:
            out["choose_plan"][f"{q},{kv}"] = plan_record(ref.choose_plan(q, kv))
            chosen = ref.choose_stream_plan(q, kv)
            out["choose_stream_plan"][f"{q},{kv}"] = plan_record(chosen)
            out["make_merge_tasks"][f"{q},{kv}"] = digest([list(t) for t in ref.make_merge_tasks(chosen)])
            out["make_block_merge_tasks"][f"{q},{kv}"] = digest([[list(t) for t in w]
                                                                 for w in ref.make_block_merge_tasks(chosen)])
            for cores in CORES:
                key = f"{q},{kv},{cores}"
                out["make_plan"][key] = plan_record(ref.make_plan(q, kv, cores))
                out["make_q_plan"][key] = plan_record(ref.make_q_plan(q, kv, cores))
                out["make_stream_plan"][key] = plan_record(ref.make_stream_plan(q, kv, cores))
                for pieces in (None, 2, 7):
                    out["make_tail_plan"][f"{key},{pieces}"] = plan_record(ref.make_tail_plan(q, kv, cores, pieces))
    (HERE / "static_schedule.json").write_text(json.dumps(out, separators=(",", ":")))
    print("wrote", HERE / "static_schedule.json")


if __name__ == "__main__":
    main()
