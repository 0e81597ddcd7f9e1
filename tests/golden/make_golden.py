"""Generate the golden fixtures that pin the oracle and the split selectors to FGW itself.

Run once, pointing ``--reference`` at a checkout of FGW:

    python tests/golden/make_golden.py --reference <FGW checkout>

It needs the reference's own Python code but none of its NPU stack:

* ``reference()`` is lifted out of ``operators/mha/kernels/mha_paged_decode_ascend_v0.py`` (:129-144)
  and ``useful_flops`` out of ``benchmarks/mha/bench_mha_mfu.py`` (:63-66) by parsing the files and
  compiling just those functions, so ``torch_npu``/``tilelang`` are never imported;
* the split selectors (``operators/mha/split_cost_model.py``, ``general_split_policy.py``,
  ``general_split_cost_model.py``) are stdlib-only and are imported directly.

Outputs (all small, committed):

* ``reference_outputs.npz`` + ``reference_outputs.json``: the reference's output (FP16/BF16 bit patterns)
  for accuracy-harness cases, with the SHA-256 of the regenerated inputs;
* ``split_selection.json``: the reference selectors' answers over shape grids;
* ``useful_flops.json``: ``useful_flops`` on assorted lengths.
"""
import argparse
import ast
import itertools
import json
import pathlib
import random
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE.parent))

from fixtures import (CUBE, GENERAL, QUICK, SPLIT, STANDARD, build_case, dtype_name, input_digest,  # noqa: E402
                      to_bits)


def _lift_function(path, name, namespace):
    tree = ast.parse(pathlib.Path(path).read_text(encoding="utf-8"))
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            module = ast.Module(body=[node], type_ignores=[])
            exec(compile(module, str(path), "exec"), namespace)
            return namespace[name]
    raise LookupError(f"{name} not found in {path}")


def _output_cases():
    """(case, seed, dtype, causal, pattern) tuples kept small enough to commit (about 2 MB).

    Small cases cover seeds x dtypes x causal x {mixed, full, empty}; cases with more than 8192
    output elements keep seed 7 and three combinations; ``empty`` outputs are all zero and are
    stored as an index entry only.
    """
    chosen = []
    small = QUICK + GENERAL + SPLIT + [c for c in CUBE if c[1] * c[2] * c[3] * c[4] <= 70000 and c[0] != "cube_q128"]
    small += [c for c in STANDARD if c not in QUICK]
    for case in small:
        size = case[1] * case[2] * case[3] * case[4]
        if size <= 8192:
            seeds = (7, 42, 2026) if size <= 1024 else (7,)
            combos = itertools.product(seeds, (torch.bfloat16, torch.float16), (False, True),
                                       ("mixed", "full", "empty"))
        elif size <= 70000:
            combos = [(7, torch.bfloat16, False, "mixed"), (7, torch.bfloat16, True, "mixed"),
                      (7, torch.float16, False, "full")]
        else:
            combos = [(7, torch.bfloat16, True, "mixed")]
        chosen.extend((case, *combo) for combo in combos)
    return chosen


def make_outputs(ref_root):
    reference = _lift_function(ref_root / "operators/mha/kernels/mha_paged_decode_ascend_v0.py", "reference",
                               {"torch": torch})
    index, arrays = [], {}
    for case, seed, dtype, causal, pattern in _output_cases():
        inputs = build_case(case, seed, dtype, causal, pattern)
        expected = reference(inputs["q"], inputs["k"], inputs["v"], inputs["table"], inputs["lengths"],
                             case[5], causal)
        key = f"{case[0]}|{seed}|{dtype_name(dtype)}|{int(causal)}|{pattern}"
        index.append({"key": key, "case": list(case), "seed": seed, "dtype": dtype_name(dtype), "causal": causal,
                      "pattern": pattern, "lengths": inputs["lengths"].tolist(),
                      "input_sha256": input_digest(inputs)})
        if pattern != "empty":
            arrays[key] = to_bits(expected)
        elif torch.count_nonzero(expected.float()).item() != 0:
            raise AssertionError(f"{key}: reference produced non-zero output for empty caches")
    np.savez_compressed(HERE / "reference_outputs.npz", **arrays)
    (HERE / "reference_outputs.json").write_text(json.dumps(
        {"source": "FGW operators/mha/kernels/mha_paged_decode_ascend_v0.py:129-144 reference(), run on CPU",
         "torch": torch.__version__, "entries": index}, indent=1) + "\n", encoding="utf-8")
    return len(index)


def make_split_tables(ref_root):
    sys.path.insert(0, str(ref_root))
    from operators.mha import general_split_cost_model as gm  # noqa: E402
    from operators.mha import general_split_policy as gp  # noqa: E402
    from operators.mha import split_cost_model as sm  # noqa: E402

    rng = random.Random(2026)
    v7 = []
    for batch, heads in itertools.product((1, 2, 3, 4, 8), (1, 2, 4, 8, 16, 32)):
        for sq in (1, 2, 4, 7, 8, 16, 33, 64, 127, 128, 129, 512, 1000, 4096, 8192, 32768):
            for kv_tiles in (1, 2, 3, 4, 8, 15, 16, 17, 64, 256):
                v7.append([batch, sq, heads, kv_tiles, sm.select_splits(batch, sq, heads, kv_tiles)])
    eligible = []
    for _ in range(400):
        args = dict(batch=rng.choice([1, 2, 4, 5]), sq=rng.choice([1, 8192, 8193]), heads=rng.choice([1, 16, 17]),
                    kv_tokens=rng.choice([384, 512, 2048, 2049, 32768, 32896]))
        kwargs = dict(dtype=rng.choice(["bfloat16", "float16", "torch.bfloat16"]), dim=rng.choice([64, 128]),
                      page_size=rng.choice([64, 128]), causal=rng.choice([False, True]),
                      pipeline_stages=rng.choice([1, 2]), buffer_versions=rng.choice([2, 3]),
                      kv_versions=rng.choice([2, 3]), q_resident=rng.choice([True, False]),
                      schedule_mode=rng.choice(["manual", "auto"]), full_kv_cache=rng.choice([True, False]),
                      cube_cores=rng.choice([28, 24, None]))
        eligible.append({"args": args, "kwargs": kwargs,
                         "result": sm.eligible_config(**args, **kwargs)})
    fill = []
    for tasks in (1, 2, 3, 7, 13, 14, 27, 28, 29, 100, 1000):
        for capacity in (1, 2, 3, 4, 5, 8, 16, 31, 32, 64, 1024):
            for target in (28, 148):
                fill.append([tasks, capacity, target, gp.select_splits(tasks, capacity, None, target)])
    general = []
    for version in (1, 2):
        for _ in range(300):
            batch = rng.choice([1, 2, 3, 8])
            sq = rng.choice([1, 4, 17, 31, 32, 33, 129, 512])
            heads = rng.choice([1, 2, 8, 16])
            dim = rng.choice(range(16, 257, 16))
            page = rng.choice([16, 32, 48, 64, 128, 256])
            width = rng.choice([1, 2, 3, 8, 24, 64])
            capacity = page * width
            lengths = [rng.choice([0, 1, capacity // 2, capacity - 1, capacity, rng.randint(0, capacity)])
                       for _ in range(batch)]
            feats = {s: gm.features(batch, sq, heads, dim, lengths, s, version) for s in gp.SPLITS}
            preds = {s: gm.predict_us(batch, sq, heads, dim, lengths, s, version=version) for s in gp.SPLITS}
            general.append({"version": version, "batch": batch, "sq": sq, "heads": heads, "dim": dim, "page": page,
                            "width": width, "lengths": lengths,
                            "features": {str(s): v for s, v in feats.items()},
                            "predict_us": {str(s): v for s, v in preds.items()},
                            "select": gm.select_model_splits(batch, sq, heads, dim, page, width, lengths,
                                                             version=version)})
    (HERE / "split_selection.json").write_text(json.dumps(
        {"source": "FGW operators/mha/{split_cost_model,general_split_policy,general_split_cost_model}.py",
         "v7_select_splits": v7, "v7_eligible_config": eligible, "general_fill": fill,
         "general_model": general}, indent=None) + "\n", encoding="utf-8")
    return len(v7) + len(eligible) + len(fill) + len(general)


def make_flops(ref_root):
    useful = _lift_function(ref_root / "benchmarks/mha/bench_mha_mfu.py", "useful_flops", {})
    rng = random.Random(7)
    rows = []
    for _ in range(200):
        batch = rng.randint(1, 6)
        sq = rng.choice([1, 2, 5, 64, 129, 4096])
        lengths = [rng.choice([0, 1, sq - 1, sq, rng.randint(0, 5000)]) for _ in range(batch)]
        heads, dim, causal = rng.choice([1, 8, 32]), rng.choice([16, 128, 256]), rng.choice([False, True])
        rows.append([lengths, sq, heads, dim, causal, useful(lengths, sq, heads, dim, causal)])
    (HERE / "useful_flops.json").write_text(json.dumps(
        {"source": "FGW benchmarks/mha/bench_mha_mfu.py:63-66 useful_flops", "rows": rows}) + "\n",
        encoding="utf-8")
    return len(rows)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, help="path of an FGW checkout")
    args = parser.parse_args(argv)
    ref_root = pathlib.Path(args.reference)
    print("outputs", make_outputs(ref_root))
    print("split rows", make_split_tables(ref_root))
    print("flops rows", make_flops(ref_root))
    return 0


if __name__ == "__main__":
    sys.exit(main())
