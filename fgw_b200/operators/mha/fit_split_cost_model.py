"""Offline fit of the B200 split-count latency model (``general_split_cost_model`` version 3).

The model predicts a launch's latency as ``max(f(shape, splits) . w, floor)`` with nonnegative weights
``w`` and one floor for single-split and one for multi-split launches. This module estimates ``w`` and the
floors from split sweeps measured on the GPU (the rows ``bench.py --sweep-splits`` writes).

Objective. The loss is the one FGW's fitter minimises (tools/mha/fit_general_split_model.py:15-64), so a
model fitted here means the same thing as one fitted there:

* absolute fit, in relative terms: for every measured (shape, split) with latency ``y`` and features ``f``,
  ``(f . w / y - 1)^2``;
* ranking within a shape (version >= 2): for a shape that measured ``k`` split counts and whose fastest
  measurement is ``y_min``, ``0.25 / ((k - 1) * y_min^2)`` times the sum over all pairs of split counts of
  ``((f_s - f_t) . w - (y_s - y_t))^2``. This term rewards getting the order of a shape's splits right even
  when a sweep session ran uniformly slow or fast.

Solution method (this module's own). The pairwise term is never formed pair by pair: with
``e_s = f_s . w - y_s``, the identity ``sum_{s<t} (e_s - e_t)^2 = k * sum_s (e_s - mean(e))^2`` turns a
shape's ``k (k - 1) / 2`` difference rows into ``k`` centred rows ``sqrt(k c) (f_s - mean f)`` with targets
``sqrt(k c) (y_s - mean y)``. The stacked system is then solved exactly (no iteration count, no stopping
tolerance) by Lawson-Hanson active-set nonnegative least squares after equilibrating the columns to unit
norm, which leaves the nonnegative minimiser unchanged.

Floors are the fastest single- and multi-split measurements in the training rows. Validation reports the
regret of the model's choice (``general_split_cost_model.pick_within_tolerance`` over the split counts a row
measured) on the training rows and leave-one-shape-out (a shape's FP16 and BF16 rows held out together).

    python -m fgw_b200.operators.mha.fit_split_cost_model --input sweep.json --output model.json
"""
import argparse
import hashlib
import json
import math
import pathlib

import numpy as np
from scipy.optimize import nnls

from fgw_b200.operators.mha.general_split_cost_model import (feature_names, features, pick_within_tolerance,
                                                             predict_us)

RANKING_WEIGHT = 0.25       # weight of the within-shape ranking term (version >= 2)
SELECTION_TOLERANCE = 0.02  # relative tolerance of the split choice
SELECTION_MARGIN_US = 1.0   # absolute tolerance of the split choice (version >= 2)


def _shape_block(row, version, cores):
    """Feature matrix [k, F] and latencies [k] of one sweep row, in its split-count order."""
    labels = list(row["median_us"])
    f = np.array([features(row["B"], row["Q"], row["H"], row["D"], list(row["lengths"]), int(s), version, cores)
                  for s in labels], dtype=np.float64)
    y = np.array([row["median_us"][s] for s in labels], dtype=np.float64)
    return f, y


def design(rows, version=3, cores=148):
    """Stacked least-squares system (matrix, target) whose nonnegative minimiser is the model's weights."""
    blocks, targets = [], []
    for row in rows:
        f, y = _shape_block(row, version, cores)
        blocks.append(f / y[:, None])
        targets.append(np.ones_like(y))
        k = len(y)
        if version >= 2 and k >= 2:
            weight = math.sqrt(k * RANKING_WEIGHT / (k - 1)) / y.min()
            blocks.append(weight * (f - f.mean(axis=0)))
            targets.append(weight * (y - y.mean()))
    return np.vstack(blocks), np.concatenate(targets)


def latency_floors(rows):
    single = [us for r in rows for s, us in r["median_us"].items() if int(s) == 1]
    multi = [us for r in rows for s, us in r["median_us"].items() if int(s) > 1]
    return {"single": min(single), "multi": min(multi)}


def fit(rows, version=3, cores=148):
    """Model dict (weights, floors, selection settings) fitted on ``rows``."""
    matrix, target = design(rows, version, cores)
    norms = np.linalg.norm(matrix, axis=0)
    norms[norms == 0.0] = 1.0  # a feature that never varies keeps weight 0
    solution, _ = nnls(matrix / norms, target, maxiter=50 * matrix.shape[1])
    return {"version": version, "cores": cores, "feature_names": list(feature_names(version)),
            "weights": (solution / norms).tolist(), "latency_floor_us": latency_floors(rows),
            "selection_tolerance": SELECTION_TOLERANCE,
            "absolute_selection_margin_us": SELECTION_MARGIN_US if version >= 2 else 0.0,
            "contrast_loss_weight": RANKING_WEIGHT if version >= 2 else 0.0, "solver": "nnls"}


def regrets(rows, model):
    """Per row: the split the model picks among the measured ones and its slowdown against the fastest."""
    out = []
    for row in rows:
        measured = {int(s): us for s, us in row["median_us"].items()}
        predicted = {s: predict_us(row["B"], row["Q"], row["H"], row["D"], list(row["lengths"]), s, model)
                     for s in measured}
        pick = pick_within_tolerance(predicted, model)
        out.append({"key": row["key"], "model_splits": pick,
                    "regret_percent": 100.0 * (measured[pick] / min(measured.values()) - 1.0)})
    return out


def summary(results):
    values = np.array([r["regret_percent"] for r in results], dtype=np.float64)
    return {"cases": int(values.size), "within_2pct": int(np.count_nonzero(values <= 2.0)),
            "max_regret_percent": float(values.max()),
            "geomean_regret_percent": float(100.0 * (np.exp(np.mean(np.log1p(values / 100.0))) - 1.0)),
            "results": results}


def fit_and_validate(rows, version=3, cores=148):
    """The fitted model with its training-set and leave-one-shape-out regret summaries."""
    model = fit(rows, version, cores)
    held_out = []
    for shape in sorted({r["case"] for r in rows}):
        trained = fit([r for r in rows if r["case"] != shape], version, cores)
        held_out += regrets([r for r in rows if r["case"] == shape], trained)
    model["validation"] = {"calibration": summary(regrets(rows, model)), "leave_one_shape_out": summary(held_out)}
    return model


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--input", required=True, help="rows written by bench.py --sweep-splits")
    parser.add_argument("--output", required=True)
    parser.add_argument("--version", type=int, choices=[1, 2, 3], default=3)
    parser.add_argument("--cores", type=int, default=148)
    args = parser.parse_args(argv)
    source = pathlib.Path(args.input)
    data = json.loads(source.read_text(encoding="utf-8"))
    rows = data["rows"]
    model = {"model": f"b200_general_v{args.version}", "status": "fitted on B200 split sweeps",
             **fit_and_validate(rows, args.version, args.cores), "hardware": data.get("gpu", "unknown"),
             "training_sha256": hashlib.sha256(source.read_bytes()).hexdigest(), "training_rows": len(rows),
             "training_shapes": len({r["case"] for r in rows}),
             "training_variants": sum(len(r["median_us"]) for r in rows),
             "fitting": "relative-error least squares plus within-shape ranking (centred rows), exact "
                        "nonnegative least squares; measured single/multi latency floors"}
    pathlib.Path(args.output).write_text(json.dumps(model, indent=1) + "\n", encoding="utf-8")
    brief = {name: {k: v for k, v in model["validation"][name].items() if k != "results"}
             for name in ("calibration", "leave_one_shape_out")}
    print(json.dumps({"weights": model["weights"], "floors": model["latency_floor_us"], **brief}, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
