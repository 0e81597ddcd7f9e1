"""Fit the split-count latency model on measured split sweeps (NumPy only; offline, on the host).

Restates the fitting method of FGW's tools/mha/fit_general_split_model.py (:15-64 ``fit``, :67-85
``evaluate`` / ``summarize``, :88-121 leave-one-shape-out) for the B200 model of
``general_split_cost_model``:

* every measured (shape, split) latency contributes one row of relative error: features / latency
  against a target of 1;
* version 2 and the B200 feature set (version 3) add, per shape, every pairwise split contrast (feature difference against latency
  difference), scaled by sqrt(0.25 / (splits - 1)) / the shape's best latency, so the fit ranks splits
  within a shape and is less sensitive to per-session constant offsets;
* columns are normalised, then nonnegative coordinate descent solves the least squares;
* the single- and multi-split latency floors are the smallest measured latencies of each kind;
* validation: calibration on all rows, and leave-one-shape-out (both dtypes of a shape held out together).

The input is the row list ``bench.py --sweep-splits`` writes. Selection during evaluation is restricted
to the split counts a row measured. ``cores`` is the SM count the features are computed for (148).

    python -m fgw_b200.operators.mha.fit_split_cost_model --input sweep.json --output model.json
"""
import argparse
import hashlib
import json
import math
import pathlib

import numpy as np

from fgw_b200.operators.mha.general_split_cost_model import feature_names, features, predict_us


def _features(row, splits, version, cores):
    return features(row["B"], row["Q"], row["H"], row["D"], list(row["lengths"]), int(splits), version, cores)


def fit(rows, version=3, cores=148, iterations=8000):
    """Nonnegative weights, latency floors and selection settings fitted on ``rows``."""
    x = np.array([_features(r, s, version, cores) for r in rows for s in r["median_us"]], dtype=float)
    y = np.array([us for r in rows for us in r["median_us"].values()], dtype=float)
    a = x / y[:, None]
    target = np.ones(len(y))
    if version >= 2:
        contrast_x, contrast_y = [], []
        for r in rows:
            values = r["median_us"]
            labels = list(values)
            if len(labels) < 2:
                continue
            vectors = {s: np.array(_features(r, s, version, cores)) for s in labels}
            factor = math.sqrt(0.25 / (len(labels) - 1)) / min(values.values())
            for i, s in enumerate(labels):
                for t in labels[i + 1:]:
                    contrast_x.append((vectors[s] - vectors[t]) * factor)
                    contrast_y.append((values[s] - values[t]) * factor)
        if contrast_x:
            a = np.vstack([a, np.array(contrast_x)])
            target = np.concatenate([target, np.array(contrast_y)])
    scale = np.maximum(np.linalg.norm(a, axis=0), 1e-12)
    a = a / scale
    weights = np.zeros(a.shape[1])
    residual = target.copy()
    norms = np.sum(a * a, axis=0)
    done = 0
    for done in range(iterations):
        old = weights.copy()
        for j in range(len(weights)):
            update = max(0.0, weights[j] + a[:, j] @ residual / max(norms[j], 1e-20))
            residual += a[:, j] * (weights[j] - update)
            weights[j] = update
        if np.max(np.abs(weights - old)) < 1e-9:
            break
    floors = {mode: min(us for r in rows for s, us in r["median_us"].items() if (int(s) > 1) == multi)
              for mode, multi in (("single", False), ("multi", True))}
    return {"version": version, "cores": cores, "feature_names": list(feature_names(version)),
            "weights": (weights / scale).tolist(), "latency_floor_us": floors, "selection_tolerance": 0.02,
            "absolute_selection_margin_us": 1.0 if version >= 2 else 0.0,
            "contrast_loss_weight": 0.25 if version >= 2 else 0.0, "coordinate_descent_iterations": done + 1}


def select_measured(row, model):
    """The model's split choice among the split counts ``row`` measured (smallest within tolerance)."""
    costs = {int(s): predict_us(row["B"], row["Q"], row["H"], row["D"], list(row["lengths"]), int(s), model)
             for s in row["median_us"]}
    best = min(costs.values())
    if model["version"] == 1:
        limit = best * (1 + model["selection_tolerance"])
    else:
        limit = best + max(best * model["selection_tolerance"], model.get("absolute_selection_margin_us", 0.0))
    return min(s for s, value in costs.items() if value <= limit)


def evaluate(rows, model):
    results = []
    for r in rows:
        split = select_measured(r, model)
        selected = r["median_us"][str(split)]
        best = min(r["median_us"].values())
        results.append({"key": r["key"], "model_splits": split, "regret_percent": (selected / best - 1) * 100})
    return results


def summarize(results):
    regrets = [r["regret_percent"] for r in results]
    return {"cases": len(results), "within_2pct": sum(v <= 2 for v in regrets), "max_regret_percent": max(regrets),
            "geomean_regret_percent": (math.exp(sum(math.log1p(v / 100) for v in regrets) / len(regrets)) - 1) * 100,
            "results": results}


def fit_and_validate(rows, version=3, cores=148):
    """The fitted model with its calibration and leave-one-shape-out summaries attached."""
    model = fit(rows, version, cores)
    folds = []
    for shape in sorted({r["case"] for r in rows}):
        train = [r for r in rows if r["case"] != shape]
        held = [r for r in rows if r["case"] == shape]
        folds.extend(evaluate(held, fit(train, version, cores)))
    model["validation"] = {"calibration": summarize(evaluate(rows, model)), "leave_one_shape_out": summarize(folds)}
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
    model = fit_and_validate(data["rows"], args.version, args.cores)
    model = {"model": f"b200_general_v{args.version}", "status": "fitted on B200 split sweeps", **model,
             "hardware": data.get("gpu", "unknown"),
             "training_sha256": hashlib.sha256(source.read_bytes()).hexdigest(),
             "training_rows": len(data["rows"]), "training_shapes": len({r["case"] for r in data["rows"]}),
             "training_variants": sum(len(r["median_us"]) for r in data["rows"]),
             "fitting": "relative-error least squares with within-shape split contrasts, nonnegative coordinate "
                        "descent, measured single/multi latency floors (FGW tools/mha/fit_general_split_model.py)"}
    out = pathlib.Path(args.output)
    out.write_text(json.dumps(model, indent=1) + "\n", encoding="utf-8")
    print(json.dumps({"weights": model["weights"], "floors": model["latency_floor_us"],
                      "calibration": {k: v for k, v in model["validation"]["calibration"].items() if k != "results"},
                      "leave_one_shape_out": {k: v for k, v in model["validation"]["leave_one_shape_out"].items()
                                              if k != "results"}}, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
