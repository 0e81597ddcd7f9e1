"""Loader for the committed golden fixtures (see tests/golden/make_golden.py)."""
import functools
import json
import pathlib

import numpy as np
import torch

from fixtures import ALL_CASES

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@functools.lru_cache(maxsize=1)
def output_index():
    return json.loads((GOLDEN / "reference_outputs.json").read_text(encoding="utf-8"))["entries"]


@functools.lru_cache(maxsize=1)
def output_arrays():
    with np.load(GOLDEN / "reference_outputs.npz") as data:
        return {key: data[key] for key in data.files}


def expected_bits(entry):
    """uint16 bit patterns of the reference output, zeros for the empty pattern."""
    arrays = output_arrays()
    case = entry["case"]
    shape = (case[1], case[2], case[3], case[4])
    if entry["key"] in arrays:
        return arrays[entry["key"]].reshape(shape)
    return np.zeros(shape, dtype=np.uint16)


def entry_params(entry):
    case = ALL_CASES[entry["case"][0]]
    assert tuple(entry["case"]) == case
    dtype = torch.bfloat16 if entry["dtype"] == "bfloat16" else torch.float16
    return case, entry["seed"], dtype, entry["causal"], entry["pattern"]


@functools.lru_cache(maxsize=1)
def split_tables():
    return json.loads((GOLDEN / "split_selection.json").read_text(encoding="utf-8"))


@functools.lru_cache(maxsize=1)
def flops_rows():
    return json.loads((GOLDEN / "useful_flops.json").read_text(encoding="utf-8"))["rows"]
