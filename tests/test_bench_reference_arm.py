"""``bench.py --impl reference`` on the host: the JSON line the driver reads, and rank > 0 staying silent.

The reference arm times the CPU restatement of FGW's reference attention on config 2's workload; it runs
on CPU only, so it is checked here as it runs on the GPU box.
"""
import contextlib
import io
import json
import pathlib
import sys

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[1]))

import bench  # noqa: E402


def test_reference_arm_prints_the_contract_line():
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "0"]) == 0
    lines = [line for line in out.getvalue().splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["steps"] == 1 and d["warmup"] == 0
    assert d["higher_is_better"] is True and d["vs_baseline"] is None
    assert d["config"] == bench.headline_config(1)  # the repo arm's config, key for key
    base = d["cpu_baseline"]
    assert base["value"] == d["value"] and base["kind"] == "port" and base["sample"]
    assert base["cores"] == bench.host_cores()  # every physical core, whatever OMP_NUM_THREADS says
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_on_other_ranks_does_no_work():
    args = bench.parse_args(["--impl", "reference", "--steps", "1", "--warmup", "0", "--gpus", "2"])
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        assert bench.reference_arm(args, 1, 2) == 0
    assert out.getvalue() == ""


def test_reference_arm_uses_every_core_under_torchrun_settings(monkeypatch):
    # torchrun exports OMP_NUM_THREADS=1; the arm raises the BLAS pools back to the host's physical cores
    from threadpoolctl import threadpool_info, threadpool_limits
    with threadpool_limits(limits=1, user_api="blas"):
        assert bench.use_all_host_cores() == bench.host_cores()
        assert max(i["num_threads"] for i in threadpool_info() if i["user_api"] == "blas") == bench.host_cores()
