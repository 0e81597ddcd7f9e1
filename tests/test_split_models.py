"""Split selection is bit-exact against FGW's selectors (golden tables from the reference itself)."""
import pytest

from fgw_b200.operators.mha import general_split_cost_model as gm
from fgw_b200.operators.mha import general_split_policy as gp
from fgw_b200.operators.mha import split_cost_model as sm
from golden_data import split_tables

TABLES = split_tables()


def test_v7_select_splits_bit_exact():
    rows = TABLES["v7_select_splits"]
    assert len(rows) > 2000
    for batch, sq, heads, kv_tiles, expected in rows:
        assert sm.select_splits(batch, sq, heads, kv_tiles) == expected, (batch, sq, heads, kv_tiles)


def test_v7_eligible_config_bit_exact():
    for row in TABLES["v7_eligible_config"]:
        assert sm.eligible_config(**row["args"], **row["kwargs"]) == row["result"], row


def test_general_fill_policy_bit_exact():
    for tasks, capacity, target, expected in TABLES["general_fill"]:
        assert gp.select_splits(tasks, capacity, None, target) == expected


@pytest.mark.parametrize("version", [1, 2])
def test_general_cost_model_bit_exact(version):
    rows = [r for r in TABLES["general_model"] if r["version"] == version]
    assert len(rows) >= 300
    for r in rows:
        args = (r["batch"], r["sq"], r["heads"], r["dim"])
        for s in gp.SPLITS:
            assert gm.features(*args, r["lengths"], s, version) == r["features"][str(s)]
            # exact float equality: same operations in the same order
            assert gm.predict_us(*args, r["lengths"], s, version=version) == r["predict_us"][str(s)]
        assert gm.select_model_splits(*args, r["page"], r["width"], r["lengths"], version=version) == r["select"]


def test_legacy_rules_known_answers():
    # v7.py:94-96 restated: tasks = B*ceil(Sq/128)*H; double while <16, 2S <= W*p/128, tasks*S < 128.
    assert sm.legacy_splits(1, 1, 1, 16, 128) == 16       # config 1: one task, 16 KV tiles
    assert sm.legacy_splits(2, 1, 8, 16, 128) == 8        # 16 tasks -> 16*8 = 128 stops
    assert sm.legacy_splits(2, 4096, 8, 16, 128) == 1     # 512 tasks
    assert sm.legacy_splits(1, 1, 1, 2, 128) == 2
    # v2.py:21-29: tile 32 when page%32 == 0 else 16; tasks = B*Sq*H.
    assert sm.vector_fallback_splits(2, 2, 2, 2, 16) == 2  # capacity 32 tokens -> 2 tiles of 16
    assert sm.vector_fallback_splits(1, 1, 1, 64, 16) == 16


def test_general_policy_errors_match_reference():
    with pytest.raises(ValueError):
        gp.select_splits(0, 4)
    with pytest.raises(ValueError):
        gp.select_splits(4, 4, num_splits=3)
    with pytest.raises(ValueError):
        gp.select_splits(4, 4, num_splits=8)
    with pytest.raises(ValueError):
        gm.select_model_splits(1, 1, 1, 128, 128, 2, None)
    with pytest.raises(ValueError):
        gm.features(1, 1, 1, 24, [0], 1)


def test_b200_models_load_and_choose_valid_splits():
    general = gm.load_model(3)
    for lengths in ([2048], [1024] * 256, [0, 32768]):
        s = gm.select_model_splits(len(lengths), 1, 32, 128, 64, 512, lengths, model=general, cores=148)
        assert s in gp.SPLITS


def _sweep():
    import json
    import pathlib
    return json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "b200_split_sweep.json").read_text())


def test_b200_model_is_the_fit_of_the_committed_sweep():
    # fit_split_cost_model minimises the loss of FGW's fitter (tools/mha/fit_general_split_model.py) by exact
    # nonnegative least squares; refitting the committed B200 sweep reproduces the shipped model and its
    # validation
    from fgw_b200.operators.mha.fit_split_cost_model import fit_and_validate
    shipped = gm.load_model(3)
    model = fit_and_validate(_sweep()["rows"], version=3, cores=148)
    assert model["weights"] == pytest.approx(shipped["weights"], rel=1e-6, abs=1e-9)
    assert model["latency_floor_us"] == shipped["latency_floor_us"]
    loso = model["validation"]["leave_one_shape_out"]
    assert loso["geomean_regret_percent"] < 5 and loso["max_regret_percent"] < 30 and loso["within_2pct"] >= 55


def test_b200_features_by_hand():
    # decode path (Q <= 8): D128 items carry 2 query rows; 2048 tokens = 16 tiles of 128
    f = gm.features(1, 1, 1, 128, [2048], 4, version=3, cores=148)
    assert f == [1.0, 4.0, 0.0, 1.0, 0.0, 1.0, 4.0, 4 / 148, 0.0, 0.0]
    # tensor path, one split, few items: the contiguous schedule spreads 16 tiles over 148 programs
    f = gm.features(1, 16, 1, 128, [2048], 1, version=3, cores=148)
    assert f == [1.0, 0.0, 1.0, 0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 16.0]
    # tensor path, 2 x 8 heads x 2 query pairs x 4 splits = 128 items in one wave
    f = gm.features(2, 512, 8, 128, [4096, 2048], 4, version=3, cores=148)
    assert f[2] == 6.0 and f[4] == 1.0 and f[8] == 8 - 6.0
    with pytest.raises(ValueError):
        gm.features(1, 1, 1, 128, [2048], 3, version=3)
    # the B200 candidates go past the reference's 32 (one request and head over a long cache); versions 1 and 2
    # keep the reference's set
    f = gm.features(1, 1, 1, 128, [131072], 64, version=3, cores=148)
    assert f[:7] == [1.0, 16.0, 0.0, 1.0, 0.0, 1.0, 64.0]
    assert gm.B200_SPLITS == (1, 2, 4, 8, 16, 32, 64, 128)
    with pytest.raises(ValueError):
        gm.features(1, 1, 1, 128, [131072], 64, version=2)


def test_b200_model_picks_past_32_splits_on_a_long_single_head_cache():
    # measured (committed sweep): B1 H1 Q1 KV131072 runs 43 us at 64 splits against 59 at 32 and 97 at 16
    model = gm.load_model(3)
    assert gm.select_model_splits(1, 1, 1, 128, 128, 1024, [131072], model=model) == 64
    assert gm.select_model_splits(2, 1, 8, 128, 128, 256, [32768, 32768], model=model) <= 32


def test_b200_model_selection_on_the_sweep():
    model = gm.load_model(3)
    rows = _sweep()["rows"]
    regret = []
    for r in rows:
        if "32" in r["median_us"] or r["B"] == 2:  # splits the route measured
            pick = gm.select_model_splits(r["B"], r["Q"], r["H"], r["D"], r["page_size"], r["table_width"],
                                          list(r["lengths"]), model=model)
            if str(pick) in r["median_us"]:
                regret.append(r["median_us"][str(pick)] / min(r["median_us"].values()))
    assert len(regret) > 40 and max(regret) < 1.5


def test_work_accounting_matches_the_oracle():
    # the product's FLOP/byte accounting (reported by bench.py) equals the oracle's restatement of FGW's policy
    import oracle
    from fgw_b200.operators.mha import work
    for lengths in ([2048, 2048], [0, 1, 130, 4096], [17, 0], [32768]):
        for sq in (1, 8, 129, 4096):
            for causal in (False, True):
                assert work.useful_flops(lengths, sq, 8, 128, causal) == oracle.useful_flops(lengths, sq, 8, 128, causal)
        assert (work.algorithmic_bytes(lengths, len(lengths), 4, 8, 128, 16, 2)
                == oracle.algorithmic_bytes(lengths, len(lengths), 4, 8, 128, 16, 2))
    assert work.useful_flops([2048, 2048], 4096, 8, 128, False) == 68_719_476_736  # config 2: 68.72 GFLOP


@pytest.mark.parametrize("bad", [dict(_b200_splits=3), dict(_b200_splits=256), dict(_b200_splits=64, num_splits=2),
                                 dict(_b200_splits=128)])
def test_b200_split_hook_is_checked_before_any_device_use(bad):
    # build_kernel(_b200_splits=...) times the B200 model's candidates past the reference's set; counts outside
    # B200_SPLITS, past the table's 128-token KV tiles (here 100 tiles) or given together with num_splits are
    # refused before the device is touched
    from fgw_b200.operators.mha.kernels.mha_paged_fwd_sm100 import build_kernel
    with pytest.raises(ValueError, match="_b200_splits"):
        build_kernel(1, 1, 1, 128, 128 * 100, 100, 128, False, "bfloat16", 0, **bad)


def test_b200_model_choice_is_a_candidate_within_the_table_capacity():
    import random
    model = gm.load_model(3)
    rng = random.Random(7)
    for _ in range(300):
        batch, heads = rng.choice([1, 2, 4, 16, 64]), rng.choice([1, 2, 8, 32])
        sq = rng.choice([1, 3, 8, 16, 128, 512, 4096])
        dim, page = rng.choice([16, 64, 128, 256]), rng.choice([16, 64, 128])
        width = rng.choice([1, 2, 7, 64, 512])
        lengths = [rng.randrange(0, page * width + 1) for _ in range(batch)]
        pick = gm.select_model_splits(batch, sq, heads, dim, page, width, lengths, model=model, cores=148)
        assert pick in gm.B200_SPLITS and pick <= max(1, -(-page * width // gm.KV_TILE))


def test_fit_cli_reproduces_the_shipped_model(tmp_path):
    import json
    import pathlib
    from fgw_b200.operators.mha import fit_split_cost_model
    sweep = pathlib.Path(__file__).resolve().parent / "golden" / "b200_split_sweep.json"
    out = tmp_path / "model.json"
    assert fit_split_cost_model.main(["--input", str(sweep), "--output", str(out), "--version", "3"]) == 0
    fitted = json.loads(out.read_text())
    shipped = gm.load_model(3)
    assert fitted["feature_names"] == shipped["feature_names"]
    assert fitted["training_rows"] == shipped["training_rows"]
    assert fitted["weights"] == pytest.approx(shipped["weights"], rel=1e-9, abs=1e-12)
