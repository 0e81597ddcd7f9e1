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
    b200 = sm.load_model(sm.B200_MODEL)
    assert b200["cores"] == 148
    s = sm.select_splits(2, 4096, 8, 16, model=b200)
    assert s in sm.SPLITS
    general = gm.load_model(2, str(gm.MODEL_DIR / "b200_general_split_cost_model.json"))
    for lengths in ([2048], [1024] * 256, [0, 32768]):
        s = gm.select_model_splits(len(lengths), 1, 32, 128, 64, 512, lengths, model=general, cores=148)
        assert s in gp.SPLITS
