"""The LightGBM model file (silvic_b200/model_text.py) against the reference's LightGBM fixtures
(tests/golden/lightgbm/, made by tests/golden/make_lightgbm_fixtures.py), as crates/silvic-core/tests/
model_lightgbm.rs:107-200 checks its own writer: LightGBM 3.3.5 files write back byte for byte, parsing a written
file is lossless, raw predictions equal LightGBM's bit for bit (all trees and a prefix), and the importances match.
Then a model trained by the oracle, written and read back, predicts what the oracle's model predicts."""

import json
import math
import struct
from pathlib import Path

import numpy as np
import pytest

from silvic_b200 import model_text as mt

GOLDEN = Path(__file__).resolve().parent / "golden" / "lightgbm"
CASES = json.loads((GOLDEN / "cases.json").read_text())


def _bits(x: float) -> int:
    return struct.unpack("<q", struct.pack("<d", x))[0]


def _cases(versions=("v3", "v4")):
    for v in versions:
        for case in CASES[v]["cases"]:
            yield case


@pytest.mark.parametrize("case", list(_cases(("v3",))), ids=lambda c: c["name"])
def test_lightgbm_files_write_back_byte_for_byte(case):
    text = (GOLDEN / case["model_file"]).read_text()
    written = mt.TextModel.from_string(text).to_string()
    if written != text:
        i = next(k for k, (a, b) in enumerate(zip(written, text)) if a != b) if any(
            a != b for a, b in zip(written, text)) else min(len(written), len(text))
        pytest.fail(f"first difference at byte {i}: {written[max(0, i - 60):i + 60]!r} vs {text[max(0, i - 60):i + 60]!r}")


@pytest.mark.parametrize("case", list(_cases()), ids=lambda c: c["name"])
def test_parsing_written_models_is_lossless(case):
    model = mt.TextModel.from_string((GOLDEN / case["model_file"]).read_text())
    again = mt.TextModel.from_string(model.to_string())
    assert again.to_string() == model.to_string()
    assert len(again.trees) == len(model.trees)
    for a, b in zip(again.trees, model.trees):
        assert a.num_leaves == b.num_leaves and a.leaf_value == b.leaf_value and a.threshold == b.threshold


@pytest.mark.parametrize("case", list(_cases()), ids=lambda c: c["name"])
def test_raw_predictions_match_lightgbm_bit_for_bit(case):
    model = mt.TextModel.from_string((GOLDEN / case["model_file"]).read_text())
    for row, raw, prefix in zip(case["rows"], case["raw"], case["raw_prefix"]):
        x = [float(v) for v in row]
        assert _bits(model.predict_raw_row(x)) == _bits(float(raw)), (row, raw)
        assert _bits(model.predict_raw_row(x, case["prefix_trees"])) == _bits(float(prefix)), (row, prefix)


@pytest.mark.parametrize("case", list(_cases()), ids=lambda c: c["name"])
def test_feature_importance_matches_lightgbm(case):
    model = mt.TextModel.from_string((GOLDEN / case["model_file"]).read_text())
    assert model.split_importance() == [int(v) for v in case["importance_split"]]
    assert [_bits(v) for v in model.gain_importance()] == [_bits(float(v)) for v in case["importance_gain"]]


def test_rejects_unsupported_and_malformed_models():
    text = (GOLDEN / "binary.txt").read_text()
    for old, new in [("num_class=1", "num_class=3"), ("objective=binary sigmoid:0.7", "objective=multiclass num_class:3"),
                     ("objective=binary sigmoid:0.7", "objective=regression_l1"), ("is_linear=0", "is_linear=1")]:
        assert old in text
        with pytest.raises(mt.UnsupportedModel):
            mt.TextModel.from_string(text.replace(old, new, 1))
    tree0 = text[text.index("Tree=0"):text.index("Tree=1")]
    left = next(line for line in tree0.splitlines() if line.startswith("left_child="))
    first = left.split("=")[1].split()
    bad_left = "left_child=" + " ".join(["0"] + first[1:])  # node 0 names itself: a cycle
    for old, new in [(left, bad_left), ("sigmoid:0.7", "sigmoid:0"), ("max_feature_idx=3", "max_feature_idx=4")]:
        with pytest.raises(mt.ModelFormatError):
            mt.TextModel.from_string(text.replace(old, new, 1))


def test_format_g_is_c_printf():
    assert mt.format_g(0.1, 17) == "0.10000000000000001"
    assert mt.format_g(1e-5) == "1e-05"
    assert mt.format_g(123456789.0) == "1.23457e+08"
    assert mt.format_g(1.015625) == "1.01562"  # half to even, as glibc
    assert mt.format_g(-0.0) == "-0" and mt.format_g(math.inf) == "inf" and mt.format_g(math.nan) == "nan"


def test_a_trained_model_writes_and_predicts(oracle):
    """An oracle-trained model as silvic's model file: it parses back, writes back identically, and predicts what
    the trained trees predict (the host `Tree` leaf walk)."""
    from synth import random_binned

    from silvic_b200.backend import Model

    data = random_binned(3000, [16, 9, 33, 5], seed=11, label_kind="binary")
    p = oracle.default_params(objective=1, num_leaves=15, num_iterations=4)
    trained = oracle.train([data], p)
    model = Model(trained.trees, trained.init_score, [])
    text = mt.from_trained(model, data, p).to_string()
    parsed = mt.TextModel.from_string(text)
    assert parsed.to_string() == text
    assert "\nparameters:\n[boosting: gbdt]\n[objective: binary]\n[num_iterations: 4]\n" in text
    rng = np.random.default_rng(5)
    for _ in range(50):
        row = rng.normal(size=len(data.features)) * 3
        want = 0.0
        for t in model.trees:  # in tree order, one rounding per add (Python's sum() compensates)
            want += float(t.leaf_value[t.leaf_index(row)])
        assert _bits(parsed.predict_raw_row(row)) == _bits(want)
