"""Writes `lightgbm_thresholds.json`: the numerical features of the reference's LightGBM 3.3.5 binning fixture
(crates/silvic-core/src/data/fixtures/lightgbm_bins.json, case "all_rows": the bin thresholds LightGBM's trees used
on 150,000 generated rows), the bounds the binning tests bin real-valued columns with. Run from the repository
root with the reference checkout's path as the argument; the output is committed, so the tests never read the
reference."""

import json
import sys
from pathlib import Path

NUMERICAL = ["normal", "zeros_nan", "integers", "mass_points", "negative", "tiny"]


def main(reference: str) -> None:
    src = Path(reference) / "crates/silvic-core/src/data/fixtures/lightgbm_bins.json"
    fixture = json.loads(src.read_text())
    case = next(c for c in fixture["cases"] if c["name"] == "all_rows")
    out = {"lightgbm": fixture["lightgbm"], "case": case["name"], "rows": case["rows"], "features": []}
    for f in case["features"]:
        if f["name"] in NUMERICAL and f.get("thresholds"):
            out["features"].append({"name": f["name"], "feature_infos": f["feature_infos"],
                                    "thresholds": f["thresholds"]})
    dst = Path(__file__).with_name("lightgbm_thresholds.json")
    dst.write_text(json.dumps(out, indent=1) + "\n")
    print(dst, [f["name"] for f in out["features"]])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_binning_fixture.py <reference checkout>")
    main(sys.argv[1])
