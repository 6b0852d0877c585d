"""Inputs of the binning tests: the reference's generated feature columns (parity_tests.rs:20-58, the numerical
ones) binned with LightGBM 3.3.5's thresholds for them (tests/golden/binning/lightgbm_thresholds.json), and
hash-drawn matrices with NaN, signed zeros, infinities and values on the bounds."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from silvic_b200.dataset import FeatureGroup, FeatureMeta
from synth import mix32

FIXTURE = Path(__file__).parent / "golden" / "binning" / "lightgbm_thresholds.json"


def unit(stream: int, rows: np.ndarray) -> np.ndarray:
    """parity_tests.rs:21-24: mix32(mix32(row) ^ mix32(stream)) >> 8 over 2^24, as f64."""
    h = mix32(mix32(rows.astype(np.uint32)) ^ mix32(np.uint32(stream)))
    return (h >> np.uint32(8)).astype(np.float64) / 16_777_216.0


def feature_column(name: str, rows: np.ndarray) -> np.ndarray:
    """parity_tests.rs:26-58 `feature_value` for the numerical features, the same operations in the same order."""
    u = lambda s: unit(s, rows)  # noqa: E731
    if name == "normal":
        return (((u(10) + u(11)) + u(12)) + u(13) - 2.0) * 1.5
    if name == "zeros_nan":
        a = u(20)
        return np.where(a < 0.3, 0.0, np.where(a < 0.4, np.nan, ((u(21) + u(22)) - 1.0) * 3.0))
    if name == "integers":
        return np.floor(u(30) * 20.0) - 5.0
    if name == "mass_points":
        return np.where(u(40) < 0.5, 1.0, ((u(41) * u(42)) * u(43)) * 1000.0)
    if name == "negative":
        v = u(50)
        return -(v * v * 10.0) - 0.5
    if name == "tiny":
        a = u(60)
        return np.where(a < 0.2, 1e-36, np.where(a < 0.3, -1e-36, u(61) - 0.5))
    raise ValueError(name)


def lightgbm_case(rows: int = 150_000):
    """(values [rows, F] f64, features, groups): the fixture's numerical features with LightGBM's thresholds (plus
    +inf) as upper bounds, `zeros_nan` with a NaN bin, in groups of two columns and a row stride of 4."""
    fx = json.loads(FIXTURE.read_text())
    r = np.arange(rows, dtype=np.uint64)
    cols, feats = [], []
    for i, f in enumerate(fx["features"]):
        ub = np.array([float(t) for t in f["thresholds"]] + [np.inf])
        nan = f["name"] == "zeros_nan"
        cols.append(feature_column(f["name"], r))
        feats.append(FeatureMeta(name=f["name"], num_bins=len(ub) + int(nan), nan_bin=nan, upper_bounds=ub,
                                 group=i // 2, column=i % 2))
    groups = [FeatureGroup([g * 2 + k for k in range(2) if g * 2 + k < len(feats)], 4, 0, 0,
                           np.zeros((0, 4), np.uint8)) for g in range((len(feats) + 1) // 2)]
    return np.stack(cols, axis=1), feats, groups


def hashed_case(rows: int, cols: int, seed: int, dtype=np.float32, per_group: int = 5, max_bounds: int = 255):
    """A rows × cols matrix of hashed values (a share NaN, ±0, ±inf, and values equal to a bound) with random
    ascending bounds per feature, in groups of `per_group` features (stride rounded up to 4)."""
    r = np.arange(rows * cols, dtype=np.uint64).reshape(rows, cols)
    u = unit(seed, r)
    v = (u - 0.5) * 40.0
    kind = unit(seed + 1, r)
    v = np.where(kind < 0.03, np.nan, v)
    v = np.where((kind >= 0.03) & (kind < 0.05), 0.0, v)
    v = np.where((kind >= 0.05) & (kind < 0.06), -0.0, v)
    v = np.where((kind >= 0.06) & (kind < 0.065), np.inf, v)
    v = np.where((kind >= 0.065) & (kind < 0.07), -np.inf, v)
    feats = []
    rng = np.random.default_rng(seed)
    for f in range(cols):
        n = int(rng.integers(1, max_bounds + 1))
        ub = np.sort(rng.uniform(-20, 20, n - 1).astype(dtype).astype(np.float64))
        ub = np.concatenate([ub, [np.inf]])
        nan = bool(rng.integers(0, 2)) and n < 256
        feats.append(FeatureMeta(name=f"f{f}", num_bins=n + int(nan), nan_bin=nan, upper_bounds=ub,
                                 group=f // per_group, column=f % per_group))
        # a tenth of the column's finite values land exactly on a bound
        on = (unit(seed + 2, r[:, f]) < 0.1) & np.isfinite(v[:, f])
        pick = (unit(seed + 3, r[:, f]) * n).astype(np.int64) % max(n - 1, 1)
        if n > 1:
            v[on, f] = ub[pick[on]]
    groups = []
    for g in range((cols + per_group - 1) // per_group):
        members = list(range(g * per_group, min(cols, (g + 1) * per_group)))
        groups.append(FeatureGroup(members, (len(members) + 3) // 4 * 4, 0, 0, np.zeros((0, 4), np.uint8)))
    return v.astype(dtype), feats, groups
