"""The oracle's dense-matrix binning (data/binning.rs bin_rows, BinMapper::value_to_bin) against the reference's own
test of it (binning.rs:143-171: the padded branch-free search equals `partition_point(bound < value)` on every
probe) and on the reference's generated feature columns with LightGBM 3.3.5's thresholds as bounds."""

from __future__ import annotations

import math

import numpy as np

import oracle_lib as orc
from binning_cases import hashed_case, lightgbm_case
from silvic_b200.dataset import FeatureGroup, FeatureMeta
from synth import mix32


def one_column(ub, nan_bin, values) -> np.ndarray:
    feat = FeatureMeta(name="x", num_bins=len(ub) + int(nan_bin), nan_bin=nan_bin, upper_bounds=np.asarray(ub))
    grp = FeatureGroup([0], 4, 0, 0, np.zeros((0, 4), np.uint8))
    return orc.bin_rows(np.asarray(values, dtype=np.float64).reshape(-1, 1), [feat], [grp])[0][:, 0]


def test_padded_search_matches_value_to_bin():
    """binning.rs:143-171, the same lengths, bounds and probes."""
    for length in [1, 2, 3, 7, 64, 127, 128, 129, 200, 254, 255]:
        ub = [i * 0.5 - 20.0 for i in range(length - 1)] + [math.inf]
        probes = [float(mix32(np.uint32(i)) >> np.uint32(20)) / 50.0 - 50.0 for i in range(500)]
        for b in ub:
            probes += [b, math.nextafter(b, math.inf), math.nextafter(b, -math.inf)]
        probes += [0.0, -0.0, math.nan, math.inf, -math.inf]
        for nan_bin in (False, True):
            got = one_column(ub, nan_bin, probes)
            want = [orc.value_to_bin(ub, nan_bin, v) for v in probes]
            assert got.tolist() == want, (length, nan_bin)


def test_value_to_bin_rules():
    """bin_mapper.rs:343-360: bounds strictly below the value; NaN to the NaN bin or to 0.0's bin."""
    ub = [-1.0, 0.5, 2.0, math.inf]
    assert [orc.value_to_bin(ub, False, v) for v in [-5, -1.0, -0.99, 0.5, 0.6, 3.0, math.inf]] == [0, 0, 1, 1, 2, 3, 3]
    assert orc.value_to_bin(ub, False, math.nan) == 1
    assert orc.value_to_bin(ub, True, math.nan) == 4


def test_lightgbm_columns_bin_into_their_thresholds():
    """Each generated column binned with LightGBM's thresholds: every value lands in the bin of the first threshold
    at or above it (NaN in zeros_nan's NaN bin), row layout and padding as the groups say."""
    values, feats, groups = lightgbm_case(30_000)
    outs = orc.bin_rows(values, feats, groups)
    for f, m in enumerate(feats):
        g = groups[m.group]
        col = outs[m.group][:, m.column]
        ub = m.upper_bounds
        v = values[:, f]
        want = np.where(np.isnan(v), len(ub) if m.nan_bin else np.searchsorted(ub, 0.0, "left"),
                        np.searchsorted(ub, np.nan_to_num(v, nan=0.0), "left"))
        assert np.array_equal(col, want.astype(np.uint8)), m.name
        assert (outs[m.group][:, len(g.features):] == 0).all()
    # column-major input bins the same
    outs_f = orc.bin_rows(np.asfortranarray(values), feats, groups)
    for a, b in zip(outs, outs_f):
        assert np.array_equal(a, b)


def test_hashed_matrices_f32_and_f64():
    for dtype in (np.float32, np.float64):
        values, feats, groups = hashed_case(2_000, 13, seed=5, dtype=dtype)
        outs = orc.bin_rows(values, feats, groups)
        for f, m in enumerate(feats):
            col = outs[m.group][:, m.column]
            for r in range(0, 2_000, 97):
                assert col[r] == orc.value_to_bin(m.upper_bounds, m.nan_bin, float(values[r, f]))
