"""LambdaRank on the device against the CPU oracle (objective/lambdarank.rs, restated in oracle/oracle.cpp), through
the C ABI: the gradients of every query at tied scores (the first iteration, where only row order ranks) and at
scores moved by trees, bit for bit, including a single-row query, queries whose labels are all equal and a query
of 3,000 rows; then whole training runs whose trees and model text equal the oracle's. The reference's own
lambdarank tests (lambdarank.rs:398-783) are ported against the oracle in test_lambdarank.py."""

from __future__ import annotations

import numpy as np
import pytest

from silvic_b200 import SilvicError, _abi
from silvic_b200.backend import B200Backend, Model, init_score
import oracle_lib as orc
from synth import ranking_binned

pytestmark = pytest.mark.gpu


def rank_params(**kw):
    base = dict(objective=_abi.LAMBDARANK, num_leaves=31, num_iterations=4, sigmoid=1.0, lambdarank_norm=1,
                lambdarank_truncation_level=30)
    base.update(kw)
    return orc.default_params(**base)


def device_gradients(b, data):
    b.compute_gradients()
    return b.read_gradients()


def test_lambdarank_gradients_match_oracle(device):
    data = ranking_binned(30_000, [63] * 6 + [255] * 2, seed=3, mean_query=60.0, long_query=3000)
    qb = data.query_boundaries
    assert np.diff(qb).max() == 3000
    p = rank_params()
    b = B200Backend(0)
    try:
        b.load(data, p.objective, p.sigmoid, p)
        b.init_scores(0, 0.0)
        g, h = device_gradients(b, data)
        want_g, want_h = orc.lambdarank_gradients(p, data.label, np.zeros(data.num_rows, np.float32), qb)
        assert np.array_equal(g.view(np.uint32), want_g.view(np.uint32)), "gradients at tied scores"
        assert np.array_equal(h.view(np.uint32), want_h.view(np.uint32)), "hessians at tied scores"
        # Scores moved by trees on several features (many distinct values and partial ties).
        rng = np.random.default_rng(9)
        for f in range(4):
            m = data.features[f]
            split = _abi.BinSplit(m.group, m.column)
            for bin_ in range(0, m.num_bins, 2):
                split.left_bins[bin_ // 32] |= 1 << (bin_ % 32)
            node = _abi.DeviceNode(split, -1, -2)
            b.add_tree([node], np.array(rng.normal(size=2), dtype=np.float32))
        scores = b.scores()
        g, h = device_gradients(b, data)
        want_g, want_h = orc.lambdarank_gradients(p, data.label, scores, qb)
        assert np.array_equal(g.view(np.uint32), want_g.view(np.uint32)), "gradients at moved scores"
        assert np.array_equal(h.view(np.uint32), want_h.view(np.uint32)), "hessians at moved scores"
    finally:
        b.close()


def test_lambdarank_single_row_and_equal_label_queries(device):
    data = ranking_binned(2_000, [31] * 4, seed=8, mean_query=5.0)
    qb = data.query_boundaries.astype(np.int64).copy()
    data.label[qb[2]:qb[3]] = 2.0  # a query whose labels are all equal
    data.query_boundaries = np.concatenate([[0, 1], qb[1:] ]).astype(np.uint32)  # a single-row query first
    p = rank_params(lambdarank_truncation_level=3)
    b = B200Backend(0)
    try:
        b.load(data, p.objective, p.sigmoid, p)
        b.init_scores(0, 0.25)
        g, h = device_gradients(b, data)
    finally:
        b.close()
    want_g, want_h = orc.lambdarank_gradients(p, data.label, np.full(data.num_rows, 0.25, np.float32),
                                              data.query_boundaries)
    assert np.array_equal(g.view(np.uint32), want_g.view(np.uint32))
    assert np.array_equal(h.view(np.uint32), want_h.view(np.uint32))
    assert g[0] == 0.0 and h[0] == 0.0


@pytest.mark.parametrize("norm,trunc", [(1, 30), (0, 10)])
def test_lambdarank_training_matches_oracle(device, norm, trunc):
    data = ranking_binned(40_000, [255] * 10 + [63] * 4, seed=5, mean_query=120.0)
    p = rank_params(lambdarank_norm=norm, lambdarank_truncation_level=trunc)
    ref = orc.train([data], p)
    b = B200Backend(0)
    b.load(data, p.objective, p.sigmoid, p)
    model = b.train(p, init_score(p, data.label))
    b.close()
    assert model.init_score == ref.init_score == 0.0
    assert len(model.trees) == len(ref.trees) == 4
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
    text = model.to_lightgbm_string(data, p)
    assert "objective=lambdarank" in text and "lambdarank_truncation_level" in text
    assert text == Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)


def test_lambdarank_rejects_bad_queries_and_labels(device):
    data = ranking_binned(1_000, [31] * 3, seed=2)
    p = rank_params()
    b = B200Backend(0)
    try:
        bad = ranking_binned(1_000, [31] * 3, seed=2)
        bad.query_boundaries = np.array([0, 10, 900], dtype=np.uint32)  # does not reach the last row
        with pytest.raises(SilvicError, match="query boundaries"):
            b.load(bad, p.objective, p.sigmoid, p)
        bad = ranking_binned(1_000, [31] * 3, seed=2)
        bad.label[5] = 0.5
        with pytest.raises(SilvicError, match="lambdarank label"):
            b.load(bad, p.objective, p.sigmoid, p)
        long = ranking_binned(5_000, [31] * 3, seed=2)
        long.query_boundaries = np.array([0, 4097, 5000], dtype=np.uint32)
        with pytest.raises(SilvicError, match="4096"):
            b.load(long, p.objective, p.sigmoid, p)
        b.load(data, p.objective, p.sigmoid, p)
        with pytest.raises(SilvicError, match="lambdarank parameters"):
            b.train(rank_params(lambdarank_truncation_level=5), 0.0)
    finally:
        b.close()
