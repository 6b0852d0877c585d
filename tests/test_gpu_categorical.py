"""Categorical features on the device against the oracle, bit for bit: the split search (one-hot and sorted scans,
split.rs:694-845) on random integer histograms through sb2_find_best_split, and whole training runs through the tree
kernel whose trees and model files must equal the oracle's (crates/silvic-gpu/tests/metal_backend.rs:718-748 checks
the same device == CPU identity)."""

from __future__ import annotations

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend, Model, init_score
from silvic_b200.dataset import BinnedDataset, categorical_mapper, numerical_mapper
import oracle_lib as orc
from synth import categorical_binned

pytestmark = pytest.mark.gpu


def mixed_dataset(rng, nfeat):
    """Numerical and categorical features of random widths (categorical: 2 .. 255 bins, some <= 4 for one-hot)."""
    mappers = []
    for f in range(nfeat):
        if f % 2:
            nb = int(rng.choice([2, 3, 4, int(rng.integers(5, 256))]))
            mappers.append(categorical_mapper(f"c{f}", list(range(1000, 1000 + nb - 1))))
        else:
            mappers.append(numerical_mapper(f"n{f}", int(rng.integers(2, 256))))
    bins = np.zeros((64, nfeat), dtype=np.uint8)
    return BinnedDataset.from_bins(bins, mappers, np.zeros(64, dtype=np.float32))


def random_hist(rng, data):
    """Integer histograms (units): counts below 40, hessian 4 units a row, integer gradients."""
    h = np.zeros(2 * data.total_bins)
    for m in data.features:
        for k in range(m.num_bins):
            n = int(rng.integers(0, 40))
            h[2 * (m.hist_offset + k)] = float(rng.integers(-2 * n, 2 * n + 1))
            h[2 * (m.hist_offset + k) + 1] = float(n * 4)
    return h


@pytest.mark.parametrize("case", range(16))
def test_categorical_split_search_matches_oracle(device, case):
    rng = np.random.default_rng(700 + case)
    data = mixed_dataset(rng, int(rng.integers(1, 40)))
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    hist = random_hist(rng, data)
    m0 = data.features[0]
    g0 = hist[2 * m0.hist_offset: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    h0 = hist[2 * m0.hist_offset + 1: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    cfg = _abi.SplitConfig(min_data_in_leaf=int(rng.integers(0, 30)), min_sum_hessian_in_leaf=[1e-3, 0.0][case % 2],
                           lambda_l1=[0.0, 0.5][case % 2], lambda_l2=[0.0, 2.0, 10.0][case % 3],
                           min_gain_to_split=[0.0, 0.1][case % 2], min_data_per_group=[1, 20, 100][case % 3],
                           cat_l2=[10.0, 0.0, 3.5][case % 3], cat_smooth=[10.0, 1.0, 0.0][case % 3],
                           max_cat_to_onehot=[4, 2, 8][case % 3], max_cat_threshold=[32, 4, 1, 200][case % 4])
    evaluate = (rng.random(len(data.features)) < 0.9).astype(np.uint8)
    scale = (0.37 + case, 0.25)
    sums = (g0, h0, int(h0 // 4))
    got, gs = b.find_best_split(hist, evaluate, sums, scale, cfg)
    want, ws = orc.find_best_split(data, hist, evaluate, sums, scale, cfg)
    b.close()
    assert got.as_tuple() == want.as_tuple()
    assert np.array_equal(gs, ws)


def test_categorical_search_finds_categorical_splits(device):
    """Histograms where only a sorted categorical feature can split: the device and the oracle pick the same
    categories."""
    data = BinnedDataset.from_bins(np.zeros((8, 1), dtype=np.uint8),
                                   [categorical_mapper("c", list(range(1, 31)))], np.zeros(8, dtype=np.float32))
    rng = np.random.default_rng(11)
    rows = rng.integers(20, 200, size=31)
    g = np.where(np.arange(31) % 3 == 0, 1, -1) * rows
    hist = np.zeros(62)
    hist[0::2], hist[1::2] = g, rows * 4
    cfg = _abi.SplitConfig(min_data_in_leaf=5, min_sum_hessian_in_leaf=1e-3, min_data_per_group=10, cat_l2=10.0,
                           cat_smooth=10.0, max_cat_to_onehot=4, max_cat_threshold=32)
    sums = (float(g.sum()), float(rows.sum() * 4), int(rows.sum()))
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    got, _ = b.find_best_split(hist, [1], sums, (0.5, 0.25), cfg)
    b.close()
    want, _ = orc.find_best_split(data, hist, [1], sums, (0.5, 0.25), cfg)
    assert want.found and want.categorical
    assert got.as_tuple() == want.as_tuple()


TRAIN_CASES = [
    ("l2", "regression", dict(objective=_abi.REGRESSION, num_leaves=31, num_iterations=5, min_data_per_group=20)),
    ("binary", "binary", dict(objective=_abi.BINARY, num_leaves=31, num_iterations=5, min_data_per_group=50,
                              max_cat_threshold=8)),
    ("defaults", "regression", dict(objective=_abi.REGRESSION, num_leaves=63, num_iterations=4)),
    ("all_onehot", "regression", dict(objective=_abi.REGRESSION, num_leaves=15, num_iterations=4,
                                      max_cat_to_onehot=64, lambda_l2=1.0, cat_l2=0.0)),
]


@pytest.mark.parametrize("name,label_kind,params", TRAIN_CASES, ids=[c[0] for c in TRAIN_CASES])
def test_categorical_training_matches_oracle(device, name, label_kind, params):
    data = categorical_binned(40_000, seed=13, label_kind=label_kind)
    p = orc.default_params(**params)
    ref = orc.train([data], p)
    assert any(int(d) & 1 for t in ref.trees for d in t.decision_type), "the oracle made no categorical split"
    b = B200Backend(0)
    b.load(data, p.objective, p.sigmoid)
    model = b.train(p, init_score(p, data.label))
    b.close()
    assert len(model.trees) == len(ref.trees)
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
    assert model.to_lightgbm_string(data, p) == Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)


def test_categorical_partition_and_add_tree(device):
    """A categorical bin split through the API partition and add_tree (bins set in left_bins go left)."""
    data = categorical_binned(30_000, seed=2)
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    r = np.arange(data.num_rows)
    b.write_gradients(((r * 7) % 13).astype(np.float32) / 4.0 - 1.5, np.ones(data.num_rows, dtype=np.float32))
    b.quantize(orc.quant_spec(1.5, 1.0, None, 4, True, 1, 0))
    b.reset_partition()
    split = _abi.BinSplit()
    split.group, split.column = 0, 1
    split.left_bins[0] = 0b1010_0110_0001_0010
    split.left_bins[1] = 0b1001
    left = b.partition(100, 25_000, split)
    ref_left, ref_rows = orc.partition(data, split, np.arange(100, 25_100))
    assert left == ref_left
    assert np.array_equal(b.read_partition()[100:25_100], ref_rows)
    b.init_scores(0, 0.0)
    nodes = [_abi.DeviceNode(split, ~0, ~1)]
    b.add_tree(nodes, [0.75, -0.5])
    assert np.array_equal(b.scores(), orc.add_tree(data, nodes, [0.75, -0.5], np.zeros(data.num_rows, np.float32)))
    b.close()
