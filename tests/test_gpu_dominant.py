"""The most-frequent-bin skip against the oracle. LightGBM skips each feature's most_freq_bin in its sparse
histograms, and the reference's hist_quant keeps it in a register (crates/silvic-gpu/kernels/kernels.kern:439-468).
Here a tile of features dominated by one bin each stores every feature's bins 0 and mfb exchanged. The tree kernel's
histogram then adds no stored 0 and recovers that bin from the rows' totals. These tests force the skip on every
tile (share 0) or on the tiles a share of 0.125 picks. They check every reader of the exchanged tile bytes: the tree
kernel's training, the standalone histogram (its slab path and its direct path for small leaves), the API partition
and add_tree. Each must equal the oracle, which never exchanges bins."""

from __future__ import annotations

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend, Model, init_score
import oracle_lib as orc
from synth import random_binned

pytestmark = pytest.mark.gpu


def dominant_binned(rows, bins, share, seed=21, label_kind="regression"):
    """Each feature's `share` of rows in one bin, spread over the bins (0 for some features, the last for others)."""
    skew_bins = [(f * 37 + 5) % nb if f % 4 else (0 if f % 8 else nb - 1) for f, nb in enumerate(bins)]
    return random_binned(rows, bins, seed=seed, skew=share, skew_bins=skew_bins, label_kind=label_kind)


def loaded(data, share, objective=_abi.REGRESSION, sigmoid=1.0):
    b = B200Backend(0)
    b.set_dominant_share(share)
    b.load(data, objective, sigmoid)
    return b


BINS = [63] * 40 + [255] * 30 + [7, 2, 3]

TRAIN_CASES = [
    ("l2_all_tiles", 0.0, 0.9, dict(objective=_abi.REGRESSION, num_leaves=31, num_iterations=4)),
    ("l2_chosen", 0.125, 0.9, dict(objective=_abi.REGRESSION, num_leaves=31, num_iterations=4)),
    ("binary_features", 0.0, 0.6, dict(objective=_abi.BINARY, num_leaves=63, num_iterations=4,
                                       feature_fraction=0.7)),
    ("l2_sparse_leaves", 0.0, 0.97, dict(objective=_abi.REGRESSION, num_leaves=127, num_iterations=3,
                                         min_data_in_leaf=5, num_grad_quant_bins=16)),
]


@pytest.mark.parametrize("name,share,skew,params", TRAIN_CASES, ids=[c[0] for c in TRAIN_CASES])
def test_training_with_skipped_bins_matches_oracle(device, name, share, skew, params):
    data = dominant_binned(60_000, BINS, skew, label_kind="binary" if "binary" in name else "regression")
    p = orc.default_params(**params)
    ref = orc.train([data], p)
    b = loaded(data, share, p.objective, p.sigmoid)
    model = b.train(p, init_score(p, data.label))
    b.close()
    assert len(model.trees) == len(ref.trees)
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
    assert model.to_lightgbm_string(data, p) == Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)


def test_uniform_data_keeps_its_tiles(device):
    """Without a dominant bin a share of 0.125 exchanges nothing, and training still matches."""
    data = random_binned(30_000, [255] * 40, seed=5)
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=31, num_iterations=2)
    ref = orc.train([data], p)
    b = loaded(data, 0.125)
    model = b.train(p, init_score(p, data.label))
    b.close()
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"


@pytest.mark.parametrize("share", [0.0, 2.0])
def test_api_readers_of_exchanged_tiles_match_oracle(device, share):
    """Histograms (a large leaf through the slabs, a small one straight to the output), the partition and add_tree
    on a handle whose every tile exchanges bins 0 and mfb (share 0), and on one that exchanges none (share 2)."""
    data = dominant_binned(50_000, BINS, 0.8, seed=3)
    b = loaded(data, share)
    n = data.num_rows
    r = np.arange(n)
    grad = ((r * 7 + 1) % 13).astype(np.float32) / 4.0 - 1.5
    hess = 0.25 + ((r + 1) % 5).astype(np.float32) / 8.0
    b.write_gradients(grad, hess)
    spec = orc.quant_spec(1.5, 0.75, None, 4, True, 9, 3)
    b.quantize(spec)
    packed = b.read_packed()
    b.reset_partition()
    for begin, count in [(0, n), (1000, 20_000), (n - 3000, 3000), (7, 100)]:
        got = b.histogram(begin, count)
        want = orc.histogram(data, packed, np.arange(begin, begin + count))
        assert np.array_equal(got, want), f"leaf {begin}+{count}"
    # a split on a feature whose dominant bin is neither 0 nor the last (feature 1), and on one dominated by bin 0
    for column, bits in [(1, 0b1011 | (1 << ((1 * 37 + 5) % 63))), (4, 0b110)]:
        b.reset_partition()
        split = _abi.BinSplit()
        split.group, split.column = 0, column
        split.left_bins[0] = bits & 0xFFFFFFFF
        split.left_bins[1] = bits >> 32
        left = b.partition(500, 40_000, split)
        part = b.read_partition()
        ref_left, ref_rows = orc.partition(data, split, np.arange(500, 40_500))
        assert left == ref_left, f"column {column}"
        assert np.array_equal(part[500:40_500], ref_rows), f"column {column}"
        b.init_scores(0, 0.0)
        nodes = [_abi.DeviceNode(split, ~0, ~1)]
        b.add_tree(nodes, [0.5, -0.25])
        want_scores = orc.add_tree(data, nodes, [0.5, -0.25], np.zeros(n, dtype=np.float32))
        assert np.array_equal(b.scores(), want_scores), f"add_tree on column {column}"
    b.close()
