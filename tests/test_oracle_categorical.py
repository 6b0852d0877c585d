"""The oracle's categorical split scan against the reference's own tests of it (no GPU).

Ports split.rs:1252-1340: the one-hot scan (at most max_cat_to_onehot bins) equals a brute force over single
categories, and the sorted scan equals a brute force over prefixes of the ctr order from both ends, with cat_l2 in
the candidates but not in the gain shift. The children's sums, counts and outputs are checked against direct sums of
the bins the rule sends left (check_children, split.rs:1101-1148). Training then grows categorical splits that two
ranks reproduce, and the emitted model file predicts what the binned trees do."""

from __future__ import annotations

import math

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import Model
from silvic_b200.dataset import BinnedDataset, categorical_mapper
import oracle_lib as orc
from synth import categorical_binned

MIN_SCORE = -math.inf


class Lcg:
    """The reference tests' generator (split.rs:991-1005)."""

    def __init__(self, seed: int):
        self.s = seed

    def next(self) -> float:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return (self.s >> 11) / float(1 << 53)

    def below(self, n: int) -> int:
        return int(self.next() * n)


def random_hist(rng: Lcg, num_bins: int, hess_per_row: float):
    """split.rs:1047-1054: rows per bin below 40, gradients (u - 0.45) * rows, hessian rows * hess_per_row."""
    rows = [rng.below(40) for _ in range(num_bins)]
    hist = []
    for n in rows:
        hist += [(rng.next() - 0.45) * n, n * hess_per_row]
    return np.array(hist, dtype=np.float64), np.array(rows, dtype=np.int64)


def config(**over):
    """SplitConfig::new of Params { min_data_in_leaf: 5, ..default } (split.rs:1040-1045)."""
    c = dict(min_data_in_leaf=5, min_sum_hessian_in_leaf=1e-3, lambda_l1=0.0, lambda_l2=0.0, min_gain_to_split=0.0,
             min_data_per_group=100, cat_l2=10.0, cat_smooth=10.0, max_cat_to_onehot=4, max_cat_threshold=32)
    c.update(over)
    return _abi.SplitConfig(**c)


def leaf_gain(g, h, l1, l2):
    r = max(abs(g) - l1, 0.0)
    return r * r / (h + l2)


def leaf_output(g, h, l1, l2):
    s = float(g > 0) - float(g < 0)
    return -(s * max(abs(g) - l1, 0.0)) / (h + l2)


def side_sums(hist, rows, left):
    idx = [b for b in range(len(rows)) if left(b)]
    return sum(hist[2 * b] for b in idx), sum(hist[2 * b + 1] for b in idx), int(sum(rows[b] for b in idx))


def brute_force(hist, rows, cfg, l2, candidates):
    """split.rs:1068-1087 with the config's l2 replaced by `l2`."""
    tg, th, tn = hist[0::2].sum(), hist[1::2].sum(), int(rows.sum())
    shift = leaf_gain(tg, th, cfg.lambda_l1, l2) + cfg.min_gain_to_split
    best = MIN_SCORE
    for left in candidates:
        lg, lh, ln = side_sums(hist, rows, left)
        rg, rh, rn = tg - lg, th - lh, tn - ln

        def ok(n, h):
            return n >= cfg.min_data_in_leaf and n > 0 and h >= cfg.min_sum_hessian_in_leaf and h > 0.0

        if not ok(ln, lh) or not ok(rn, rh):
            continue
        gain = leaf_gain(lg, lh, cfg.lambda_l1, l2) + leaf_gain(rg, rh, cfg.lambda_l1, l2)
        if gain > shift:
            best = max(best, gain - shift)
    return best


def assert_close(found, expected, case):
    assert abs(found - expected) <= 1e-9 * max(abs(expected), 1.0), f"{case}: found {found}, brute force {expected}"


def left_bins(info):
    return [b for b in range(256) if (info.cat_bins[b // 32] >> (b % 32)) & 1]


def check_children(info, hist, rows, cfg, case):
    bins = left_bins(info)
    lg, lh, ln = side_sums(hist, rows, lambda b: b in bins)
    assert_close(info.left_grad, lg, f"{case}: left grad")
    assert_close(info.left_hess, lh, f"{case}: left hess")
    assert info.left_count == ln, f"{case}: left count"
    l2 = cfg.lambda_l2 + cfg.cat_l2 if len(bins) > 1 or len(rows) > cfg.max_cat_to_onehot else cfg.lambda_l2
    assert_close(info.left_output, leaf_output(lg, lh, cfg.lambda_l1, l2), f"{case}: left output")


def one_feature(num_bins):
    """A dataset whose one feature is categorical with categories 1 .. num_bins - 1 (split.rs:1027-1038)."""
    return BinnedDataset.from_bins(np.zeros((16, 1), dtype=np.uint8),
                                   [categorical_mapper("c", list(range(1, num_bins)))], np.zeros(16))


def search(hist, rows, cfg, num_bins):
    sums = (float(hist[0::2].sum()), float(hist[1::2].sum()), int(rows.sum()))
    return orc.find_best_split(one_feature(num_bins), hist, [1], sums, (1.0, 1.0), cfg)


def test_onehot_matches_brute_force(oracle):
    rng = Lcg(3)
    for case in range(200):
        num_bins = 2 + rng.below(3)
        hist, rows = random_hist(rng, num_bins, 1.0)
        cfg = config()
        info, _ = search(hist, rows, cfg, num_bins)
        expected = brute_force(hist, rows, cfg, cfg.lambda_l2, [lambda b, t=t: b == t for t in range(1, num_bins)])
        name = f"onehot case {case}"
        if not info.found:
            assert expected == MIN_SCORE, f"{name}: brute force found a split"
            continue
        assert_close(info.gain, expected, name)
        assert info.categorical == 1 and len(left_bins(info)) == 1, f"{name}: one category"
        check_children(info, hist, rows, cfg, name)


def test_sorted_categorical_matches_brute_force(oracle):
    rng = Lcg(5)
    found = 0
    for case in range(200):
        num_bins = 6 + rng.below(12)
        hist, rows = random_hist(rng, num_bins, 1.0)
        cfg = config(min_data_per_group=1, cat_smooth=1.0, max_cat_threshold=4)
        info, _ = search(hist, rows, cfg, num_bins)
        ctr = {t: hist[2 * t] / (hist[2 * t + 1] + cfg.cat_smooth) for t in range(num_bins)}
        ordered = sorted((t for t in range(1, num_bins) if rows[t] >= cfg.cat_smooth), key=lambda t: ctr[t])
        used = len(ordered)
        max_cat = min(cfg.max_cat_threshold, (used + 1) // 2)
        candidates = []
        for k in range(1, min(max_cat, used) + 1):
            low, high = set(ordered[:k]), set(ordered[used - k:])
            candidates += [lambda b, s=low: b in s, lambda b, s=high: b in s]
        cat_l2 = cfg.lambda_l2 + cfg.cat_l2
        tg, th = hist[0::2].sum(), hist[1::2].sum()
        # the gain shift keeps the plain l2 while the candidates use cat_l2, as in LightGBM
        shift_fix = leaf_gain(tg, th, 0.0, cat_l2) - leaf_gain(tg, th, 0.0, cfg.lambda_l2)
        expected = brute_force(hist, rows, cfg, cat_l2, candidates)
        if expected != MIN_SCORE:
            expected += shift_fix
        name = f"sorted case {case}"
        if not info.found:
            assert expected <= 0.0, f"{name}: brute force found {expected}"
            continue
        found += 1
        assert_close(info.gain, expected, name)
        check_children(info, hist, rows, cfg, name)
        assert 0 not in left_bins(info), f"{name}: bin 0 never goes left"
    assert found > 50, f"only {found} sorted cases split"


def raw_rows(data: BinnedDataset, bins: np.ndarray) -> np.ndarray:
    """Raw feature values that bin to `bins`: a categorical bin's category (bin 0: -1), a numerical bin's index."""
    out = np.zeros(bins.shape, dtype=np.float64)
    for f, m in enumerate(data.features):
        if m.kind == _abi.CATEGORICAL:
            lut = np.array([-1] + m.categories, dtype=np.float64)
            out[:, f] = lut[bins[:, f]]
        else:
            out[:, f] = bins[:, f]
    return out


def test_training_grows_categorical_splits(oracle):
    data = categorical_binned(20_000)
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=15, num_iterations=4, min_data_per_group=20)
    model = orc.train([data], p)
    kinds = [int(d) & 1 for t in model.trees for d in t.decision_type]
    assert any(kinds), "no categorical split"
    # the model file's categorical splits predict as the binned trees route the rows
    from silvic_b200 import model_text

    text = model_text.from_trained(Model(model.trees, model.init_score, []), data, p)
    parsed = model_text.TextModel.from_string(text.to_string())
    bins = np.stack([data.groups[0].data[:, m.column] for m in data.features], axis=1)[:300]
    raw = raw_rows(data, bins)
    for row in range(300):
        want = 0.0
        for t in model.trees:
            node = 0 if t.num_leaves > 1 else -1
            while node >= 0:
                f = int(t.split_feature[node])
                b = int(bins[row, f])
                if int(t.decision_type[node]) & 1:
                    left = bool((int(t.cat_bins[node][b // 32]) >> (b % 32)) & 1)
                else:
                    left = b <= int(t.threshold_bin[node])
                node = int(t.left_child[node] if left else t.right_child[node])
            want += float(t.leaf_value[~node])
        assert parsed.predict_raw_row(raw[row]) == want, row


def test_two_ranks_train_the_categorical_model_of_one(oracle):
    """train_cpu.rs:270-286 with categorical features: shards of the rows train the one-rank trees."""
    data = categorical_binned(8_000, seed=4, label_kind="binary")
    p = orc.default_params(objective=_abi.BINARY, num_leaves=15, num_iterations=3, min_data_per_group=20)
    one = orc.train([data], p)
    two = orc.train([data.shard(0, 3_000), data.shard(3_000, 8_000)], p)
    assert any(int(d) & 1 for t in one.trees for d in t.decision_type), "no categorical split"
    for k, (a, b) in enumerate(zip(one.trees, two.trees)):
        assert orc.trees_equal(a, b) == [], f"tree {k}"
