"""The oracle against the reference's own unit tests and properties (no GPU).

Ports: quantize.rs:167-216 (uniform, unbiased stochastic rounding, pack round trip, constant hessian, fixed-point
scale), backend/cpu.rs:1014-1121 (histogram == direct sums with bagging and masks; packed flush before i32
overflow; stable partition), split.rs:1151-1235 (numerical scan == brute force), learner.rs:691-722 and
tests/train_cpu.rs:250-286 (max_depth; two ranks grow the tree of one; identical runs)."""

from __future__ import annotations

import math

import numpy as np
import pytest

from silvic_b200 import _abi
import oracle_lib as orc
from synth import mix32, random_binned


def py_mix32(x: int) -> int:
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return x


def test_mix32_known_answers(oracle):
    # lowbias32 from its published constants, computed in Python.
    for x in [0, 1, 2, 0xDEADBEEF, 0xFFFFFFFF, 12345]:
        assert oracle.lib().orc_mix32(x) == py_mix32(x)
    assert int(mix32(np.array([7], dtype=np.uint32))[0]) == py_mix32(7)


def test_uniform_is_in_unit_interval_and_row_keyed(oracle):
    draws = np.array([oracle.lib().orc_uniform(7, 0, 3, r) for r in range(10_000)])
    assert np.all((draws >= 0) & (draws < 1))
    assert abs(draws.mean() - 0.5) < 0.02
    assert oracle.lib().orc_uniform(7, 0, 3, 1 << 32) != oracle.lib().orc_uniform(7, 0, 3, 0)
    # the same hash written out in Python
    for r in [0, 5, 1 << 33]:
        rh = py_mix32((r & 0xFFFFFFFF) ^ py_mix32(r >> 32))
        h = py_mix32(7 ^ py_mix32(0 ^ py_mix32(3 ^ rh)))
        assert oracle.lib().orc_uniform(7, 0, 3, r) == np.float32(h >> 8) * np.float32(1.0 / 16777216.0)


def test_stochastic_rounding_is_unbiased(oracle):
    spec = oracle.quant_spec(2.0, 1.0, None, 4, True, 11, 0)
    n = 200_000
    packed = oracle.quantize(spec, np.full(n, 0.3, np.float32), np.full(n, 0.5, np.float32))
    g, _ = oracle.unpack(packed)
    assert abs(g.sum() / n * spec.grad_scale - 0.3) < 0.01


def test_pack_round_trips_negative_gradients(oracle):
    for g in range(-32, 33):
        for h in range(0, 65):
            gg, hh = _abi_unpack(oracle, h * 65536 + g)
            assert (gg, hh) == (g, h)


def _abi_unpack(oracle, packed):
    import ctypes as C

    g, h = C.c_int32(), C.c_int32()
    oracle.lib().orc_unpack(packed, C.byref(g), C.byref(h))
    return g.value, h.value


def test_constant_hessian_counts_rows(oracle):
    spec = oracle.quant_spec(1.0, 1.0, 1.0, 4, True, 1, 0)
    packed = oracle.quantize(spec, np.array([-0.7], np.float32), np.array([1.0], np.float32), row_offset=5)
    assert oracle.unpack(packed)[1][0] == 1


def test_fixed_point_scale_bounds_magnitude(oracle):
    scale = oracle.lib().orc_fixed_point_scale(3.7)
    assert float(np.float32(3.7) * np.float32(scale)) <= 2.0**30
    assert float(np.float32(3.7) * np.float32(scale)) > 2.0**29
    assert oracle.lib().orc_fixed_point_scale(0.0) == 1.0
    # powers of two and their neighbours
    for x in [1.0, 2.0, 0.5, float(np.nextafter(np.float32(2), np.float32(3))), 1e-3, 123.0]:
        e = 30 - math.ceil(math.log2(x))
        assert oracle.lib().orc_fixed_point_scale(x) == 2.0 ** max(-126, min(127, e))


def naive_hist(data, packed, rows):
    g, h = orc.unpack(packed)
    out = np.zeros(2 * data.total_bins)
    for f, m in enumerate(data.features):
        if m.num_bins == 0:
            continue
        idx = m.hist_offset + data.feature_bins(f)[rows].astype(np.int64)
        np.add.at(out, 2 * idx, g[rows])
        np.add.at(out, 2 * idx + 1, h[rows])
    return out


def test_histograms_match_direct_sums(oracle):
    data = random_binned(50_000, [7, 3, 5], seed=2)
    r = np.arange(data.num_rows)
    grad = (r % 13).astype(np.float32) / 4.0 - 1.5
    hess = 0.25 + (r % 5).astype(np.float32) / 8.0
    spec = oracle.quant_spec(1.5, 0.75, None, 16, True, 9, 3)
    packed = oracle.quantize(spec, grad, hess, row_offset=100)
    part = oracle.reset_partition(_abi.BagSpec(1, 4, 1, 0, 0.7), data.num_rows, 100)
    assert 0.65 < len(part) / data.num_rows < 0.75
    rows = part[1000:31_000]
    got = oracle.histogram(data, packed, rows, max_quant=16)
    assert np.array_equal(got, naive_hist(data, packed, rows))
    for used in ([1, 0, 1], [0, 1, 0], [0, 0, 1]):
        got = oracle.histogram(data, packed, rows, used=np.array(used, np.uint8), max_quant=16)
        want = naive_hist(data, packed, rows)
        for f, m in enumerate(data.features):
            if used[f]:
                sl = slice(2 * m.hist_offset, 2 * (m.hist_offset + m.num_bins))
                assert np.array_equal(got[sl], want[sl])


def test_packed_accumulators_flush_before_overflow(oracle):
    data = random_binned(400_000, [7, 3, 5], seed=3)
    packed = np.full(data.num_rows, 3 * 65536 - 32000, dtype=np.int32)
    rows = np.arange(data.num_rows)
    got = oracle.histogram(data, packed, rows, max_quant=(2**31 - 1) // 1000)
    assert np.array_equal(got, naive_hist(data, packed, rows))
    assert np.any(got[0::2] < -(2.0**31)), "sums leave i32"


def test_partition_is_stable(oracle):
    data = random_binned(30_000, [7, 3, 5], seed=4)
    split = _abi.BinSplit()
    split.group, split.column = 0, 0
    split.left_bins[0] = 0b10110
    left, rows = oracle.partition(data, split, np.arange(500, 25_500))
    goes = lambda r: (0b10110 >> data.bin(0, r)) & 1  # noqa: E731
    exp_left = [r for r in range(500, 25_500) if goes(r)]
    exp_right = [r for r in range(500, 25_500) if not goes(r)]
    assert left == len(exp_left)
    assert list(rows[:left]) == exp_left and list(rows[left:]) == exp_right


# ---- split search vs brute force (split.rs:1151-1235) ----

def leaf_gain(g, h, l1, l2):
    r = max(abs(g) - l1, 0.0)
    return r * r / (h + l2)


def brute_force(hist, rows, nan_bin, cfg, scale):
    """The best gain - shift over every numerical split the rules allow, by direct summation of real sums."""
    nb = len(rows)
    G = hist[0::2] * scale[0]
    H = hist[1::2] * scale[1]
    tg, th, tn = G.sum(), H.sum(), rows.sum()
    shift = leaf_gain(tg, th, cfg.lambda_l1, cfg.lambda_l2) + cfg.min_gain_to_split
    numeric = nb - int(nan_bin)
    end = numeric if nan_bin else numeric - 1
    best = -math.inf
    for t in range(end):
        for nan_left in (False, True):
            left = np.array([(nan_left if b == numeric else b <= t) for b in range(nb)])
            lg, lh, ln = G[left].sum(), H[left].sum(), rows[left].sum()
            rg, rh, rn = tg - lg, th - lh, tn - ln
            ok = lambda n, h: n >= cfg.min_data_in_leaf and n > 0 and h >= cfg.min_sum_hessian_in_leaf and h > 0  # noqa
            if not ok(ln, lh) or not ok(rn, rh):
                continue
            gain = leaf_gain(lg, lh, cfg.lambda_l1, cfg.lambda_l2) + leaf_gain(rg, rh, cfg.lambda_l1, cfg.lambda_l2)
            if gain > shift:
                best = max(best, gain - shift)
    return best


@pytest.mark.parametrize("case", range(60))
def test_numerical_matches_brute_force(oracle, case):
    rng = np.random.default_rng(case)
    nan_bin = case % 2 == 1
    nb = int(rng.integers(3 if nan_bin else 2, 32))
    data = random_binned(16, [nb], nan_bins=[nan_bin], seed=case)
    rows = rng.integers(0, 40, size=nb)
    hist = np.zeros(2 * nb)
    hist[0::2] = np.round((rng.random(nb) - 0.45) * rows * 4)  # integer units
    hist[1::2] = rows * 1.0  # one hessian unit per row: count estimates are exact
    cfg = _abi.SplitConfig(5, 1e-3, 0.5 if case % 3 == 0 else 0.0, 2.0 if case % 5 == 0 else 0.0, 0.0)
    scale = (0.25, 1.0)
    info, spl = oracle.find_best_split(data, hist, [1], (hist[0::2].sum(), hist[1::2].sum(), int(rows.sum())),
                                       scale, cfg)
    expected = brute_force(hist, rows, nan_bin, cfg, scale)
    if info.found:
        assert abs(info.gain - expected) <= 1e-9 * max(abs(expected), 1.0), (info.gain, expected)
        assert spl[0] == 1
    else:
        assert expected == -math.inf
        assert spl[0] == 0


def test_ties_go_to_the_lower_feature(oracle):
    # Two identical features: the split must be on feature 0 (split.rs:1474).
    data = random_binned(16, [6, 6], seed=1)
    one = np.array([3, -5, 2, 8, -1, 0], dtype=np.float64)
    hist = np.zeros(24)
    for f in range(2):
        hist[12 * f:12 * f + 12:2] = one
        hist[12 * f + 1:12 * f + 12:2] = 10.0
    cfg = _abi.SplitConfig(1, 1e-3, 0.0, 0.0, 0.0)
    info, _ = oracle.find_best_split(data, hist, [1, 1], (one.sum(), 60.0, 60), (1.0, 1.0), cfg)
    assert info.found and info.feature == 0


# ---- learner and trainer properties ----

def test_max_depth_limits_growth(oracle):
    data = random_binned(3000, [8, 5, 6], seed=2)
    m = oracle.train([data], orc.default_params(max_depth=2, num_leaves=31, num_iterations=1, min_data_in_leaf=5))
    t = m.trees[0]
    assert t.num_leaves == 4


def test_two_ranks_grow_the_tree_of_one(oracle):
    data = random_binned(4000, [8, 5, 6], seed=3)
    # integer labels sum exactly in any order, so the init score is the same over ranks too
    data.label[:] = np.round(data.label * 4)
    p = orc.default_params(num_leaves=8, num_iterations=3, min_data_in_leaf=5)
    single = oracle.train([data], p)
    ranks = oracle.train([data.shard(0, 1500), data.shard(1500, 4000)], p)
    assert len(single.trees) == len(ranks.trees) == 3
    for a, b in zip(single.trees, ranks.trees):
        assert orc.trees_equal(a, b) == []


def test_identical_runs_identical_trees(oracle):
    data = random_binned(5000, [16] * 6, seed=4)
    p = orc.default_params(num_leaves=15, num_iterations=4)
    a, b = oracle.train([data], p), oracle.train([data], p)
    for x, y in zip(a.trees, b.trees):
        assert orc.trees_equal(x, y) == []


def test_training_reduces_l2(oracle):
    data = random_binned(8000, [32] * 6, seed=5)
    p = orc.default_params(num_leaves=15, num_iterations=20)
    m = oracle.train([data], p)
    from silvic_b200.backend import Model

    model = Model(m.trees, m.init_score, [])
    raw = np.array([[data.features[f].upper_bounds[min(data.bin(f, r), len(data.features[f].upper_bounds) - 1)] - 0.25
                     for f in range(6)] for r in range(500)])
    pred = np.array([model.predict_raw_row(raw[r]) for r in range(500)])
    mse = float(np.mean((pred - data.label[:500]) ** 2))
    base = float(np.mean((data.label[:500] - data.label.mean()) ** 2))
    assert mse < 0.5 * base
