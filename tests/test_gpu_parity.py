"""Device vs oracle, bit for bit, through the C ABI: each Backend operation, the split search and whole training
runs. Patterned on the reference's device-parity suite (crates/silvic-gpu/tests/metal_backend.rs:391-748) and
CpuBackend tests (crates/silvic-core/src/backend/cpu.rs:1014-1179)."""

from __future__ import annotations

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend, init_score
import oracle_lib as orc
from synth import nested_binned, random_binned

pytestmark = pytest.mark.gpu


def loaded(data, objective=_abi.REGRESSION, sigmoid=1.0):
    b = B200Backend(0)
    b.load(data, objective, sigmoid)
    return b


def set_gradients(b, data, seed=0):
    n = data.num_rows
    r = np.arange(n)
    grad = ((r * 7 + seed) % 13).astype(np.float32) / 4.0 - 1.5
    hess = 0.25 + ((r + seed) % 5).astype(np.float32) / 8.0
    b.write_gradients(grad, hess)
    return grad, hess


SHAPES = [
    ([7, 3, 5], 50_000),
    ([255] * 28, 60_000),
    ([255] * 70 + [64] * 30, 40_000),
    ([63] * 40 + [2, 3, 200], 30_000),
    # units of two and of four full tiles (row-chunk loads of 64- and 128-byte unit rows), then a unit of one
    ([255] * 64 + [31] * 2, 30_000),
    ([255] * 128 + [15] * 160, 20_000),
]


@pytest.mark.parametrize("bins,rows", SHAPES)
@pytest.mark.parametrize("quant_bins", [4, 16])
def test_histogram_matches_oracle(device, bins, rows, quant_bins):
    data = random_binned(rows, bins, seed=len(bins))
    b = loaded(data)
    grad, hess = set_gradients(b, data)
    spec = orc.quant_spec(1.5, 0.75, None, quant_bins, True, 9, 3)
    b.quantize(spec)
    packed = b.read_packed()
    assert np.array_equal(packed, orc.quantize(spec, grad, hess)), "quantize"
    n = b.reset_partition(_abi.BagSpec(1, 4, 1, 0, 0.7))
    part = b.read_partition(n)
    assert np.array_equal(part, orc.reset_partition(_abi.BagSpec(1, 4, 1, 0, 0.7), rows)), "bag"
    for begin, count in [(0, n), (1000, n // 3), (n - 77, 77), (5, 0)]:
        got = b.histogram(begin, count)
        want = orc.histogram(data, packed, part[begin:begin + count], max_quant=quant_bins)
        assert np.array_equal(got, want), f"leaf {begin}+{count}"
    rng = np.random.default_rng(3)
    for _ in range(3):
        used = (rng.random(len(bins)) < 0.5).astype(np.uint8)
        b.set_histogram_features(used)
        got = b.histogram(100, n - 200)
        want = orc.histogram(data, packed, part[100:n - 100], used=used, max_quant=quant_bins)
        for f, m in enumerate(data.features):
            if used[f]:
                sl = slice(2 * m.hist_offset, 2 * (m.hist_offset + m.num_bins))
                assert np.array_equal(got[sl], want[sl]), f"mask feature {f}"
    b.close()


@pytest.mark.parametrize("quant_bins,rows", [(64, 400_000), (512, 60_000)],
                         ids=["packed_rounds", "wide_quantization"])
def test_histogram_packing_limits(device, quant_bins, rows):
    """Histograms whose packed per-bin sums would pass 16 bits within one CTA: 64 quant bins over 400k rows make
    every CTA flush its packed shared histogram several times (sums exact while |g| <= 32767, h <= 65535 per
    round); 512 quant bins are too wide for packed rounds and go straight to the output."""
    data = random_binned(rows, [255] * 6 + [16] * 3, seed=quant_bins)
    b = loaded(data)
    grad, hess = set_gradients(b, data, seed=4)
    spec = orc.quant_spec(1.5, 0.75, None, quant_bins, True, 9, 3)
    b.quantize(spec)
    packed = b.read_packed()
    assert np.array_equal(packed, orc.quantize(spec, grad, hess)), "quantize"
    n = b.reset_partition(_abi.BagSpec(1, 4, 1, 0, 0.9))
    part = b.read_partition(n)
    for begin, count in [(0, n), (n // 3, n // 2)]:
        got = b.histogram(begin, count)
        want = orc.histogram(data, packed, part[begin:begin + count], max_quant=quant_bins)
        assert np.array_equal(got, want), f"leaf {begin}+{count}"
    b.close()


def test_identity_root_histogram(device):
    data = random_binned(100_003, [255] * 33, seed=5)
    b = loaded(data)
    grad, hess = set_gradients(b, data, seed=2)
    spec = orc.quant_spec(1.5, 0.75, None, 4, True, 1, 0)
    b.quantize(spec)
    n = b.reset_partition()
    assert n == data.num_rows
    got = b.histogram(0, n)
    want = orc.histogram(data, b.read_packed(), np.arange(n))
    assert np.array_equal(got, want)
    b.close()


def test_partition_is_stable_and_matches_oracle(device):
    data = random_binned(30_000, [7, 3, 5], seed=1)
    b = loaded(data)
    set_gradients(b, data)
    b.quantize(orc.quant_spec(1.5, 0.75, None, 4, True, 1, 0))
    b.reset_partition()
    split = _abi.BinSplit()
    split.group, split.column = 0, 0
    split.left_bins[0] = 0b10110
    left = b.partition(500, 25_000, split)
    part = b.read_partition()
    ref_left, ref_rows = orc.partition(data, split, np.arange(500, 25_500))
    assert left == ref_left
    assert np.array_equal(part[500:25_500], ref_rows)
    assert np.array_equal(part[:500], np.arange(500)), "rows before the leaf"
    # partition_and_histogram of the right child
    split2 = _abi.BinSplit()
    split2.group, split2.column = 0, 2
    split2.left_bins[0] = 0b11
    packed = b.read_packed()
    left2, hist = b.partition_and_histogram(500, left, split2, _abi.RIGHT)
    part = b.read_partition()
    l2, rows2 = orc.partition(data, split2, ref_rows[:left])
    assert left2 == l2
    assert np.array_equal(part[500:500 + left], rows2)
    assert np.array_equal(hist, orc.histogram(data, packed, rows2[l2:]))
    b.close()


def test_gradients_leaf_sums_and_add_tree(device):
    data = random_binned(20_000, [7, 3, 5], seed=3, label_kind="binary")
    for objective, sigmoid in [(_abi.REGRESSION, 1.0), (_abi.BINARY, 1.5)]:
        b = loaded(data, objective, sigmoid)
        scores = (np.arange(data.num_rows) % 17 - 8).astype(np.float32) / 7.0
        b.init_scores(0, 0.0)
        # scores through add_tree of a one-leaf tree would be constant; write them through a two-node tree instead
        split = _abi.BinSplit()
        split.group, split.column = 0, 2
        split.left_bins[0] = 0b11
        nodes = [_abi.DeviceNode(split, ~0, ~1)]
        b.add_tree(nodes, [0.5, -0.25])
        got_scores = b.scores()
        want_scores = orc.add_tree(data, nodes, [0.5, -0.25], np.zeros(data.num_rows, dtype=np.float32))
        assert np.array_equal(got_scores, want_scores), "add_tree"
        mg, mh = b.compute_gradients()
        g, h = b.read_gradients()
        wg, wh = orc.gradients(objective, want_scores, data.label, sigmoid=sigmoid)
        mism = int(np.sum(g.view(np.uint32) != wg.view(np.uint32)) + np.sum(h.view(np.uint32) != wh.view(np.uint32)))
        if objective == _abi.REGRESSION:
            assert mism == 0
        else:
            assert mism <= data.num_rows // 1000, f"{mism} binary gradient bits differ"
        assert mg == float(np.max(np.abs(g))) and mh == float(np.max(np.abs(h)))
        b.reset_partition()
        leaves = [(0, 7000), (7000, 13_000)]
        got = b.leaf_sums(leaves, 1024.0, 256.0)
        want = orc.leaf_sums(g, h, b.read_partition(), leaves, 1024.0, 256.0)
        assert np.array_equal(got, want)
        b.close()


def random_hist(rng, data, hess_per_row=0.25):
    """Integer-valued quantized histograms (units) with positive hessians."""
    h = np.zeros(2 * data.total_bins)
    for m in data.features:
        for k in range(m.num_bins):
            n = int(rng.integers(0, 40))
            h[2 * (m.hist_offset + k)] = float(rng.integers(-2 * n, 2 * n + 1))
            h[2 * (m.hist_offset + k) + 1] = float(n * 4)
    return h


@pytest.mark.parametrize("case", range(12))
def test_split_search_matches_oracle(device, case):
    rng = np.random.default_rng(100 + case)
    nb = [int(x) for x in rng.integers(2, 256, size=int(rng.integers(1, 60)))]
    nan = [bool(x) for x in rng.integers(0, 2, size=len(nb))]
    data = random_binned(64, nb, nan_bins=nan, seed=case)
    b = loaded(data)
    hist = random_hist(rng, data)
    m0 = data.features[0]
    g0 = hist[2 * m0.hist_offset: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    h0 = hist[2 * m0.hist_offset + 1: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    count = int(h0 // 4)
    cfg = _abi.SplitConfig(int(rng.integers(0, 30)), [1e-3, 0.0, 0.5][case % 3], [0.0, 0.5][case % 2],
                           [0.0, 2.0, 10.0][case % 3], [0.0, 0.1][case % 2])
    evaluate = (rng.random(len(nb)) < 0.8).astype(np.uint8)
    scale = (0.37 + case, 0.25)
    got, gs = b.find_best_split(hist, evaluate, (g0, h0, count), scale, cfg)
    want, ws = orc.find_best_split(data, hist, evaluate, (g0, h0, count), scale, cfg)
    assert got.as_tuple() == want.as_tuple()
    assert np.array_equal(gs, ws)
    b.close()


def test_split_division_is_correctly_rounded(device):
    """The split scan's FMA division equals CUDA's correctly rounded division bit for bit (so the gains equal the
    CPU's IEEE divisions) on 2^27 hashed operand pairs: random and awkward mantissas, exact quotients, zero
    numerators, and operands outside its fast range."""
    import ctypes as C

    b = B200Backend(0)
    try:
        for seed in (1, 20261107):
            bad = C.c_uint64()
            b._check(b._lib.sb2_check_division(b._h, 1 << 27, seed, C.byref(bad)))
            assert bad.value == 0, f"seed {seed}: {bad.value} mismatches"
    finally:
        b.close()


TRAIN_CASES = [
    ("l2_small", [255] * 10 + [17, 2], 20_000, dict(objective=_abi.REGRESSION, num_leaves=31, num_iterations=8)),
    ("l2_depth", [63] * 12, 15_000, dict(objective=_abi.REGRESSION, num_leaves=63, max_depth=4, num_iterations=5)),
    ("binary", [255] * 20, 25_000, dict(objective=_abi.BINARY, num_leaves=63, num_iterations=6)),
    ("l2_reg", [31] * 40, 12_000, dict(objective=_abi.REGRESSION, num_leaves=15, lambda_l1=0.5, lambda_l2=2.0,
                                        min_data_in_leaf=50, num_iterations=6, feature_fraction=0.6,
                                        num_grad_quant_bins=16)),
    ("l2_nan", [40] * 8, 10_000, dict(objective=_abi.REGRESSION, num_leaves=20, num_iterations=4)),
    # more features than CTAs (several per CTA in the search) and several histogram units
    ("wide", [255] * 60 + [15] * 140, 6_000, dict(objective=_abi.REGRESSION, num_leaves=31, num_iterations=3)),
]


@pytest.mark.parametrize("name,bins,rows,params", TRAIN_CASES, ids=[c[0] for c in TRAIN_CASES])
def test_training_matches_oracle(device, name, bins, rows, params):
    nan = [True] * len(bins) if name == "l2_nan" else None
    data = random_binned(rows, bins, nan_bins=nan, seed=11, label_kind="binary" if "binary" in name else "regression")
    p = orc.default_params(**params)
    ref = orc.train([data], p)
    b = loaded(data, p.objective, p.sigmoid)
    model = b.train(p, init_score(p, data.label))
    b.close()
    assert model.init_score == ref.init_score
    assert len(model.trees) == len(ref.trees)
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
    # the emitted model file is the oracle model's, byte for byte (silvic_b200.model_text, pinned on LightGBM's
    # files in test_model_text.py)
    from silvic_b200.backend import Model

    assert model.to_lightgbm_string(data, p) == Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)


def test_speculative_splits_drop_and_match_oracle(device):
    """The tree kernel runs the next leaves' splits beside the best one's and drops those a fresh child outranks,
    keeping their work for the step that commits them. On data where the best leaf is often a child of the last
    split, some grid steps drop splits and later ones commit them ready; the trees stay the oracle's, and the last
    tree's committed splits are its leaves (the root counts one)."""
    data = nested_binned(20_000)
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=31, num_iterations=3)
    ref = orc.train([data], p)
    b = loaded(data, p.objective, p.sigmoid)
    s0 = init_score(p, data.label)
    model = b.train(p, s0)
    steps = b.profile_steps(p, s0)
    b.close()
    assert len(model.trees) == len(ref.trees)
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
    fields = B200Backend.STEP_FIELDS
    splits = int(steps[:, fields.index("splits")].sum())
    committed = int(steps[:, fields.index("committed")].sum())
    kept = int(steps[:, fields.index("kept")].sum())
    assert committed == ref.trees[-1].num_leaves
    # every committed split ran once, here or in the step that dropped it and kept its work
    assert splits - (committed - kept) > 0, "no speculative split was dropped"
    assert kept <= splits - (committed - kept)
    assert kept > 0, "no dropped split was committed from its kept work"
