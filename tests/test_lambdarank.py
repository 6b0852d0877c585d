"""The oracle's lambdarank objective against the reference's own tests of it
(crates/silvic-core/src/objective/lambdarank.rs:398-783), ported: gradients equal a line-by-line transcription of
LightGBM 3.3.5's GetGradientsForOneQuery pair loop (sigmoid 1.3, ties, weights, truncation levels, norm on and off)
within the reference's tolerance, items with a -inf score get no pairs, the sigmoid table follows LightGBM's
ConstructSigmoidTable/GetSigmoid exactly, max DCG and the label checks follow DCGCalculator."""

from __future__ import annotations

import math

import numpy as np
import pytest

import oracle_lib as orc


def default_label_gain():
    return [float((1 << i) - 1) for i in range(31)]


def discount(rank: int) -> float:
    return 1.0 / math.log2(2.0 + rank)


def lightgbm_pair_loop(label, score, weight, label_gain, inverse_max_dcg, sigmoid, norm, truncation_level):
    """LightGBM 3.3.5 GetGradientsForOneQuery and RankingObjective::GetGradients' weight loop, transcribed as the
    reference's test does (lambdarank.rs:443-510): f64 sums, the pair loop's order, the sigmoid table."""
    cnt = len(label)
    score = [float(s) for s in score]
    lambdas, hessians = [0.0] * cnt, [0.0] * cnt
    order = sorted(range(cnt), key=lambda r: -score[r])  # stable: ties keep row order
    best = score[order[0]]
    worst_idx = cnt - 1
    if worst_idx > 0 and score[order[worst_idx]] == -math.inf:
        worst_idx -= 1
    worst = score[order[worst_idx]]
    sum_lambdas = 0.0
    i = 0
    while i + 1 < cnt and i < truncation_level:
        if score[order[i]] == -math.inf:
            i += 1
            continue
        for j in range(i + 1, cnt):
            if score[order[j]] == -math.inf or label[order[i]] == label[order[j]]:
                continue
            hr, lr = (i, j) if label[order[i]] > label[order[j]] else (j, i)
            high, low = order[hr], order[lr]
            delta_score = score[high] - score[low]
            dcg_gap = label_gain[int(label[high])] - label_gain[int(label[low])]
            paired = abs(discount(hr) - discount(lr))
            dpn = dcg_gap * paired * inverse_max_dcg
            if norm and best != worst:
                dpn /= float(np.float32(0.01)) + abs(delta_score)
            p_lambda = orc.lambdarank_sigmoid(sigmoid, delta_score)
            p_hessian = p_lambda * (1.0 - p_lambda)
            p_lambda *= -sigmoid * dpn
            p_hessian *= sigmoid * sigmoid * dpn
            lambdas[low] -= p_lambda
            hessians[low] += p_hessian
            lambdas[high] += p_lambda
            hessians[high] += p_hessian
            sum_lambdas -= 2.0 * p_lambda
        i += 1
    if norm and sum_lambdas > 0.0:
        f = math.log2(1.0 + sum_lambdas) / sum_lambdas
        lambdas = [v * f for v in lambdas]
        hessians = [v * f for v in hessians]
    if weight is not None:
        lambdas = [v * float(w) for v, w in zip(lambdas, weight)]
        hessians = [v * float(w) for v, w in zip(hessians, weight)]
    return lambdas, hessians


def assert_close(what, got, want):
    """The reference's tolerance (lambdarank.rs:565-575): f32 storage rounds at 6e-8 relative."""
    scale = max((abs(v) for v in want), default=0.0)
    for row, (g, w) in enumerate(zip(got, want)):
        tol = 1e-6 * max(abs(w), scale * 1e-3) + 1e-30
        assert abs(float(g) - w) <= tol, f"{what} of row {row}: {g} vs {w}"


def params(norm=True, truncation_level=30, sigmoid=1.3):
    return orc.default_params(objective=2, sigmoid=sigmoid, lambdarank_norm=int(norm),
                              lambdarank_truncation_level=truncation_level)


def one_query(label, score, weight, norm, trunc, sigmoid=1.3):
    grad, hess = orc.lambdarank_gradients(params(norm, trunc, sigmoid), label, score, [0, len(label)], weight)
    gain = default_label_gain()
    m = orc.lambdarank_max_dcg(trunc, label, gain)
    want_g, want_h = lightgbm_pair_loop(label, score, weight, gain, 1.0 / m if m > 0 else 0.0, sigmoid, norm, trunc)
    return grad, hess, want_g, want_h


def test_gradients_match_lightgbm_pair_loop():
    rng = np.random.default_rng(0x9E3779B9)
    for index in range(400):
        cnt = 1 + int(rng.integers(60))
        label = rng.integers(0, 5, size=cnt).astype(np.float32)
        if index % 4 == 0:
            score = np.zeros(cnt, dtype=np.float32)  # every score tied: only row order ranks
        elif index % 4 == 1:
            score = (rng.integers(0, 4, size=cnt) * 0.5).astype(np.float32)  # partial ties
        else:
            score = ((rng.random(cnt, dtype=np.float32) - 0.5) * 8.0).astype(np.float32)
        weight = (0.5 + rng.random(cnt, dtype=np.float32)).astype(np.float32) if index % 3 == 0 else None
        trunc = [1, 3, 10, 30, 1000][index % 5]
        norm = index % 7 != 6
        grad, hess, want_g, want_h = one_query(label, score, weight, norm, trunc)
        assert_close(f"case {index} gradient", grad, want_g)
        assert_close(f"case {index} hessian", hess, want_h)


def test_queries_are_independent():
    """Several queries in one call: each equals its own single-query gradients."""
    rng = np.random.default_rng(5)
    sizes = [7, 1, 30, 12]
    qb = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)
    label = rng.integers(0, 5, size=qb[-1]).astype(np.float32)
    score = rng.normal(size=qb[-1]).astype(np.float32)
    grad, hess = orc.lambdarank_gradients(params(), label, score, qb)
    for q in range(len(sizes)):
        b, e = qb[q], qb[q + 1]
        g1, h1 = orc.lambdarank_gradients(params(), label[b:e], score[b:e], [0, e - b])
        assert np.array_equal(grad[b:e], g1) and np.array_equal(hess[b:e], h1)


def test_min_score_items_get_no_pairs():
    label = np.array([2.0, 0.0, 1.0, 0.0], dtype=np.float32)
    score = np.array([0.5, -np.inf, -0.2, 0.1], dtype=np.float32)
    grad, hess, want_g, want_h = one_query(label, score, None, True, 30)
    assert (grad[1], hess[1]) == (0.0, 0.0)
    assert_close("min score gradient", grad, want_g)
    assert_close("min score hessian", hess, want_h)


def test_sigmoid_table_follows_lightgbm():
    sigmoid = 2.0
    lo, hi = -50.0 / sigmoid / 2.0, 50.0 / sigmoid / 2.0
    factor = (1024.0 * 1024.0) / (hi - lo)

    def entry(i):
        return 1.0 / (1.0 + math.exp((i / factor + lo) * sigmoid))

    def want(x):
        if x <= lo:
            return entry(0)
        if x >= hi:
            return entry(1024 * 1024 - 1)
        return entry(int((x - lo) * factor))

    for x in [-100.0, lo, -3.7, -1e-9, 0.0, 1e-9, 0.25, 4.0, hi - 1e-12, hi, 30.0]:
        assert orc.lambdarank_sigmoid(sigmoid, x) == want(x), x
    assert abs(orc.lambdarank_sigmoid(sigmoid, 0.0) - 0.5) < 1e-4


def test_max_dcg_follows_lightgbm():
    gain = [0.0, 1.0, 3.0, 7.0]
    labels = [1.0, 3.0, 0.0, 2.0, 3.0]
    assert orc.lambdarank_max_dcg(3, labels, gain) == 7.0 * discount(0) + 7.0 * discount(1) + 3.0 * discount(2)
    assert orc.lambdarank_max_dcg(3, [0.0, 0.0], gain) == 0.0
    assert orc.lambdarank_max_dcg(10, [1.0], gain) == 1.0


@pytest.mark.parametrize("labels", [[0.0, 31.0], [0.5], [-1.0]])
def test_rank_labels_are_checked(labels):
    with pytest.raises(ValueError, match="lambdarank label"):
        orc.lambdarank_gradients(params(), labels, [0.0] * len(labels), [0, len(labels)])


def test_queries_must_cover_the_rows():
    with pytest.raises(ValueError, match="query information"):
        orc.lambdarank_gradients(params(), [0.0, 1.0, 2.0], [0.0] * 3, [0, 2])


def test_two_ranks_train_the_lambdarank_model_of_one():
    """Ranks hold whole queries: two shards cut at a query boundary train the one-rank model (the reference's
    two_ranks_train_the_model_of_one, crates/silvic-core/tests/train_cpu.rs:270-286, for the ranking objective)."""
    from synth import ranking_binned

    data = ranking_binned(6_000, [63] * 5 + [255], seed=4, mean_query=50.0)
    p = params()
    p.num_leaves, p.num_iterations = 15, 3
    one = orc.train([data], p)
    cut = int(data.query_boundaries[len(data.query_boundaries) // 2])
    two = orc.train([data.shard(0, cut), data.shard(cut, data.num_rows)], p)
    assert len(one.trees) == len(two.trees) == 3
    for k, (a, b) in enumerate(zip(one.trees, two.trees)):
        assert orc.trees_equal(a, b) == [], f"tree {k}"
