"""Seeded synthetic datasets for the tests, built from silvic's counter hash (quantize.rs:16-31) so every rank can
regenerate its rows."""

from __future__ import annotations

import numpy as np

from silvic_b200.dataset import BinnedDataset, categorical_mapper, numerical_mapper


def mix32(x: np.ndarray) -> np.ndarray:
    """lowbias32 (crates/silvic-core/src/quantize.rs:16-23) over uint32 arrays."""
    x = np.asarray(x, dtype=np.uint32).copy()
    with np.errstate(over="ignore"):
        x ^= x >> np.uint32(16)
        x *= np.uint32(0x7FEB352D)
        x ^= x >> np.uint32(15)
        x *= np.uint32(0x846CA68B)
        x ^= x >> np.uint32(16)
    return x


def unit(stream: int, rows: np.ndarray) -> np.ndarray:
    """A 24-bit uniform in [0, 1) per row from (stream, row)."""
    h = mix32(mix32(rows.astype(np.uint32)) ^ mix32(np.uint32(stream)))
    return (h >> np.uint32(8)).astype(np.float64) / 16777216.0


def random_binned(rows: int, bins_per_feature: list[int], nan_bins: list[bool] | None = None, seed: int = 1,
                  skew: float = 0.0, label_kind: str = "regression",
                  skew_bins: list[int] | None = None) -> BinnedDataset:
    """Rows with hash-drawn bins per feature (a `skew` share of rows in bin 0, or in feature f's skew_bins[f]) and a
    label that depends on a few bins, so trees have structure."""
    r = np.arange(rows, dtype=np.uint64)
    nf = len(bins_per_feature)
    nan_bins = nan_bins or [False] * nf
    bins = np.empty((rows, nf), dtype=np.uint8)
    for f, nb in enumerate(bins_per_feature):
        u = unit(seed * 1000 + f, r)
        b = (u * nb).astype(np.int64)
        if skew > 0:
            zero = unit(seed * 1000 + 500 + f, r) < skew
            b[zero] = skew_bins[f] if skew_bins is not None else 0
        bins[:, f] = np.minimum(b, nb - 1).astype(np.uint8)
    signal = np.zeros(rows)
    for f in range(min(nf, 6)):
        signal += (bins[:, f].astype(np.float64) / max(bins_per_feature[f] - 1, 1) - 0.5) * (1.0 + f)
    if nf >= 2:
        signal += 0.5 * (bins[:, 0] > bins_per_feature[0] // 2) * (bins[:, 1] > bins_per_feature[1] // 2)
    noise = unit(seed * 1000 + 999, r) - 0.5
    if label_kind == "binary":
        label = ((signal + noise) > 0).astype(np.float32)
    else:
        label = (signal + 0.3 * noise).astype(np.float32)
    mappers = [numerical_mapper(f"f{f}", nb, nb > 2 and nan_bins[f]) for f, nb in enumerate(bins_per_feature)]
    return BinnedDataset.from_bins(bins, mappers, label)


def nested_binned(rows: int, seed: int = 7) -> BinnedDataset:
    """Three binary features whose conjunction carries most of the label (8 when all three are set) beside six
    63-bin features with small effects: each split on the conjunction's path leaves a child with a larger gain than
    any other leaf, so the learner's next leaf is often a child of its last split."""
    r = np.arange(rows, dtype=np.uint64)
    widths = [2, 2, 2] + [63] * 6
    bins = np.empty((rows, len(widths)), dtype=np.uint8)
    for f, nb in enumerate(widths):
        bins[:, f] = np.minimum((unit(seed * 1000 + f, r) * nb).astype(np.int64), nb - 1).astype(np.uint8)
    label = 8.0 * (bins[:, 0] & bins[:, 1] & bins[:, 2])
    for f in range(3, len(widths)):
        label = label + 0.3 * (f - 2) * bins[:, f].astype(np.float64) / 62.0
    label = (label + 0.2 * (unit(seed * 1000 + 999, r) - 0.5)).astype(np.float32)
    mappers = [numerical_mapper(f"f{f}", nb, False) for f, nb in enumerate(widths)]
    return BinnedDataset.from_bins(bins, mappers, label)


def ranking_binned(rows: int, bins_per_feature: list[int], seed: int = 1, mean_query: float = 40.0,
                   long_query: int = 0) -> BinnedDataset:
    """A lambdarank dataset: hash-drawn bins, queries of Poisson(mean_query) rows (at least 1; one query of
    `long_query` rows first when given), labels 0..4: a noisy score of a few features cut into five levels."""
    data = random_binned(rows, bins_per_feature, seed=seed)
    rng = np.random.default_rng(seed)
    sizes = [long_query] if long_query else []
    while sum(sizes) < rows:
        sizes.append(max(1, int(rng.poisson(mean_query))))
    sizes[-1] -= sum(sizes) - rows
    if sizes[-1] == 0:
        sizes.pop()
    qb = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)
    score = data.label.astype(np.float64) + 0.3 * rng.normal(size=rows)
    label = np.clip(np.floor((score - score.min()) / (np.ptp(score) + 1e-12) * 5.0), 0, 4).astype(np.float32)
    data.label = label
    data.query_boundaries = qb
    return data


def categorical_binned(rows: int, seed: int = 9, label_kind: str = "regression") -> BinnedDataset:
    """Two categorical features (3 bins: one-hot; 40 bins: sorted) whose categories carry the label, beside four
    63-bin numerical ones; bin 0 ("other") holds a tenth of the rows."""
    r = np.arange(rows, dtype=np.uint64)
    cats = [[7, 3], list(range(100, 139))]
    bins = np.zeros((rows, 6), dtype=np.uint8)
    for f, cs in enumerate(cats):
        u = unit(seed * 1000 + f, r)
        bins[:, f] = np.where(unit(seed * 1000 + 50 + f, r) < 0.1, 0, 1 + (u * len(cs)).astype(np.int64))
    for f in range(2, 6):
        bins[:, f] = np.minimum((unit(seed * 1000 + f, r) * 63).astype(np.int64), 62)
    effect = np.sin(np.arange(40) * 1.7) * 2.0
    signal = effect[bins[:, 1]] + 1.5 * (bins[:, 0] == 2) + bins[:, 2] / 62.0
    noise = unit(seed * 1000 + 999, r) - 0.5
    label = ((signal + noise) > 0.5).astype(np.float32) if label_kind == "binary" else (signal + 0.3 * noise)
    mappers = [categorical_mapper(f"c{f}", cs) for f, cs in enumerate(cats)]
    mappers += [numerical_mapper(f"n{f}", 63) for f in range(2, 6)]
    return BinnedDataset.from_bins(bins, mappers, label.astype(np.float32))
