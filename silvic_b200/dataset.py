"""Binned training data in silvic's layout (crates/silvic-core/src/data/mod.rs:22-87).

`BinnedDataset` holds what the reference's `BinnedDataset` holds: per-feature bin mappers and histogram offsets,
features packed into groups of at most `GROUP_BIN_BUDGET` bins with row-major byte rows, labels, weights and the
rank's `row_offset`. `BinnedDataset.c_struct()` is the flat `sb2_dataset` the C ABI takes.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _abi

GROUP_BIN_BUDGET = 8192  # crates/silvic-core/src/data/mod.rs:22


@dataclass
class FeatureMeta:
    """FeatureMeta (data/mod.rs:25-36) with its numerical BinMapper (data/bin_mapper.rs:26-41)."""

    name: str
    kind: int = _abi.NUMERICAL
    num_bins: int = 0          # NaN bin included; 0 for a trivial feature
    nan_bin: bool = False
    upper_bounds: np.ndarray | None = None  # ascending, the last +inf
    categories: list[int] | None = None     # categorical: categories[b - 1] is bin b's value; bin 0 is "other"
    min_value: float = 0.0
    max_value: float = 0.0
    group: int = 0
    column: int = 0
    hist_offset: int = 0

    @property
    def is_trivial(self) -> bool:
        return self.num_bins == 0


@dataclass
class FeatureGroup:
    """FeatureGroup (data/mod.rs:49-59): `data[row, column]`, row_stride = features rounded up to 4."""

    features: list[int]
    row_stride: int
    hist_offset: int
    total_bins: int
    data: np.ndarray  # uint8 [rows, row_stride]


@dataclass
class BinnedDataset:
    num_rows: int
    row_offset: int
    features: list[FeatureMeta]
    groups: list[FeatureGroup]
    total_bins: int
    label: np.ndarray
    weight: np.ndarray | None = None
    # lambdarank: num_queries + 1 row boundaries of the rank's queries (data/mod.rs:62-74), starting at 0
    query_boundaries: np.ndarray | None = None
    _keep: list = field(default_factory=list, repr=False)

    @staticmethod
    def from_bins(bins: np.ndarray, mappers: list[FeatureMeta], label: np.ndarray, *, weight=None,
                  row_offset: int = 0, query_boundaries=None) -> "BinnedDataset":
        """Packs per-feature bins (uint8 [rows, features]) into groups: `layout` (data/build.rs:336-382), the
        non-trivial features in input order, a new group whenever the next feature's bins would take the current one
        over GROUP_BIN_BUDGET."""
        bins = np.asarray(bins, dtype=np.uint8)
        rows, nf = bins.shape
        assert nf == len(mappers)
        features, shells, total_bins = layout(mappers)
        out_groups = []
        for g in shells:
            data = np.zeros((rows, g.row_stride), dtype=np.uint8)
            data[:, : len(g.features)] = bins[:, g.features]
            out_groups.append(FeatureGroup(g.features, g.row_stride, g.hist_offset, g.total_bins, data))
        label = np.ascontiguousarray(label, dtype=np.float32)
        weight = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        qb = None if query_boundaries is None else np.ascontiguousarray(query_boundaries, dtype=np.uint32)
        return BinnedDataset(rows, row_offset, features, out_groups, total_bins, label, weight, qb)

    @staticmethod
    def from_chunks(chunks, rows: int, mappers: list[FeatureMeta], label: np.ndarray, binner, *, weight=None,
                    row_offset: int = 0, query_boundaries=None, out: list[np.ndarray] | None = None) -> "BinnedDataset":
        """Streaming construction (BinnedDataset::construct's bin_rows, data/build.rs:81-126 and
        data/binning.rs:71-135, with the mappers given): `chunks` yields (first row, values) for consecutive row
        ranges covering 0 .. rows, each values a chunk × features matrix (numpy, or a CUDA tensor made on the
        device); `binner` (a B200Backend) bins each into its rows of the groups, so the raw matrix never exists
        whole. `out` (optional, e.g. page-locked) receives the groups' rows: C-contiguous uint8 arrays of rows ×
        row_stride per group of layout(mappers)."""
        features, shells, total_bins = layout(mappers)
        data = out if out is not None else [np.zeros((rows, g.row_stride), dtype=np.uint8) for g in shells]
        done = 0
        for first, values in chunks:
            n = int(values.shape[0])
            if first != done or first + n > rows:
                raise ValueError(f"chunk of rows {first}..{first + n}: expected it to start at {done} and end by {rows}")
            binner.bin_dense(values, features, shells, out=[d[first:first + n] for d in data])
            done += n
        if done != rows:
            raise ValueError(f"the chunks covered {done} of {rows} rows")
        groups = [FeatureGroup(g.features, g.row_stride, g.hist_offset, g.total_bins, d) for g, d in zip(shells, data)]
        label = np.ascontiguousarray(label, dtype=np.float32)
        weight = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        qb = None if query_boundaries is None else np.ascontiguousarray(query_boundaries, dtype=np.uint32)
        return BinnedDataset(rows, row_offset, features, groups, total_bins, label, weight, qb)

    def bin(self, feature: int, row: int) -> int:
        m = self.features[feature]
        return int(self.groups[m.group].data[row, m.column])

    def feature_bins(self, feature: int) -> np.ndarray:
        m = self.features[feature]
        return self.groups[m.group].data[:, m.column]

    def shard(self, begin: int, end: int) -> "BinnedDataset":
        """Rows begin..end as one rank holds them: `row_offset` moves by `begin` (data/mod.rs:64-65). With queries,
        begin and end must be query boundaries: a query's rows stay on one rank."""
        groups = [FeatureGroup(g.features, g.row_stride, g.hist_offset, g.total_bins,
                               np.ascontiguousarray(g.data[begin:end])) for g in self.groups]
        qb = None
        if self.query_boundaries is not None:
            qb_all = self.query_boundaries.astype(np.int64)
            lo, hi = np.searchsorted(qb_all, [begin, end])
            if lo >= len(qb_all) or qb_all[lo] != begin or hi >= len(qb_all) or qb_all[hi] != end:
                raise ValueError(f"rows {begin}..{end} cut a query")
            qb = np.ascontiguousarray(qb_all[lo:hi + 1] - begin, dtype=np.uint32)
        return BinnedDataset(end - begin, self.row_offset + begin, self.features, groups, self.total_bins,
                             np.ascontiguousarray(self.label[begin:end]),
                             None if self.weight is None else np.ascontiguousarray(self.weight[begin:end]), qb)

    def c_struct(self) -> _abi.Dataset:
        """The dataset as `sb2_dataset`; the arrays it points to live as long as this object."""
        keep = []
        feats = (_abi.Feature * max(len(self.features), 1))()
        for i, m in enumerate(self.features):
            f = feats[i]
            f.num_bins, f.group, f.column, f.hist_offset = m.num_bins, m.group, m.column, m.hist_offset
            f.kind = m.kind if m.num_bins else _abi.TRIVIAL
            f.nan_bin = int(m.nan_bin)
            if m.upper_bounds is not None:
                ub = np.ascontiguousarray(m.upper_bounds, dtype=np.float64)
                keep.append(ub)
                f.upper_bounds = ub.ctypes.data_as(C.POINTER(C.c_double))
                f.num_upper_bounds = len(ub)
            f.min_value, f.max_value = m.min_value, m.max_value
            if m.categories is not None:
                cats = np.ascontiguousarray(m.categories, dtype=np.int32)
                keep.append(cats)
                f.categories = cats.ctypes.data_as(C.POINTER(C.c_int32))
                f.num_categories = len(cats)
        groups = (_abi.Group * max(len(self.groups), 1))()
        for i, g in enumerate(self.groups):
            data = np.ascontiguousarray(g.data, dtype=np.uint8)
            fl = np.ascontiguousarray(g.features, dtype=np.uint32)
            keep += [data, fl]
            groups[i].data = data.ctypes.data_as(C.POINTER(C.c_uint8))
            groups[i].row_stride, groups[i].hist_offset = g.row_stride, g.hist_offset
            groups[i].total_bins, groups[i].num_features = g.total_bins, len(g.features)
            groups[i].features = fl.ctypes.data_as(C.POINTER(C.c_uint32))
        d = _abi.Dataset()
        d.num_rows, d.row_offset = self.num_rows, self.row_offset
        d.num_features, d.num_groups, d.total_bins = len(self.features), len(self.groups), self.total_bins
        d.features, d.groups = feats, groups
        label = np.ascontiguousarray(self.label, dtype=np.float32)
        keep += [feats, groups, label]
        d.label = label.ctypes.data_as(C.POINTER(C.c_float))
        if self.weight is not None:
            w = np.ascontiguousarray(self.weight, dtype=np.float32)
            keep.append(w)
            d.weight = w.ctypes.data_as(C.POINTER(C.c_float))
        if self.query_boundaries is not None:
            qb = np.ascontiguousarray(self.query_boundaries, dtype=np.uint32)
            keep.append(qb)
            d.num_queries = len(qb) - 1
            d.query_boundaries = qb.ctypes.data_as(C.POINTER(C.c_uint32))
        d._keep = keep  # ctypes keeps Python attributes on the struct object alive with it
        return d


def layout(mappers: list[FeatureMeta]) -> tuple[list[FeatureMeta], list[FeatureGroup], int]:
    """`layout` (data/build.rs:336-382): the features with their groups, columns and histogram offsets, and the
    groups (no rows yet): the non-trivial features in input order, a new group whenever the next feature's bins would
    take the current one over GROUP_BIN_BUDGET. Returns (features, groups, total_bins)."""
    features: list[FeatureMeta] = []
    groups: list[dict] = []
    offset = 0
    for index, m in enumerate(mappers):
        meta = FeatureMeta(name=m.name, kind=m.kind, num_bins=m.num_bins, nan_bin=m.nan_bin,
                           upper_bounds=m.upper_bounds, categories=m.categories, min_value=m.min_value,
                           max_value=m.max_value)
        if meta.num_bins == 0:
            meta.group, meta.column, meta.hist_offset = 0, 0, offset
            features.append(meta)
            continue
        if not groups or groups[-1]["total_bins"] + meta.num_bins > GROUP_BIN_BUDGET:
            groups.append({"features": [], "hist_offset": offset, "total_bins": 0})
        g = groups[-1]
        meta.group = len(groups) - 1
        meta.column = len(g["features"])
        meta.hist_offset = offset
        g["features"].append(index)
        g["total_bins"] += meta.num_bins
        offset += meta.num_bins
        features.append(meta)
    shells = [FeatureGroup(g["features"], (len(g["features"]) + 3) // 4 * 4, g["hist_offset"], g["total_bins"],
                           np.zeros((0, (len(g["features"]) + 3) // 4 * 4), np.uint8)) for g in groups]
    return features, shells, offset


def numerical_mapper(name: str, num_bins: int, nan_bin: bool = False) -> FeatureMeta:
    """A numerical mapper with bins `0..num_bins` (NaN bin last when `nan_bin`): upper bounds b + 0.5, the last
    +inf, as the reference's learner tests build them (learner.rs:497-507)."""
    numeric = num_bins - int(nan_bin)
    ub = np.arange(numeric, dtype=np.float64) + 0.5
    ub[-1] = np.inf
    return FeatureMeta(name=name, num_bins=num_bins, nan_bin=nan_bin, upper_bounds=ub, min_value=0.0,
                       max_value=float(numeric))


def categorical_mapper(name: str, categories: list[int]) -> FeatureMeta:
    """A categorical mapper (bin_mapper.rs:36-39): bin b >= 1 holds category categories[b - 1], bin 0 every
    negative, NaN or unseen value."""
    return FeatureMeta(name=name, kind=_abi.CATEGORICAL, num_bins=len(categories) + 1,
                       categories=[int(c) for c in categories])
