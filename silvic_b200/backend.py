"""The B200 backend as silvic's `trait Backend` (crates/silvic-core/src/backend/mod.rs:115-179), and training.

`B200Backend` wraps one `sb2_backend*` handle: the same methods, argument meanings and error behaviour as the
reference trait (a failure raises `SilvicError` with the reference's error kind). `train()` mirrors
`silvic.train(params, Dataset)` (python/silvic/engine.py:152-200) for the parameters this backend trains with,
running every boosting iteration on the device (`sb2_train`).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _abi
from .dataset import BinnedDataset

_PARAM_ALIASES = {
    "objective": ["objective_type", "app", "application", "loss"],
    "num_iterations": ["num_iteration", "n_iter", "num_tree", "num_trees", "num_round", "num_rounds",
                       "num_boost_round", "n_estimators", "max_iter"],
    "learning_rate": ["shrinkage_rate", "eta"],
    "num_leaves": ["num_leaf", "max_leaves", "max_leaf", "max_leaf_nodes"],
    "max_depth": [],
    "min_data_in_leaf": ["min_data_per_leaf", "min_data", "min_child_samples", "min_samples_leaf"],
    "min_sum_hessian_in_leaf": ["min_sum_hessian_per_leaf", "min_sum_hessian", "min_hessian", "min_child_weight"],
    "lambda_l1": ["reg_alpha", "l1_regularization"],
    "lambda_l2": ["reg_lambda", "lambda", "l2_regularization"],
    "min_gain_to_split": ["min_split_gain"],
    "bagging_fraction": ["sub_row", "subsample", "bagging"],
    "bagging_freq": ["subsample_freq"],
    "bagging_seed": ["bagging_fraction_seed"],
    "feature_fraction": ["sub_feature", "colsample_bytree"],
    "feature_fraction_seed": [],
    "data_random_seed": ["data_seed"],
    "boost_from_average": [],
    "use_quantized_grad": [],
    "sigmoid": [],
    "num_grad_quant_bins": [],
    "quant_train_renew_leaf": [],
    "stochastic_rounding": [],
    "lambdarank_truncation_level": [],
    "lambdarank_norm": [],
    "label_gain": [],
    "max_cat_to_onehot": [],
    "max_cat_threshold": [],
    "cat_l2": [],
    "cat_smooth": [],
    "min_data_per_group": [],
}
_OBJECTIVES = {"regression": _abi.REGRESSION, "regression_l2": _abi.REGRESSION, "l2": _abi.REGRESSION,
               "mean_squared_error": _abi.REGRESSION, "mse": _abi.REGRESSION, "binary": _abi.BINARY,
               "lambdarank": _abi.LAMBDARANK}
# Accepted for LightGBM compatibility, no effect (crates/silvic-core/src/config.rs NO_EFFECT_KEYS), plus the ones
# that select this backend or describe binning, which happens before training.
_IGNORED = {"force_row_wise", "force_col_wise", "deterministic", "histogram_pool_size", "feature_pre_filter",
            "first_metric_only", "gpu_platform_id", "gpu_use_dp", "num_gpu", "device_type", "device",
            "gpu_device_id", "num_threads", "verbosity", "verbose", "max_bin", "min_data_in_bin",
            "bin_construct_sample_cnt", "metric", "seed"}


def params_from_dict(params: dict) -> _abi.Params:
    """`Params::from_json` (crates/silvic-core/src/config.rs:274) for this backend's subset: LightGBM names and
    aliases, unknown keys rejected as config errors."""
    lib = _abi.load_library()
    p = _abi.Params()
    lib.sb2_default_params(C.byref(p))
    canonical = {}
    for name, aliases in _PARAM_ALIASES.items():
        canonical[name] = name
        for a in aliases:
            canonical[a] = name
    for key, value in params.items():
        if key in _IGNORED:
            continue
        name = canonical.get(key)
        if name is None:
            raise _abi.SilvicError(_abi.ECONFIG, f"unknown or unsupported parameter `{key}`")
        if name == "objective":
            if value not in _OBJECTIVES:
                raise _abi.SilvicError(_abi.EUNSUPPORTED, f"objective `{value}` on the B200 backend")
            p.objective = _OBJECTIVES[value]
        elif name in ("boost_from_average", "use_quantized_grad", "quant_train_renew_leaf", "stochastic_rounding",
                      "lambdarank_norm"):
            setattr(p, name, int(bool(value)))
        elif name == "label_gain":
            gains = [float(v) for v in (value.split(",") if isinstance(value, str) else value)]
            arr = (C.c_double * max(len(gains), 1))(*gains)
            p._label_gain = arr  # kept alive with the struct
            p.label_gain = C.cast(arr, C.POINTER(C.c_double))
            p.num_label_gain = len(gains)
        else:
            setattr(p, name, type(getattr(p, name))(value))
    return p


def _matrix_view(values):
    """(pointer, rows, cols, value bytes, row-major, keep-alive) of a 2-D float32/float64 matrix: a numpy array
    (C- or Fortran-ordered) or a CUDA torch tensor (contiguous or its transpose). A tensor's device finishes its queued
    work first: the library's stream is not ordered after torch's streams, so a kernel still writing the tensor would
    race with the call's reads."""
    if hasattr(values, "data_ptr") and getattr(values, "is_cuda", False):
        import torch

        if values.dim() != 2 or values.element_size() not in (4, 8) or not values.is_floating_point():
            raise ValueError("a 2-D float32 or float64 tensor")
        rows, cols = values.shape
        if not values.is_contiguous() and not values.t().is_contiguous():
            values = values.contiguous()
        torch.cuda.synchronize(values.device)  # whichever of torch's streams wrote it
        if values.is_contiguous():
            return C.c_void_p(values.data_ptr()), rows, cols, values.element_size(), True, values
        return C.c_void_p(values.data_ptr()), rows, cols, values.element_size(), False, values
    a = np.asarray(values)
    if a.ndim != 2 or a.dtype not in (np.float32, np.float64):
        raise ValueError("a 2-D float32 or float64 array")
    if not (a.flags.c_contiguous or a.flags.f_contiguous):
        a = np.ascontiguousarray(a)
    rows, cols = a.shape
    return C.c_void_p(a.ctypes.data), rows, cols, a.itemsize, bool(a.flags.c_contiguous), a


class B200Backend:
    """One GPU's backend handle (`trait Backend`). Not thread-safe; handles are independent."""

    def __init__(self, device: int = 0):
        self._lib = _abi.load_library()
        h = C.c_void_p()
        code = self._lib.sb2_create(device, C.byref(h))
        if code != _abi.OK:
            raise _abi.SilvicError(code, _abi.global_error())
        self._h = h
        self._data: BinnedDataset | None = None

    def close(self):
        if getattr(self, "_h", None):
            self._lib.sb2_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, code: int):
        if code != _abi.OK:
            buf = C.create_string_buffer(4096)
            self._lib.sb2_last_error(self._h, buf, len(buf))
            raise _abi.SilvicError(code, buf.value.decode())

    # ---- trait Backend ----
    def name(self) -> str:
        buf = C.create_string_buffer(256)
        self._lib.sb2_name(self._h, buf, len(buf))
        return buf.value.decode()

    def load(self, train: BinnedDataset, objective: str = "regression", sigmoid: float = 1.0,
             params: _abi.Params | None = None):
        """Backend::load. Lambdarank takes its normalization, truncation level and label gains from `params`
        (LightGBM's defaults without it)."""
        obj = _abi.Objective(_OBJECTIVES[objective] if isinstance(objective, str) else objective, 0, sigmoid)
        obj.lambdarank_norm, obj.lambdarank_truncation_level = 1, 30
        if params is not None:
            obj.lambdarank_norm = params.lambdarank_norm
            obj.lambdarank_truncation_level = params.lambdarank_truncation_level
            obj.label_gain, obj.num_label_gain = params.label_gain, params.num_label_gain
        d = train.c_struct()
        self._check(self._lib.sb2_load(self._h, C.byref(d), C.byref(obj)))
        self._data = train

    def bin_dense(self, values, features, groups, out: list[np.ndarray] | None = None) -> list[np.ndarray]:
        """data::binning::bin_rows on the device (`sb2_bin_dense`): `values` (rows × features, float32 or float64,
        C- or Fortran-ordered numpy array, or a CUDA torch tensor) binned with `features`' upper bounds into each of
        `groups`' rows; returns one uint8 array of rows × row_stride per group (`out`, when given: C-contiguous
        arrays of that shape, written in place)."""
        from .dataset import BinnedDataset

        ptr, rows, cols, vbytes, row_major, keep = _matrix_view(values)
        shell = BinnedDataset(rows, 0, list(features), [g.__class__(g.features, g.row_stride, g.hist_offset,
                                                                      g.total_bins, np.zeros((0, g.row_stride), np.uint8))
                                                        for g in groups], 0, np.zeros(0, np.float32))
        d = shell.c_struct()
        if out is None:
            outs = [np.zeros((rows, g.row_stride), dtype=np.uint8) for g in groups]
        else:
            outs = list(out)
            for o, g in zip(outs, groups):
                if o.shape != (rows, g.row_stride) or o.dtype != np.uint8 or not o.flags.c_contiguous:
                    raise ValueError(f"output of shape {o.shape}, expected C-contiguous uint8 {(rows, g.row_stride)}")
        ptrs = (C.POINTER(C.c_uint8) * max(len(outs), 1))(*[o.ctypes.data_as(C.POINTER(C.c_uint8)) for o in outs])
        self._check(self._lib.sb2_bin_dense(self._h, ptr, vbytes, rows, cols, int(row_major), d.features,
                                            len(features), d.groups, len(groups), ptrs))
        del keep
        return outs

    def init_scores(self, dataset: int, value: float):
        self._check(self._lib.sb2_init_scores(self._h, dataset, value))

    def compute_gradients(self) -> tuple[float, float]:
        s = _abi.GradientStats()
        self._check(self._lib.sb2_compute_gradients(self._h, C.byref(s)))
        return s.max_abs_grad, s.max_hess

    def quantize(self, spec: _abi.QuantSpec):
        self._check(self._lib.sb2_quantize(self._h, C.byref(spec)))

    def reset_partition(self, bag: _abi.BagSpec | None = None) -> int:
        bag = bag or _abi.BagSpec(0, 0, 0, 0, 1.0)
        rows = C.c_uint32()
        self._check(self._lib.sb2_reset_partition(self._h, C.byref(bag), C.byref(rows)))
        return rows.value

    def set_histogram_features(self, used):
        u = np.ascontiguousarray(used, dtype=np.uint8)
        self._check(self._lib.sb2_set_histogram_features(self._h, u.ctypes.data_as(C.POINTER(C.c_uint8)), len(u)))

    def histogram(self, begin: int, count: int, quantized: bool = True, out: np.ndarray | None = None) -> np.ndarray:
        out = np.empty(2 * self._data.total_bins) if out is None else out
        self._check(self._lib.sb2_histogram(self._h, _abi.LeafRange(begin, count), int(quantized),
                                            out.ctypes.data_as(C.POINTER(C.c_double)), len(out)))
        return out

    def partition(self, begin: int, count: int, split: _abi.BinSplit) -> int:
        left = C.c_uint32()
        self._check(self._lib.sb2_partition(self._h, _abi.LeafRange(begin, count), C.byref(split), C.byref(left)))
        return left.value

    def partition_and_histogram(self, begin: int, count: int, split: _abi.BinSplit, side: int,
                                quantized: bool = True) -> tuple[int, np.ndarray]:
        out = np.empty(2 * self._data.total_bins)
        left = C.c_uint32()
        self._check(self._lib.sb2_partition_and_histogram(
            self._h, _abi.LeafRange(begin, count), C.byref(split), side, int(quantized),
            out.ctypes.data_as(C.POINTER(C.c_double)), len(out), C.byref(left)))
        return left.value, out

    def leaf_sums(self, leaves, grad_scale: float, hess_scale: float) -> np.ndarray:
        arr = (_abi.LeafRange * max(len(leaves), 1))(*[_abi.LeafRange(b, c) for b, c in leaves])
        out = np.zeros(2 * len(leaves), dtype=np.int64)
        self._check(self._lib.sb2_leaf_sums(self._h, arr, len(leaves), grad_scale, hess_scale,
                                            out.ctypes.data_as(C.POINTER(C.c_int64))))
        return out.reshape(-1, 2)

    def add_tree(self, nodes, leaf_values):
        arr = (_abi.DeviceNode * max(len(nodes), 1))(*nodes)
        lv = np.ascontiguousarray(leaf_values, dtype=np.float32)
        self._check(self._lib.sb2_add_tree(self._h, arr, len(nodes), lv.ctypes.data_as(C.POINTER(C.c_float)),
                                           len(lv)))

    def scores(self, dataset: int = 0) -> np.ndarray:
        out = np.empty(self._data.num_rows, dtype=np.float32)
        self._check(self._lib.sb2_scores(self._h, dataset, out.ctypes.data_as(C.POINTER(C.c_float)), len(out)))
        return out

    # ---- state access for tests (the reference's CpuBackend tests read the same fields) ----
    def read_partition(self, n: int | None = None) -> np.ndarray:
        n = self._data.num_rows if n is None else n
        out = np.empty(n, dtype=np.uint32)
        self._check(self._lib.sb2_read_partition(self._h, out.ctypes.data_as(C.POINTER(C.c_uint32)), n))
        return out

    def read_packed(self) -> np.ndarray:
        out = np.empty(self._data.num_rows, dtype=np.int32)
        self._check(self._lib.sb2_read_packed(self._h, out.ctypes.data_as(C.POINTER(C.c_int32)), len(out)))
        return out

    def write_gradients(self, grad, hess):
        g = np.ascontiguousarray(grad, dtype=np.float32)
        h = np.ascontiguousarray(hess, dtype=np.float32)
        self._check(self._lib.sb2_write_gradients(self._h, g.ctypes.data_as(C.POINTER(C.c_float)),
                                                  h.ctypes.data_as(C.POINTER(C.c_float)), len(g)))

    def read_gradients(self) -> tuple[np.ndarray, np.ndarray]:
        n = self._data.num_rows
        g, h = np.empty(n, dtype=np.float32), np.empty(n, dtype=np.float32)
        self._check(self._lib.sb2_read_gradients(self._h, g.ctypes.data_as(C.POINTER(C.c_float)),
                                                 h.ctypes.data_as(C.POINTER(C.c_float)), n))
        return g, h

    def find_best_split(self, hist: np.ndarray, evaluate, sums: tuple[float, float, int],
                        scale: tuple[float, float], cfg: _abi.SplitConfig) -> tuple[_abi.SplitInfo, np.ndarray]:
        h = np.ascontiguousarray(hist, dtype=np.float64)
        ev = np.ascontiguousarray(evaluate, dtype=np.uint8)
        info = _abi.SplitInfo()
        spl = np.zeros(len(ev), dtype=np.uint8)
        self._check(self._lib.sb2_find_best_split(
            self._h, h.ctypes.data_as(C.POINTER(C.c_double)), len(h), ev.ctypes.data_as(C.POINTER(C.c_uint8)),
            sums[0], sums[1], sums[2], scale[0], scale[1], C.byref(cfg), C.byref(info),
            spl.ctypes.data_as(C.POINTER(C.c_uint8))))
        return info, spl

    def time_histogram(self, repeats: int = 10, rows: int = 0) -> float:
        """Mean seconds of one histogram of the first `rows` rows (all when 0), CUDA events on the handle's
        stream."""
        secs = C.c_double()
        self._check(self._lib.sb2_time_histogram(self._h, rows, repeats, C.byref(secs)))
        return secs.value

    def time_shared_adds(self, pattern: int = 0) -> tuple[float, float]:
        """(lane adds per second, per SM clock) of red.shared.add.u32 alone at the histogram's address pattern
        (0: every lane its own bins; 1: one bin per instruction)."""
        per_s, per_clk = C.c_double(), C.c_double()
        self._check(self._lib.sb2_time_shared_adds(self._h, pattern, C.byref(per_s), C.byref(per_clk)))
        return per_s.value, per_clk.value

    PROFILE_OPS = ("gradients", "quantize", "histogram", "partition", "search", "leaf_sums", "finalize",
                   "add_tree", "collectives", "tree", "tree.partition_histogram", "tree.search_context",
                   "tree.reduce_search", "tree.finish", "tree.barriers")

    def profile_train(self, params: _abi.Params, init_score: float) -> tuple[dict, "Model"]:
        """Device seconds per operation of the last iteration (graph-free, CUDA events), and the model."""
        secs = (C.c_double * len(self.PROFILE_OPS))()
        m = C.c_void_p()
        self._check(self._lib.sb2_profile_train(self._h, C.byref(params), init_score, secs, len(secs), C.byref(m)))
        try:
            return dict(zip(self.PROFILE_OPS, list(secs))), Model.from_handle(self._lib, m, init_score)
        finally:
            self._lib.sb2_model_free(m)

    STEP_FIELDS = ("partition_histogram", "search_context", "reduce_search", "finish", "barriers", "hist_rows",
                   "splits", "committed", "kept")

    def profile_steps(self, params: _abi.Params, init_score: float, max_steps: int = 1 << 17) -> np.ndarray:
        """Per split step of the last tree (row 0 the root): the tree kernel's phase seconds and the step's sizes,
        columns STEP_FIELDS."""
        rows = np.zeros((max_steps, len(self.STEP_FIELDS)), dtype=np.float64)
        n = C.c_size_t()
        self._check(self._lib.sb2_profile_steps(self._h, C.byref(params), init_score,
                                                rows.ctypes.data_as(C.POINTER(C.c_double)), max_steps, C.byref(n)))
        return rows[: n.value]

    # ---- multi-GPU ----
    @staticmethod
    def nccl_unique_id() -> bytes:
        lib = _abi.load_library()
        buf = (C.c_uint8 * 128)()
        code = lib.sb2_nccl_unique_id(buf, 128)
        if code != _abi.OK:
            raise _abi.SilvicError(code, _abi.global_error())
        return bytes(buf)

    def set_dominant_share(self, share: float):
        """sb2_set_dominant_share: tiles whose features hold at least `share` of the rows in their most frequent bins
        (on average) skip those bins in the tree kernel's histogram; 0: every tile, above 1 (the default): none.
        Takes effect at the next load."""
        self._check(self._lib.sb2_set_dominant_share(self._h, float(share)))

    def set_rank_exchange(self, mode: int):
        """sb2_set_rank_exchange: _abi.EXCHANGE_AUTO (NVLink inside the tree kernel) or _abi.EXCHANGE_NCCL."""
        self._check(self._lib.sb2_set_rank_exchange(self._h, mode))

    def test_unanswered_peer(self, spin_limit: int):
        """sb2_test_unanswered_peer: train as rank 0 of two whose other rank never answers (0: one rank again)."""
        self._check(self._lib.sb2_test_unanswered_peer(self._h, spin_limit))

    def join_ranks(self, unique_id: bytes, world: int, rank: int):
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        self._check(self._lib.sb2_join_ranks(self._h, buf, 128, world, rank))

    # ---- training ----
    def train(self, params: _abi.Params, init_score: float) -> "Model":
        m = C.c_void_p()
        self._check(self._lib.sb2_train(self._h, C.byref(params), init_score, C.byref(m)))
        try:
            return Model.from_handle(self._lib, m, init_score)
        finally:
            self._lib.sb2_model_free(m)


@dataclass
class Tree:
    """A tree in LightGBM 3.3.5 array layout (crates/silvic-core/src/tree.rs:47-73)."""

    num_leaves: int
    shrinkage: float
    split_feature: np.ndarray
    split_gain: np.ndarray
    threshold: np.ndarray
    threshold_bin: np.ndarray
    decision_type: np.ndarray
    left_child: np.ndarray
    right_child: np.ndarray
    leaf_value: np.ndarray
    leaf_weight: np.ndarray
    leaf_count: np.ndarray
    internal_value: np.ndarray
    internal_weight: np.ndarray
    internal_count: np.ndarray
    cat_bins: np.ndarray  # [splits, 8] u32: the bins a categorical split sends left (zeros for numerical)

    FIELDS = ("split_feature", "split_gain", "threshold", "threshold_bin", "decision_type", "left_child",
              "right_child", "leaf_value", "leaf_weight", "leaf_count", "internal_value", "internal_weight",
              "internal_count", "cat_bins")

    @staticmethod
    def from_view(v: _abi.TreeView) -> "Tree":
        n, nl = max(v.num_leaves - 1, 0), v.num_leaves
        arr = lambda ptr, k: np.ctypeslib.as_array(ptr, shape=(k,)).copy() if k else np.zeros(0)  # noqa: E731
        return Tree(nl, v.shrinkage, arr(v.split_feature, n), arr(v.split_gain, n), arr(v.threshold, n),
                    arr(v.threshold_bin, n), arr(v.decision_type, n), arr(v.left_child, n), arr(v.right_child, n),
                    arr(v.leaf_value, nl), arr(v.leaf_weight, nl), arr(v.leaf_count, nl), arr(v.internal_value, n),
                    arr(v.internal_weight, n), arr(v.internal_count, n),
                    (arr(v.cat_bins, 8 * n) if v.cat_bins else np.zeros(8 * n, dtype=np.uint32)).reshape(n, 8))

    def leaf_index(self, row: np.ndarray) -> int:
        """`Tree::GetLeaf` with NumericalDecision (crates/silvic-core/src/model/predict.rs:98-141); trees with
        categorical splits predict through their model text (silvic_b200.model_text), which holds the categories."""
        if self.num_leaves <= 1:
            return 0
        if any(int(d) & 1 for d in self.decision_type):
            raise ValueError("a categorical split: predict through the model text")
        zero = float(np.float32(1e-35))
        node = 0
        while node >= 0:
            value = float(row[self.split_feature[node]])
            if abs(value) <= zero:
                value = 0.0
            dt = int(self.decision_type[node])
            missing = (dt >> 2) & 3
            if np.isnan(value) and missing != 2:
                value = 0.0
            is_missing = (-zero <= value <= zero) if missing == 1 else (np.isnan(value) if missing == 2 else False)
            left = bool(dt & 2) if is_missing else value <= self.threshold[node]
            node = int(self.left_child[node] if left else self.right_child[node])
        return ~node


@dataclass
class Model:
    trees: list[Tree]
    init_score: float
    iteration_seconds: list[float]
    tree_seconds: list[float] = field(default_factory=list)  # the tree kernel's own time per iteration (1 GPU)

    @staticmethod
    def from_handle(lib, handle, init_score: float) -> "Model":
        trees = []
        for i in range(lib.sb2_model_num_trees(handle)):
            v = _abi.TreeView()
            lib.sb2_model_tree(handle, i, C.byref(v))
            trees.append(Tree.from_view(v))
        secs = (C.c_double * 100000)()
        k = lib.sb2_model_iteration_seconds(handle, secs, 100000)
        tsecs = (C.c_double * 100000)()
        kt = lib.sb2_model_tree_seconds(handle, tsecs, 100000)
        return Model(trees, init_score, list(secs[: min(k, 100000)]), list(tsecs[: min(kt, 100000)]))

    def to_lightgbm_string(self, dataset, params: _abi.Params) -> str:
        """The model file silvic writes for this training run (`Model::to_lightgbm_string`,
        crates/silvic-core/src/model/text.rs:48-70): feature names and infos from `dataset`, parameters from
        `params` (silvic_b200.model_text)."""
        from . import model_text

        return model_text.from_trained(self, dataset, params).to_string()

    def predict_raw_row(self, row: np.ndarray) -> float:
        """Model::predict_raw_row (crates/silvic-core/src/model/predict.rs:19-23): f64 sum of leaf values."""
        score = 0.0
        for t in self.trees:
            score = score + float(t.leaf_value[t.leaf_index(row)])
        return score


def init_score(params: _abi.Params, label: np.ndarray, weight: np.ndarray | None = None) -> float:
    """objective::init_score over every rank's labels, in row order (the device trainer's caller computes it)."""
    lib = _abi.load_library()
    lab = np.ascontiguousarray(label, dtype=np.float32)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    out = C.c_double()
    code = lib.sb2_boost_from_average(C.byref(params), lab.ctypes.data_as(C.POINTER(C.c_float)),
                                      None if w is None else w.ctypes.data_as(C.POINTER(C.c_float)), len(lab),
                                      C.byref(out))
    if code != _abi.OK:
        raise _abi.SilvicError(code, _abi.global_error())
    return out.value


def train(params: dict, train_set: BinnedDataset, device: int = 0) -> Model:
    """`silvic.train(params, Dataset)` on one B200: every boosting iteration on the device."""
    p = params_from_dict(params)
    backend = B200Backend(device)
    try:
        backend.load(train_set, p.objective, p.sigmoid, p)
        return backend.train(p, init_score(p, train_set.label, train_set.weight))
    finally:
        backend.close()
