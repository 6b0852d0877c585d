"""ctypes binding of the CPU oracle (oracle/oracle.cpp) — the checker the device is compared against.

Test infrastructure only: tests, the smoke check and the bench's CPU-baseline leg load it.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

from silvic_b200 import _abi
from silvic_b200.backend import Tree

ROOT = Path(__file__).resolve().parent.parent
ORACLE = ROOT / "oracle" / "_build" / "liboracle.so"
P = C.POINTER
VP = C.c_void_p

_SIGS = {
    "orc_num_threads": (C.c_int, []),
    "orc_set_num_threads": (None, [C.c_int]),
    "orc_mix32": (C.c_uint32, [C.c_uint32]),
    "orc_uniform": (C.c_float, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]),
    "orc_quant_spec": (None, [C.c_double, C.c_double, C.c_int, C.c_double, C.c_uint32, C.c_int, C.c_uint32,
                              C.c_uint32, P(_abi.QuantSpec)]),
    "orc_quantize": (None, [P(_abi.QuantSpec), P(C.c_float), P(C.c_float), C.c_size_t, C.c_uint64, P(C.c_int32)]),
    "orc_unpack": (None, [C.c_int32, P(C.c_int32), P(C.c_int32)]),
    "orc_in_bag": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint64, C.c_double]),
    "orc_fixed_point_scale": (C.c_float, [C.c_double]),
    "orc_to_fixed": (C.c_int64, [C.c_float, C.c_float]),
    "orc_gradients": (None, [P(_abi.Objective), P(C.c_float), P(C.c_float), P(C.c_float), C.c_size_t, P(C.c_float),
                             P(C.c_float)]),
    "orc_init_score": (C.c_double, [P(_abi.Params), P(C.c_float), P(C.c_float), C.c_size_t]),
    "orc_lambdarank_gradients": (C.c_int, [P(_abi.Params), P(_abi.Dataset), P(C.c_float), P(C.c_float),
                                           P(C.c_float)]),
    "orc_lambdarank_max_dcg": (C.c_double, [C.c_size_t, P(C.c_float), C.c_size_t, P(C.c_double), C.c_size_t]),
    "orc_lambdarank_sigmoid": (C.c_double, [C.c_double, C.c_double]),
    "orc_histogram": (C.c_int, [P(_abi.Dataset), P(C.c_int32), C.c_int32, P(C.c_uint32), C.c_size_t, P(C.c_uint8),
                                P(C.c_double)]),
    "orc_partition": (C.c_uint32, [P(_abi.Dataset), P(_abi.BinSplit), P(C.c_uint32), C.c_size_t]),
    "orc_leaf_sums": (None, [P(C.c_float), P(C.c_float), P(C.c_uint32), P(_abi.LeafRange), C.c_size_t, C.c_float,
                             C.c_float, P(C.c_int64)]),
    "orc_add_tree": (C.c_int, [P(_abi.Dataset), P(_abi.DeviceNode), C.c_size_t, P(C.c_float), C.c_size_t,
                               P(C.c_float)]),
    "orc_reset_partition": (C.c_uint32, [P(_abi.BagSpec), C.c_uint64, C.c_uint64, P(C.c_uint32)]),
    "orc_bin_rows": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_uint32, C.c_int, P(_abi.Feature), C.c_uint32,
                               P(_abi.Group), C.c_uint32, P(P(C.c_uint8))]),
    "orc_value_to_bin": (C.c_uint32, [P(C.c_double), C.c_uint32, C.c_int, C.c_double]),
    "orc_find_best_split": (C.c_int, [P(_abi.Dataset), P(C.c_double), P(C.c_uint8), C.c_double, C.c_double,
                                      C.c_int64, C.c_double, C.c_double, P(_abi.SplitConfig), P(_abi.SplitInfo),
                                      P(C.c_uint8)]),
    "orc_feature_mask": (None, [P(_abi.Dataset), C.c_double, C.c_uint32, C.c_uint32, P(C.c_uint8)]),
    "orc_train": (C.c_int, [P(_abi.Dataset), C.c_int, P(_abi.Params), P(VP)]),
    "orc_model_free": (None, [VP]),
    "orc_model_num_trees": (C.c_int, [VP]),
    "orc_model_tree": (C.c_int, [VP, C.c_int, P(_abi.TreeView)]),
    "orc_model_init_score": (C.c_double, [VP]),
    "orc_model_iteration_seconds": (C.c_int, [VP, P(C.c_double), C.c_size_t]),
    "orc_model_op_seconds": (C.c_int, [VP, P(C.c_double), C.c_size_t]),
    "orc_model_predict_raw": (C.c_double, [VP, P(_abi.Dataset), P(C.c_double)]),
    "orc_last_error": (C.c_char_p, []),
}

_lib = None


def build():
    if not (ROOT / "oracle").exists():
        return
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE.exists() or ORACLE.stat().st_mtime < (ROOT / "oracle" / "oracle.cpp").stat().st_mtime:
            build()
        _lib = C.CDLL(str(ORACLE))
        for name, (res, args) in _SIGS.items():
            f = getattr(_lib, name)
            f.restype, f.argtypes = res, args
    return _lib


def _p(arr, ctype):
    return arr.ctypes.data_as(P(ctype))


def quant_spec(max_abs_grad, max_hess, constant_hessian, num_bins, stochastic, seed, iteration) -> _abi.QuantSpec:
    s = _abi.QuantSpec()
    has = constant_hessian is not None
    lib().orc_quant_spec(max_abs_grad, max_hess, int(has), constant_hessian if has else 0.0, num_bins,
                         int(stochastic), seed, iteration, C.byref(s))
    return s


def quantize(spec, grad, hess, row_offset=0) -> np.ndarray:
    g = np.ascontiguousarray(grad, dtype=np.float32)
    h = np.ascontiguousarray(hess, dtype=np.float32)
    out = np.empty(len(g), dtype=np.int32)
    lib().orc_quantize(C.byref(spec), _p(g, C.c_float), _p(h, C.c_float), len(g), row_offset, _p(out, C.c_int32))
    return out


def unpack(packed: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    packed = np.asarray(packed, dtype=np.int32)
    g = (packed.astype(np.uint32) & 0xFFFF).astype(np.uint16).astype(np.int16).astype(np.int64)
    h = (packed.astype(np.int64) - g) >> 16
    return g, h


def histogram(data, packed, rows, used=None, max_quant=4) -> np.ndarray:
    d = data.c_struct()
    pk = np.ascontiguousarray(packed, dtype=np.int32)
    r = np.ascontiguousarray(rows, dtype=np.uint32)
    out = np.empty(2 * data.total_bins)
    u = None if used is None else np.ascontiguousarray(used, dtype=np.uint8)
    code = lib().orc_histogram(C.byref(d), _p(pk, C.c_int32), max_quant, _p(r, C.c_uint32), len(r),
                               None if u is None else _p(u, C.c_uint8), _p(out, C.c_double))
    assert code == 0, lib().orc_last_error()
    return out


def partition(data, split, rows) -> tuple[int, np.ndarray]:
    d = data.c_struct()
    r = np.array(rows, dtype=np.uint32)
    left = lib().orc_partition(C.byref(d), C.byref(split), _p(r, C.c_uint32), len(r))
    return left, r


def gradients(objective, scores, label, weight=None, sigmoid=1.0):
    o = _abi.Objective(objective, 0, sigmoid)
    s = np.ascontiguousarray(scores, dtype=np.float32)
    lb = np.ascontiguousarray(label, dtype=np.float32)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    g, h = np.empty(len(s), dtype=np.float32), np.empty(len(s), dtype=np.float32)
    lib().orc_gradients(C.byref(o), _p(s, C.c_float), _p(lb, C.c_float), None if w is None else _p(w, C.c_float),
                        len(s), _p(g, C.c_float), _p(h, C.c_float))
    return g, h


def lambdarank_gradients(params: _abi.Params, label, scores, query_boundaries, weight=None):
    """objective/lambdarank.rs gradients of every query at `scores`: (grad, hess) f32, or raises on rejected
    labels or queries."""
    label = np.ascontiguousarray(label, dtype=np.float32)
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    qb = np.ascontiguousarray(query_boundaries, dtype=np.uint32)
    d = _abi.Dataset()
    d.num_rows, d.num_queries = len(label), len(qb) - 1
    d.label = _p(label, C.c_float)
    d.query_boundaries = _p(qb, C.c_uint32)
    w = None
    if weight is not None:
        w = np.ascontiguousarray(weight, dtype=np.float32)
        d.weight = _p(w, C.c_float)
    grad = np.full(len(label), np.nan, dtype=np.float32)
    hess = np.full(len(label), np.nan, dtype=np.float32)
    code = lib().orc_lambdarank_gradients(C.byref(params), C.byref(d), _p(scores, C.c_float), _p(grad, C.c_float),
                                          _p(hess, C.c_float))
    if code != 0:
        raise ValueError(lib().orc_last_error().decode())
    return grad, hess


def lambdarank_max_dcg(k, labels, gain) -> float:
    labels = np.ascontiguousarray(labels, dtype=np.float32)
    gain = np.ascontiguousarray(gain, dtype=np.float64)
    return lib().orc_lambdarank_max_dcg(k, _p(labels, C.c_float), len(labels), _p(gain, C.c_double), len(gain))


def lambdarank_sigmoid(sigmoid: float, delta: float) -> float:
    return lib().orc_lambdarank_sigmoid(sigmoid, delta)


def leaf_sums(grad, hess, partition_rows, leaves, gs, hs) -> np.ndarray:
    g = np.ascontiguousarray(grad, dtype=np.float32)
    h = np.ascontiguousarray(hess, dtype=np.float32)
    pr = np.ascontiguousarray(partition_rows, dtype=np.uint32)
    arr = (_abi.LeafRange * max(len(leaves), 1))(*[_abi.LeafRange(b, c) for b, c in leaves])
    out = np.zeros(2 * len(leaves), dtype=np.int64)
    lib().orc_leaf_sums(_p(g, C.c_float), _p(h, C.c_float), _p(pr, C.c_uint32), arr, len(leaves), gs, hs,
                        _p(out, C.c_int64))
    return out.reshape(-1, 2)


def add_tree(data, nodes, leaf_values, scores) -> np.ndarray:
    d = data.c_struct()
    arr = (_abi.DeviceNode * max(len(nodes), 1))(*nodes)
    lv = np.ascontiguousarray(leaf_values, dtype=np.float32)
    s = np.array(scores, dtype=np.float32)
    code = lib().orc_add_tree(C.byref(d), arr, len(nodes), _p(lv, C.c_float), len(lv), _p(s, C.c_float))
    assert code == 0, lib().orc_last_error()
    return s


def value_to_bin(upper_bounds, nan_bin, value) -> int:
    ub = np.ascontiguousarray(upper_bounds, dtype=np.float64)
    return int(lib().orc_value_to_bin(_p(ub, C.c_double), len(ub), int(nan_bin), float(value)))


def bin_rows(values: np.ndarray, features, groups) -> list[np.ndarray]:
    """data/binning.rs bin_rows of a C- or Fortran-ordered f32/f64 matrix into each group's rows."""
    from silvic_b200.dataset import BinnedDataset

    a = np.asarray(values)
    if not (a.flags.c_contiguous or a.flags.f_contiguous):
        a = np.ascontiguousarray(a)
    rows, cols = a.shape
    shell = BinnedDataset(rows, 0, list(features), [g.__class__(g.features, g.row_stride, g.hist_offset, g.total_bins,
                                                                np.zeros((0, g.row_stride), np.uint8)) for g in groups],
                          0, np.zeros(0, np.float32))
    d = shell.c_struct()
    outs = [np.zeros((rows, g.row_stride), dtype=np.uint8) for g in groups]
    ptrs = (P(C.c_uint8) * max(len(outs), 1))(*[_p(o, C.c_uint8) for o in outs])
    code = lib().orc_bin_rows(C.c_void_p(a.ctypes.data), a.itemsize, rows, cols, int(a.flags.c_contiguous),
                              d.features, len(features), d.groups, len(groups), ptrs)
    assert code == 0, code
    return outs


def reset_partition(bag, num_rows, row_offset=0) -> np.ndarray:
    out = np.empty(num_rows, dtype=np.uint32)
    k = lib().orc_reset_partition(C.byref(bag), num_rows, row_offset, _p(out, C.c_uint32))
    return out[:k]


def find_best_split(data, hist, evaluate, sums, scale, cfg) -> tuple[_abi.SplitInfo, np.ndarray]:
    d = data.c_struct()
    h = np.ascontiguousarray(hist, dtype=np.float64)
    ev = np.ascontiguousarray(evaluate, dtype=np.uint8)
    info = _abi.SplitInfo()
    spl = np.zeros(len(ev), dtype=np.uint8)
    code = lib().orc_find_best_split(C.byref(d), _p(h, C.c_double), _p(ev, C.c_uint8), sums[0], sums[1], sums[2],
                                     scale[0], scale[1], C.byref(cfg), C.byref(info), _p(spl, C.c_uint8))
    assert code == 0, lib().orc_last_error()
    return info, spl


def feature_mask(data, fraction, seed, iteration) -> np.ndarray:
    d = data.c_struct()
    out = np.zeros(len(data.features), dtype=np.uint8)
    lib().orc_feature_mask(C.byref(d), fraction, seed, iteration, _p(out, C.c_uint8))
    return out


OP_NAMES = ("gradients", "quantize", "histogram", "split_search", "partition", "leaf_sums", "add_tree")


class OracleModel:
    def __init__(self, trees, init_score, seconds, op_seconds=None):
        self.trees, self.init_score, self.iteration_seconds = trees, init_score, seconds
        self.op_seconds = dict(zip(OP_NAMES, op_seconds or []))


def train(shards, params: _abi.Params) -> OracleModel:
    """Trains on the row shards as that many ranks (one shard: one rank)."""
    structs = [s.c_struct() for s in shards]
    arr = (_abi.Dataset * len(structs))(*structs)
    m = C.c_void_p()
    code = lib().orc_train(arr, len(structs), C.byref(params), C.byref(m))
    assert code == 0, lib().orc_last_error()
    try:
        trees = []
        for i in range(lib().orc_model_num_trees(m)):
            v = _abi.TreeView()
            lib().orc_model_tree(m, i, C.byref(v))
            trees.append(Tree.from_view(v))
        secs = (C.c_double * 100000)()
        k = lib().orc_model_iteration_seconds(m, secs, 100000)
        ops = (C.c_double * 16)()
        kops = lib().orc_model_op_seconds(m, ops, 16)
        return OracleModel(trees, lib().orc_model_init_score(m), list(secs[:k]), list(ops[:kops]))
    finally:
        lib().orc_model_free(m)


class OracleTrainer:
    """An oracle training run whose model stays open for prediction (Model::predict_raw_row, model/predict.rs:19-23,
    restated in oracle.cpp): `trees`, `init_score`, `predict_raw(row)` on raw f64 feature values."""

    def __init__(self, shards, params: _abi.Params):
        self._structs = [s.c_struct() for s in shards]
        arr = (_abi.Dataset * len(self._structs))(*self._structs)
        self._m = C.c_void_p()
        code = lib().orc_train(arr, len(self._structs), C.byref(params), C.byref(self._m))
        assert code == 0, lib().orc_last_error()
        self.trees = []
        for i in range(lib().orc_model_num_trees(self._m)):
            v = _abi.TreeView()
            lib().orc_model_tree(self._m, i, C.byref(v))
            self.trees.append(Tree.from_view(v))
        self.init_score = lib().orc_model_init_score(self._m)

    def predict_raw(self, row) -> float:
        r = np.ascontiguousarray(row, dtype=np.float64)
        return lib().orc_model_predict_raw(self._m, C.byref(self._structs[0]), _p(r, C.c_double))

    def close(self):
        if self._m:
            lib().orc_model_free(self._m)
            self._m = None

    def __del__(self):
        self.close()


def default_params(**overrides) -> _abi.Params:
    """sb2_default_params' defaults (crates/silvic-core/src/config.rs:123-165) without loading the CUDA library."""
    p = _abi.Params()
    defaults = dict(objective=0, num_iterations=100, learning_rate=0.1, num_leaves=31, max_depth=-1,
                    min_data_in_leaf=20, min_sum_hessian_in_leaf=1e-3, lambda_l1=0.0, lambda_l2=0.0,
                    min_gain_to_split=0.0, bagging_fraction=1.0, bagging_freq=0, bagging_seed=3,
                    feature_fraction=1.0, feature_fraction_seed=2, data_random_seed=1, boost_from_average=1,
                    use_quantized_grad=1, sigmoid=1.0, num_grad_quant_bins=4, quant_train_renew_leaf=1,
                    stochastic_rounding=1, lambdarank_norm=1, lambdarank_truncation_level=30,
                    max_cat_to_onehot=4, max_cat_threshold=32, cat_l2=10.0, cat_smooth=10.0,
                    min_data_per_group=100)
    defaults.update(overrides)
    for k, v in defaults.items():
        setattr(p, k, v)
    return p


def trees_equal(a: Tree, b: Tree) -> list[str]:
    """Field names where two trees differ bit for bit (NaN equal to NaN)."""
    diffs = []
    if a.num_leaves != b.num_leaves:
        return ["num_leaves"]
    if a.shrinkage != b.shrinkage:
        diffs.append("shrinkage")
    for name in Tree.FIELDS:
        x, y = np.asarray(getattr(a, name)), np.asarray(getattr(b, name))
        if x.shape != y.shape or not np.array_equal(x.view(np.uint8), y.view(np.uint8)):
            diffs.append(name)
    return diffs
