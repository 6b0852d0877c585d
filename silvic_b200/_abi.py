"""ctypes mirror of include/silvic_b200.h and the loader of the compiled backend.

The library is built in-tree (silvic_b200/_lib/libsilvic_b200.so, see build.py). Loading fails loudly when it is
missing: there is no CPU fallback for anything this package computes.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "_lib" / "libsilvic_b200.so"

OK, ECONFIG, EDATA, EINTERNAL, EDEVICE, ECOLLECTIVE, EMODEL, EUNSUPPORTED = range(8)
NUMERICAL, CATEGORICAL, TRIVIAL = 0, 1, 2
REGRESSION, BINARY, LAMBDARANK = 0, 1, 2
EXCHANGE_AUTO, EXCHANGE_NCCL = 0, 1
LEFT, RIGHT = 0, 1

ERROR_KINDS = {
    ECONFIG: "config",
    EDATA: "data",
    EINTERNAL: "internal",
    EDEVICE: "device",
    ECOLLECTIVE: "collective",
    EMODEL: "model",
    EUNSUPPORTED: "unsupported",
}


class Feature(C.Structure):
    _fields_ = [
        ("num_bins", C.c_uint32),
        ("group", C.c_uint32),
        ("column", C.c_uint32),
        ("hist_offset", C.c_uint32),
        ("kind", C.c_uint32),
        ("nan_bin", C.c_uint32),
        ("upper_bounds", C.POINTER(C.c_double)),
        ("num_upper_bounds", C.c_uint32),
        ("pad_", C.c_uint32),
        ("min_value", C.c_double),
        ("max_value", C.c_double),
        ("categories", C.POINTER(C.c_int32)),
        ("num_categories", C.c_uint32),
        ("pad2_", C.c_uint32),
    ]


class Group(C.Structure):
    _fields_ = [
        ("data", C.POINTER(C.c_uint8)),
        ("row_stride", C.c_uint32),
        ("hist_offset", C.c_uint32),
        ("total_bins", C.c_uint32),
        ("num_features", C.c_uint32),
        ("features", C.POINTER(C.c_uint32)),
    ]


class Dataset(C.Structure):
    _fields_ = [
        ("num_rows", C.c_uint64),
        ("row_offset", C.c_uint64),
        ("num_features", C.c_uint32),
        ("num_groups", C.c_uint32),
        ("total_bins", C.c_uint32),
        ("num_queries", C.c_uint32),
        ("features", C.POINTER(Feature)),
        ("groups", C.POINTER(Group)),
        ("label", C.POINTER(C.c_float)),
        ("weight", C.POINTER(C.c_float)),
        ("query_boundaries", C.POINTER(C.c_uint32)),
    ]


class Objective(C.Structure):
    _fields_ = [("kind", C.c_int32), ("pad_", C.c_int32), ("sigmoid", C.c_double), ("lambdarank_norm", C.c_int32),
                ("lambdarank_truncation_level", C.c_uint32), ("label_gain", C.POINTER(C.c_double)),
                ("num_label_gain", C.c_uint32), ("pad2_", C.c_uint32)]


class LeafRange(C.Structure):
    _fields_ = [("begin", C.c_uint32), ("count", C.c_uint32)]


class BinSplit(C.Structure):
    _fields_ = [("group", C.c_uint32), ("column", C.c_uint32), ("left_bins", C.c_uint32 * 8)]


class DeviceNode(C.Structure):
    _fields_ = [("split", BinSplit), ("left", C.c_int32), ("right", C.c_int32)]


class QuantSpec(C.Structure):
    _fields_ = [
        ("inv_grad_scale", C.c_float),
        ("inv_hess_scale", C.c_float),
        ("grad_scale", C.c_double),
        ("hess_scale", C.c_double),
        ("grad_max_q", C.c_int32),
        ("hess_max_q", C.c_int32),
        ("constant_hessian", C.c_int32),
        ("stochastic", C.c_int32),
        ("seed", C.c_uint32),
        ("iteration", C.c_uint32),
    ]


class GradientStats(C.Structure):
    _fields_ = [("max_abs_grad", C.c_double), ("max_hess", C.c_double)]


class BagSpec(C.Structure):
    _fields_ = [("kind", C.c_int32), ("seed", C.c_uint32), ("round", C.c_uint32), ("pad_", C.c_uint32),
                ("fraction", C.c_double)]


class SplitConfig(C.Structure):
    _fields_ = [
        ("min_data_in_leaf", C.c_int64),
        ("min_sum_hessian_in_leaf", C.c_double),
        ("lambda_l1", C.c_double),
        ("lambda_l2", C.c_double),
        ("min_gain_to_split", C.c_double),
        ("min_data_per_group", C.c_int64),
        ("cat_l2", C.c_double),
        ("cat_smooth", C.c_double),
        ("max_cat_to_onehot", C.c_int32),
        ("max_cat_threshold", C.c_int32),
    ]


class SplitInfo(C.Structure):
    _fields_ = [
        ("found", C.c_int32),
        ("feature", C.c_int32),
        ("gain", C.c_double),
        ("threshold", C.c_uint32),
        ("default_left", C.c_int32),
        ("left_grad", C.c_double),
        ("left_hess", C.c_double),
        ("left_count", C.c_int64),
        ("right_grad", C.c_double),
        ("right_hess", C.c_double),
        ("right_count", C.c_int64),
        ("left_output", C.c_double),
        ("right_output", C.c_double),
        ("categorical", C.c_int32),
        ("pad_", C.c_int32),
        ("cat_bins", C.c_uint32 * 8),
    ]

    def as_tuple(self):
        """Every field's value (arrays as tuples), for comparisons."""
        return tuple(tuple(v) if isinstance(v, C.Array) else v
                     for v in (getattr(self, name) for name, _ in self._fields_))


class Params(C.Structure):
    _fields_ = [
        ("objective", C.c_int32),
        ("num_iterations", C.c_int32),
        ("learning_rate", C.c_double),
        ("num_leaves", C.c_int32),
        ("max_depth", C.c_int32),
        ("min_data_in_leaf", C.c_int64),
        ("min_sum_hessian_in_leaf", C.c_double),
        ("lambda_l1", C.c_double),
        ("lambda_l2", C.c_double),
        ("min_gain_to_split", C.c_double),
        ("bagging_fraction", C.c_double),
        ("bagging_freq", C.c_int32),
        ("bagging_seed", C.c_uint32),
        ("feature_fraction", C.c_double),
        ("feature_fraction_seed", C.c_uint32),
        ("data_random_seed", C.c_uint32),
        ("boost_from_average", C.c_int32),
        ("use_quantized_grad", C.c_int32),
        ("sigmoid", C.c_double),
        ("num_grad_quant_bins", C.c_int32),
        ("quant_train_renew_leaf", C.c_int32),
        ("stochastic_rounding", C.c_int32),
        ("pad_", C.c_int32),
        ("lambdarank_norm", C.c_int32),
        ("lambdarank_truncation_level", C.c_uint32),
        ("label_gain", C.POINTER(C.c_double)),
        ("num_label_gain", C.c_uint32),
        ("pad2_", C.c_uint32),
        ("max_cat_to_onehot", C.c_int32),
        ("max_cat_threshold", C.c_int32),
        ("cat_l2", C.c_double),
        ("cat_smooth", C.c_double),
        ("min_data_per_group", C.c_int64),
    ]


class TreeView(C.Structure):
    _fields_ = [
        ("num_leaves", C.c_int32),
        ("pad_", C.c_int32),
        ("shrinkage", C.c_double),
        ("split_feature", C.POINTER(C.c_int32)),
        ("split_gain", C.POINTER(C.c_float)),
        ("threshold", C.POINTER(C.c_double)),
        ("threshold_bin", C.POINTER(C.c_uint32)),
        ("decision_type", C.POINTER(C.c_int8)),
        ("left_child", C.POINTER(C.c_int32)),
        ("right_child", C.POINTER(C.c_int32)),
        ("leaf_value", C.POINTER(C.c_double)),
        ("leaf_weight", C.POINTER(C.c_double)),
        ("leaf_count", C.POINTER(C.c_int64)),
        ("internal_value", C.POINTER(C.c_double)),
        ("internal_weight", C.POINTER(C.c_double)),
        ("internal_count", C.POINTER(C.c_int64)),
        ("cat_bins", C.POINTER(C.c_uint32)),
    ]


# Exported functions: name -> (restype, argtypes). Every symbol the header declares.
P = C.POINTER
VP = C.c_void_p
SIGNATURES = {
    "sb2_global_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "sb2_default_params": (None, [P(Params)]),
    "sb2_create": (C.c_int, [C.c_int, P(VP)]),
    "sb2_destroy": (C.c_int, [VP]),
    "sb2_last_error": (C.c_int, [VP, C.c_char_p, C.c_size_t]),
    "sb2_name": (C.c_int, [VP, C.c_char_p, C.c_size_t]),
    "sb2_load": (C.c_int, [VP, P(Dataset), P(Objective)]),
    "sb2_init_scores": (C.c_int, [VP, C.c_int, C.c_double]),
    "sb2_compute_gradients": (C.c_int, [VP, P(GradientStats)]),
    "sb2_quantize": (C.c_int, [VP, P(QuantSpec)]),
    "sb2_reset_partition": (C.c_int, [VP, P(BagSpec), P(C.c_uint32)]),
    "sb2_set_histogram_features": (C.c_int, [VP, P(C.c_uint8), C.c_size_t]),
    "sb2_histogram": (C.c_int, [VP, LeafRange, C.c_int, P(C.c_double), C.c_size_t]),
    "sb2_partition": (C.c_int, [VP, LeafRange, P(BinSplit), P(C.c_uint32)]),
    "sb2_partition_and_histogram": (C.c_int, [VP, LeafRange, P(BinSplit), C.c_int, C.c_int, P(C.c_double),
                                              C.c_size_t, P(C.c_uint32)]),
    "sb2_leaf_sums": (C.c_int, [VP, P(LeafRange), C.c_size_t, C.c_float, C.c_float, P(C.c_int64)]),
    "sb2_add_tree": (C.c_int, [VP, P(DeviceNode), C.c_size_t, P(C.c_float), C.c_size_t]),
    "sb2_scores": (C.c_int, [VP, C.c_int, P(C.c_float), C.c_size_t]),
    "sb2_read_partition": (C.c_int, [VP, P(C.c_uint32), C.c_size_t]),
    "sb2_read_packed": (C.c_int, [VP, P(C.c_int32), C.c_size_t]),
    "sb2_write_gradients": (C.c_int, [VP, P(C.c_float), P(C.c_float), C.c_size_t]),
    "sb2_read_gradients": (C.c_int, [VP, P(C.c_float), P(C.c_float), C.c_size_t]),
    "sb2_find_best_split": (C.c_int, [VP, P(C.c_double), C.c_size_t, P(C.c_uint8), C.c_double, C.c_double,
                                      C.c_int64, C.c_double, C.c_double, P(SplitConfig), P(SplitInfo),
                                      P(C.c_uint8)]),
    "sb2_find_best_split_noalloc": (C.c_int, [VP, VP, C.c_size_t, VP, C.c_double, C.c_double, C.c_int64,
                                              C.c_double, C.c_double, P(SplitConfig), VP, VP]),
    "sb2_check_division": (C.c_int, [VP, C.c_uint64, C.c_uint32, P(C.c_uint64)]),
    "sb2_time_histogram": (C.c_int, [VP, C.c_uint64, C.c_int, P(C.c_double)]),
    "sb2_time_shared_adds": (C.c_int, [VP, C.c_int, P(C.c_double), P(C.c_double)]),
    "sb2_profile_train": (C.c_int, [VP, P(Params), C.c_double, P(C.c_double), C.c_size_t, P(VP)]),
    "sb2_profile_steps": (C.c_int, [VP, P(Params), C.c_double, P(C.c_double), C.c_size_t, P(C.c_size_t)]),
    "sb2_nccl_unique_id": (C.c_int, [P(C.c_uint8), C.c_size_t]),
    "sb2_join_ranks": (C.c_int, [VP, P(C.c_uint8), C.c_size_t, C.c_int, C.c_int]),
    "sb2_set_rank_exchange": (C.c_int, [VP, C.c_int]),
    "sb2_set_dominant_share": (C.c_int, [VP, C.c_double]),
    "sb2_test_unanswered_peer": (C.c_int, [VP, C.c_uint32]),
    "sb2_train": (C.c_int, [VP, P(Params), C.c_double, P(VP)]),
    "sb2_boost_from_average": (C.c_int, [P(Params), P(C.c_float), P(C.c_float), C.c_size_t, P(C.c_double)]),
    "sb2_model_free": (C.c_int, [VP]),
    "sb2_model_num_trees": (C.c_int, [VP]),
    "sb2_model_tree": (C.c_int, [VP, C.c_int, P(TreeView)]),
    "sb2_model_iteration_seconds": (C.c_int, [VP, P(C.c_double), C.c_size_t]),
    "sb2_model_tree_seconds": (C.c_int, [VP, P(C.c_double), C.c_size_t]),
    "sb2_bin_dense": (C.c_int, [VP, VP, C.c_int, C.c_uint64, C.c_uint32, C.c_int, P(Feature), C.c_uint32, P(Group),
                                C.c_uint32, P(P(C.c_uint8))]),
}

_lib = None


def load_library(path: Path | None = None) -> C.CDLL:
    """The backend library with every signature set; raises if it was not built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    target = Path(path) if path else LIBRARY
    if not target.exists():
        raise RuntimeError(
            f"silvic_b200: the CUDA backend {target} is not built (run `python silvic_b200/build.py`); "
            "this package has no CPU fallback")
    lib = C.CDLL(str(target))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if path is None:
        _lib = lib
    return lib


class SilvicError(RuntimeError):
    """A failed backend call; `kind` names the SilvicError variant (config, data, device, ...)."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.kind = ERROR_KINDS.get(code, "unknown")
        super().__init__(f"{self.kind} error: {message}")


def global_error() -> str:
    buf = C.create_string_buffer(4096)
    load_library().sb2_global_error(buf, len(buf))
    return buf.value.decode()
