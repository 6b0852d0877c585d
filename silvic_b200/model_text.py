"""LightGBM 3.3.5's model file, as silvic writes and reads it (crates/silvic-core/src/model/text.rs).

Writing follows `Model::to_lightgbm_string` (text.rs:48-70): the header (`GBDT::SaveModelToString`), one
`Tree=<i>` block per tree (`Tree::ToString`), `end of trees`, the split-count feature importances, the `parameters:`
block and the `pandas_categorical:` line. `threshold`, `leaf_value` and `leaf_weight` print with C's `%.17g` (exact
round trip); `split_gain`, `internal_value`, `internal_weight`, `shrinkage` and the sigmoid with `%g` (text.rs:1-15,
config.rs:501-531). Python's `%` float formatting follows C's `printf` rules (correctly rounded digits, trailing
zeros removed, two-digit exponents, `inf`, `nan`, `-0`), so the digits are the ones glibc prints.

Parsing follows `Model::from_lightgbm_string` (text.rs:72-96, 197-531): LightGBM 3.x and 4.x files, header lines it
has no use for skipped, the `parameters:` block kept line for line, and every tree checked to be one tree rooted at
node 0 so that prediction cannot loop on a corrupt file.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import _abi

MODEL_VERSION = "v3"
END_OF_TREES = "end of trees"
PANDAS_CATEGORICAL_KEY = "pandas_categorical:"
CATEGORICAL_MASK = 1
DEFAULT_LEFT_MASK = 2
REGRESSION_NAMES = ("regression", "regression_l2", "l2", "mean_squared_error", "mse", "l2_root",
                    "root_mean_squared_error", "rmse")
MULTICLASS_NAMES = ("multiclass", "softmax", "multiclassova", "multiclass_ova", "ova", "ovr")


class ModelFormatError(ValueError):
    """A malformed model file (SilvicError::Model)."""


class UnsupportedModel(ValueError):
    """A valid LightGBM file of a kind silvic does not predict (SilvicError::Unsupported)."""


def format_g(value: float, precision: int = 6) -> str:
    """C `printf("%.<precision>g")` (config.rs:507-531)."""
    return "%.*g" % (max(precision, 1), float(value))


def format_g17(value: float) -> str:
    return format_g(value, 17)


@dataclass
class TextTree:
    """One tree in LightGBM's arrays (tree.rs:47-73); a one-leaf tree has only `leaf_value` and `shrinkage`."""

    num_leaves: int = 1
    num_cat: int = 0
    split_feature: list = field(default_factory=list)
    split_gain: list = field(default_factory=list)      # f32 values
    threshold: list = field(default_factory=list)
    decision_type: list = field(default_factory=list)
    left_child: list = field(default_factory=list)
    right_child: list = field(default_factory=list)
    leaf_value: list = field(default_factory=lambda: [0.0])
    leaf_weight: list = field(default_factory=list)
    leaf_count: list = field(default_factory=list)
    internal_value: list = field(default_factory=list)
    internal_weight: list = field(default_factory=list)
    internal_count: list = field(default_factory=list)
    cat_boundaries: list = field(default_factory=list)
    cat_threshold: list = field(default_factory=list)
    shrinkage: float = 1.0

    def leaf_index(self, row) -> int:
        """`Tree::GetLeaf` (predict.rs): numerical and categorical decisions with LightGBM's missing-value rules."""
        if self.num_leaves <= 1:
            return 0
        zero = float(np.float32(1e-35))
        node = 0
        while node >= 0:
            value = float(row[self.split_feature[node]])
            dt = int(self.decision_type[node])
            if self.num_cat > 0 and dt & CATEGORICAL_MASK:
                left = self._categorical_left(node, value)
            else:
                missing = (dt >> 2) & 3
                if abs(value) <= zero:
                    value = 0.0
                if math.isnan(value) and missing != 2:
                    value = 0.0
                is_missing = (missing == 1 and -zero <= value <= zero) or (missing == 2 and math.isnan(value))
                left = bool(dt & DEFAULT_LEFT_MASK) if is_missing else value <= self.threshold[node]
            node = int(self.left_child[node] if left else self.right_child[node])
        return ~node

    def _categorical_left(self, node: int, value: float) -> bool:
        """`CategoricalDecision` (predict.rs:156-173): NaN and negative values go right, others left when their bit
        is set (the cast truncates toward zero; a category past every bitset goes right)."""
        if abs(value) <= float(np.float32(1e-35)):
            value = 0.0
        if math.isnan(value) or int(value) < 0:
            return False
        category = int(value)
        k = int(self.threshold[node])
        lo, hi = self.cat_boundaries[k], self.cat_boundaries[k + 1]
        word = category // 32
        if word >= hi - lo:
            return False
        return bool((int(self.cat_threshold[lo + word]) >> (category % 32)) & 1)

    def lines(self) -> str:
        """`Tree::ToString` (text.rs:159-199): every list clipped to the entries LightGBM prints."""
        leaves = self.num_leaves
        nodes = max(leaves - 1, 0)
        stats = leaves if leaves > 1 else 0
        out = [f"num_leaves={leaves}", f"num_cat={self.num_cat}"]

        def put(key, values, fmt):
            out.append(key + "=" + " ".join(fmt(v) for v in list(values)[:]))

        put("split_feature", self.split_feature[:nodes], lambda v: str(int(v)))
        put("split_gain", self.split_gain[:nodes], lambda v: format_g(float(np.float32(v))))
        put("threshold", self.threshold[:nodes], format_g17)
        put("decision_type", self.decision_type[:nodes], lambda v: str(int(v)))
        put("left_child", self.left_child[:nodes], lambda v: str(int(v)))
        put("right_child", self.right_child[:nodes], lambda v: str(int(v)))
        put("leaf_value", self.leaf_value[:leaves], format_g17)
        put("leaf_weight", self.leaf_weight[:stats], format_g17)
        put("leaf_count", self.leaf_count[:stats], lambda v: str(int(v)))
        put("internal_value", self.internal_value[:nodes], format_g)
        put("internal_weight", self.internal_weight[:nodes], format_g)
        put("internal_count", self.internal_count[:nodes], lambda v: str(int(v)))
        if self.num_cat > 0:
            put("cat_boundaries", self.cat_boundaries[: self.num_cat + 1], lambda v: str(int(v)))
            put("cat_threshold", self.cat_threshold, lambda v: str(int(v)))
        out.append("is_linear=0")
        out.append(f"shrinkage={format_g(self.shrinkage)}")
        return "\n".join(out) + "\n\n"


@dataclass
class TextModel:
    """`Model` (model/mod.rs:20-40): objective, feature names and infos, trees, the `parameters:` block."""

    objective: str                       # "regression", "binary" or "lambdarank"
    feature_names: list
    feature_infos: list
    trees: list
    sigmoid: float = 1.0                 # binary only
    parameters: list = field(default_factory=list)  # (key, value) strings
    pandas_categorical: str | None = None

    # ---- writing -------------------------------------------------------------------------------------------
    def split_importance(self) -> list:
        counts = [0] * len(self.feature_names)
        for t in self.trees:
            for f in t.split_feature[: max(t.num_leaves - 1, 0)]:
                counts[int(f)] += 1
        return counts

    def gain_importance(self) -> list:
        gains = [0.0] * len(self.feature_names)
        for t in self.trees:
            for f, g in zip(t.split_feature[: max(t.num_leaves - 1, 0)], t.split_gain):
                gains[int(f)] += float(np.float32(g))
        return gains

    def to_string(self) -> str:
        """`Model::to_lightgbm_string` (text.rs:48-70), byte for byte."""
        blocks = [f"Tree={i}\n" + t.lines() + "\n" for i, t in enumerate(self.trees)]
        if self.objective == "binary":
            objective = f"binary sigmoid:{format_g(self.sigmoid)}"
        else:
            objective = self.objective
        head = ["tree", f"version={MODEL_VERSION}", "num_class=1", "num_tree_per_iteration=1", "label_index=0",
                f"max_feature_idx={len(self.feature_names) - 1}", f"objective={objective}",
                "feature_names=" + " ".join(self.feature_names), "feature_infos=" + " ".join(self.feature_infos),
                "tree_sizes=" + " ".join(str(len(b)) for b in blocks)]
        out = "\n".join(head) + "\n\n" + "".join(blocks) + END_OF_TREES + "\n"
        # feature_importances: split counts above zero, stable-sorted by count descending (text.rs:122-136)
        counts = [(c, name) for c, name in zip(self.split_importance(), self.feature_names) if c > 0]
        counts.sort(key=lambda cn: -cn[0])
        out += "\nfeature_importances:\n" + "".join(f"{name}={c}\n" for c, name in counts)
        if self.parameters:
            out += "\nparameters:\n" + "".join(f"[{k}: {v}]\n" for k, v in self.parameters) + "\nend of parameters\n"
        out += "\n" + PANDAS_CATEGORICAL_KEY + (self.pandas_categorical or "null") + "\n"
        return out

    # ---- reading -------------------------------------------------------------------------------------------
    @staticmethod
    def from_string(text: str) -> "TextModel":
        """`Model::from_lightgbm_string` (text.rs:72-96)."""
        lines = text.splitlines()
        i = 0
        header = []
        while i < len(lines) and not lines[i].startswith("Tree=") and lines[i] != END_OF_TREES:
            if lines[i]:
                k, _, v = lines[i].partition("=")
                header.append((k, v))
            i += 1

        def get(key):
            for k, v in reversed(header):
                if k == key:
                    return v
            return None

        def require(key):
            v = get(key)
            if v is None:
                raise ModelFormatError(f"no {key} line")
            return v

        num_class = _number(require("num_class"), "num_class", int)
        per_iteration = _number(get("num_tree_per_iteration"), "num_tree_per_iteration", int) \
            if get("num_tree_per_iteration") is not None else num_class
        if num_class != 1 or per_iteration != 1:
            raise UnsupportedModel(f"multiclass models (num_class={num_class}, num_tree_per_iteration={per_iteration})")
        if get("average_output") is not None:
            raise UnsupportedModel("average_output (random forest) models")
        max_idx = _number(require("max_feature_idx"), "max_feature_idx", int)
        if max_idx < -1 or max_idx + 1 > 1 << 31:
            raise ModelFormatError(f"max_feature_idx={max_idx}")
        nf = max_idx + 1
        objective_line = get("objective")
        if objective_line is None:
            raise UnsupportedModel("models without an objective (trained with a custom objective)")
        objective, sigmoid = _parse_objective(objective_line)
        names = _words(require("feature_names"), "feature_names", nf)
        infos = _words(require("feature_infos"), "feature_infos", nf)
        sizes = get("tree_sizes")
        trees = []
        while i < len(lines):
            if not lines[i]:
                i += 1
                continue
            if not lines[i].startswith("Tree="):
                break
            i += 1
            fields = []
            while i < len(lines) and lines[i]:
                k, _, v = lines[i].partition("=")
                fields.append((k, v))
                i += 1
            try:
                trees.append(_parse_tree(fields, nf))
            except ModelFormatError as e:
                raise ModelFormatError(f"tree {len(trees)}: {e}") from None
        if sizes is not None and len([s for s in sizes.split(" ") if s]) != len(trees):
            raise ModelFormatError(f"tree_sizes lists {len([s for s in sizes.split(' ') if s])} trees, "
                                   f"the file has {len(trees)}")
        model = TextModel(objective, names, infos, trees, sigmoid)
        in_params = False
        for line in lines[i:]:
            if in_params:
                if line == "end of parameters":
                    in_params = False
                elif line:
                    if not (line.startswith("[") and line.endswith("]") and ": " in line):
                        raise ModelFormatError(f"parameter line `{line}` is not `[key: value]`")
                    k, _, v = line[1:-1].partition(": ")
                    model.parameters.append((k, v))
            elif line == "parameters:":
                in_params = True
            elif line.startswith(PANDAS_CATEGORICAL_KEY):
                value = line[len(PANDAS_CATEGORICAL_KEY):]
                model.pandas_categorical = None if value == "null" else value
        return model

    # ---- prediction ----------------------------------------------------------------------------------------
    def predict_raw_row(self, row, num_trees: int | None = None) -> float:
        """`Model::predict_raw_row` (predict.rs:19-23): the f64 sum of the first `num_trees` trees' leaf values."""
        total = 0.0
        for t in self.trees[: len(self.trees) if num_trees is None else num_trees]:
            total += float(t.leaf_value[t.leaf_index(row)])
        return total


def _number(text, what, kind):
    try:
        return kind(text.strip())
    except (ValueError, AttributeError):
        raise ModelFormatError(f"{what}: cannot parse `{text}`") from None


def _words(value: str, key: str, expected: int) -> list:
    words = [w for w in value.split(" ") if w]
    if len(words) != expected:
        raise ModelFormatError(f"{key} has {len(words)} entries, max_feature_idx says {expected}")
    return words


def _parse_objective(line: str):
    tokens = [t for t in line.split(" ") if t]
    name = tokens[0] if tokens else ""
    args = tokens[1:]
    if name in REGRESSION_NAMES:
        if "sqrt" in args:
            raise UnsupportedModel("regression with reg_sqrt")
        return "regression", 1.0
    if name == "binary":
        sig = next((a[len("sigmoid:"):] for a in args if a.startswith("sigmoid:")), None)
        value = _number(sig, "sigmoid", float) if sig is not None else None
        if value is None or not value > 0.0:
            raise ModelFormatError(f"binary objective needs sigmoid > 0, got `{line}`")
        return "binary", value
    if name == "lambdarank":
        return "lambdarank", 1.0
    if name in MULTICLASS_NAMES:
        raise UnsupportedModel(f"multiclass objective `{line}`")
    raise UnsupportedModel(f"objective `{line}`")


def _parse_tree(fields, num_features: int) -> TextTree:
    """`Tree::Tree(const char*)` (text.rs:412-452) with the structure checks of text.rs:454-520."""
    def get(key):
        for k, v in reversed(fields):
            if k == key:
                return v
        return None

    def lst(key, n, kind, default=False):
        v = get(key)
        if v is None:
            if default:
                return [kind(0)] * n
            raise ModelFormatError(f"no {key} field")
        vals = [_number(s, key, kind) for s in v.split(" ") if s]
        if len(vals) != n:
            raise ModelFormatError(f"{key} has {len(vals)} values, expected {n}")
        return vals

    if get("num_leaves") is None:
        raise ModelFormatError("no num_leaves field")
    leaves = _number(get("num_leaves"), "num_leaves", int)
    if leaves <= 0:
        raise ModelFormatError("num_leaves=0")
    if get("is_linear") is not None and get("is_linear").strip() != "0":
        raise UnsupportedModel("linear trees")
    if get("num_cat") is None:
        raise ModelFormatError("no num_cat field")
    num_cat = _number(get("num_cat"), "num_cat", int)
    if num_cat < 0 or num_cat >= 1 << 63:
        raise ModelFormatError(f"num_cat={num_cat}")
    t = TextTree()
    t.leaf_value = lst("leaf_value", leaves, float)
    t.shrinkage = _number(get("shrinkage"), "shrinkage", float) if get("shrinkage") is not None else 1.0
    if leaves == 1:
        return t
    nodes = leaves - 1
    t.num_leaves, t.num_cat = leaves, num_cat
    t.left_child = lst("left_child", nodes, int)
    t.right_child = lst("right_child", nodes, int)
    t.split_feature = lst("split_feature", nodes, int)
    t.threshold = lst("threshold", nodes, float)
    t.split_gain = [float(np.float32(g)) for g in lst("split_gain", nodes, float, True)]
    t.internal_count = lst("internal_count", nodes, int, True)
    t.internal_value = lst("internal_value", nodes, float, True)
    t.internal_weight = lst("internal_weight", nodes, float, True)
    t.leaf_weight = lst("leaf_weight", leaves, float, True)
    t.leaf_count = lst("leaf_count", leaves, int, True)
    t.decision_type = lst("decision_type", nodes, int, True)
    if num_cat > 0:
        t.cat_boundaries = lst("cat_boundaries", num_cat + 1, int)
        if t.cat_boundaries[-1] < 0:
            raise ModelFormatError("negative cat_boundaries")
        t.cat_threshold = lst("cat_threshold", t.cat_boundaries[-1], int)
    # every split reads a real feature; every categorical split names a bitset inside cat_threshold
    if any(a < 0 or a > b for a, b in zip(t.cat_boundaries, t.cat_boundaries[1:])):
        raise ModelFormatError("cat_boundaries are not ascending")
    for node, f in enumerate(t.split_feature):
        if not 0 <= f < num_features:
            raise ModelFormatError(f"node {node} splits on feature {f}")
        if num_cat > 0 and t.decision_type[node] & CATEGORICAL_MASK:
            th = t.threshold[node]
            if not (th >= 0.0 and int(th) < num_cat):
                raise ModelFormatError(f"node {node} names categorical bitset {th}")
    # one tree rooted at node 0: a child node has a higher index than its parent, every node and leaf reached once
    depth = [None] * nodes
    depth[0] = 0
    leaf_seen = [False] * leaves
    for node in range(nodes):
        if depth[node] is None:
            raise ModelFormatError(f"node {node} is unreachable")
        for child in (t.left_child[node], t.right_child[node]):
            if child >= 0:
                if child <= node or child >= nodes or depth[child] is not None:
                    raise ModelFormatError(f"node {node} has an invalid or repeated child {child}")
                depth[child] = depth[node] + 1
            else:
                leaf = ~child
                if leaf >= leaves or leaf_seen[leaf]:
                    raise ModelFormatError(f"node {node} has an invalid or repeated child {child}")
                leaf_seen[leaf] = True
    if not all(leaf_seen):
        raise ModelFormatError(f"leaf {leaf_seen.index(False)} is unreachable")
    return t


# ---- a trained model as a file ---------------------------------------------------------------------------

def model_parameters(params: _abi.Params) -> list:
    """`Params::model_parameters` (config.rs:444-498) for the parameters a device-trained model carries (lambdarank's
    three after the quantization ones, config.rs:486-493); the binning parameters the device trainer does not take
    keep the reference's defaults (config.rs:123-167)."""
    objective = {_abi.REGRESSION: "regression", _abi.BINARY: "binary"}.get(params.objective, "lambdarank")
    g = format_g
    out = [("boosting", "gbdt"), ("objective", objective), ("num_iterations", str(params.num_iterations)),
           ("learning_rate", g(params.learning_rate)), ("num_leaves", str(params.num_leaves)),
           ("max_depth", str(params.max_depth)), ("min_data_in_leaf", str(params.min_data_in_leaf)),
           ("min_sum_hessian_in_leaf", g(params.min_sum_hessian_in_leaf)),
           ("bagging_fraction", g(params.bagging_fraction)), ("bagging_freq", str(params.bagging_freq)),
           ("bagging_seed", str(params.bagging_seed)), ("feature_fraction", g(params.feature_fraction)),
           ("feature_fraction_seed", str(params.feature_fraction_seed)), ("lambda_l1", g(params.lambda_l1)),
           ("lambda_l2", g(params.lambda_l2)), ("min_gain_to_split", g(params.min_gain_to_split)),
           ("max_cat_threshold", str(params.max_cat_threshold)), ("cat_l2", g(params.cat_l2)),
           ("cat_smooth", g(params.cat_smooth)), ("max_cat_to_onehot", str(params.max_cat_to_onehot)),
           ("max_bin", "255"), ("min_data_in_bin", "3"), ("bin_construct_sample_cnt", "200000"),
           ("data_random_seed", "1"), ("boost_from_average", str(int(bool(params.boost_from_average)))),
           ("use_quantized_grad", str(int(bool(params.use_quantized_grad)))),
           ("num_grad_quant_bins", str(params.num_grad_quant_bins)),
           ("quant_train_renew_leaf", str(int(bool(params.quant_train_renew_leaf)))),
           ("stochastic_rounding", str(int(bool(params.stochastic_rounding))))]
    if objective == "lambdarank":
        if params.label_gain and params.num_label_gain:
            gains = [params.label_gain[i] for i in range(params.num_label_gain)]
        else:
            gains = [float((1 << i) - 1) for i in range(31)]  # config.rs:118-121
        out += [("lambdarank_truncation_level", str(params.lambdarank_truncation_level)),
                ("lambdarank_norm", str(int(bool(params.lambdarank_norm)))),
                ("label_gain", ",".join(g(v) for v in gains))]
    if objective != "regression":
        out.append(("sigmoid", g(params.sigmoid)))
    return out


def feature_info(meta) -> str:
    """`BinMapper::info_string` (bin_mapper.rs:362-377): `[min:max]`, `-1:c1:c2:...` (the "other" bin listed as
    category -1) or `none`."""
    if meta.is_trivial:
        return "none"
    if meta.kind == _abi.CATEGORICAL:
        return ":".join(["-1"] + [str(int(c)) for c in meta.categories])
    return f"[{format_g17(meta.min_value)}:{format_g17(meta.max_value)}]"


def to_bitset(values) -> list[int]:
    """`to_bitset` (tree.rs:230-237): the non-negative values as bits of u32 words, max / 32 + 1 words."""
    vals = [int(v) for v in values if int(v) >= 0]
    words = [0] * (max(vals, default=0) // 32 + 1)
    for v in vals:
        words[v // 32] |= 1 << (v % 32)
    return words


def _categorical_splits(tr, n: int, dataset):
    """A trained tree's categorical splits as LightGBM writes them (Tree::split_categorical, tree.rs:125-141): per
    categorical node in node order, the bitset of the categories of the bins it sends left, and the boundaries."""
    boundaries, words = [0], []
    for k in range(n):
        if not int(tr.decision_type[k]) & CATEGORICAL_MASK:
            continue
        meta = dataset.features[int(tr.split_feature[k])]
        bins = [b for b in range(1, meta.num_bins) if (int(tr.cat_bins[k][b // 32]) >> (b % 32)) & 1]
        bits = to_bitset(meta.categories[b - 1] for b in bins)
        if float(tr.threshold[k]) != len(boundaries) - 1:
            raise ModelFormatError(f"categorical node {k} has index {tr.threshold[k]}, not {len(boundaries) - 1}")
        words += bits
        boundaries.append(boundaries[-1] + len(bits))
    return len(boundaries) - 1, boundaries, words


def from_trained(model, dataset, params: _abi.Params) -> TextModel:
    """A device- (or oracle-) trained model (`silvic_b200.backend.Model`) as silvic's model file of the same
    training run (`boosting::train_from`, boosting.rs:151-190): feature names and infos from the dataset's features,
    the parameters of `params`."""
    objective = {_abi.REGRESSION: "regression", _abi.BINARY: "binary"}.get(params.objective, "lambdarank")
    trees = []
    for tr in model.trees:
        n = max(tr.num_leaves - 1, 0)
        num_cat, boundaries, words = _categorical_splits(tr, n, dataset)
        trees.append(TextTree(
            num_leaves=tr.num_leaves, num_cat=num_cat, split_feature=[int(v) for v in tr.split_feature[:n]],
            split_gain=[float(v) for v in tr.split_gain[:n]], threshold=[float(v) for v in tr.threshold[:n]],
            decision_type=[int(v) for v in tr.decision_type[:n]], left_child=[int(v) for v in tr.left_child[:n]],
            right_child=[int(v) for v in tr.right_child[:n]], leaf_value=[float(v) for v in tr.leaf_value],
            leaf_weight=[float(v) for v in tr.leaf_weight], leaf_count=[int(v) for v in tr.leaf_count],
            internal_value=[float(v) for v in tr.internal_value[:n]],
            internal_weight=[float(v) for v in tr.internal_weight[:n]],
            internal_count=[int(v) for v in tr.internal_count[:n]], shrinkage=float(tr.shrinkage),
            cat_boundaries=boundaries if num_cat else [], cat_threshold=words))
    return TextModel(objective, [m.name for m in dataset.features], [feature_info(m) for m in dataset.features],
                     trees, sigmoid=float(params.sigmoid), parameters=model_parameters(params))
