"""Benchmark: boosting iterations/s of silvic's quantized-histogram training on B200 (BASELINE.json's metric).

Default workload: BASELINE.json configs[3] ("c4"), the largest configuration that fits one B200 and the one the
scaling target names: L2 regression, 100,000,000 rows x 256 f32 features ~ N(0,1), target = a random 32-feature
linear function + N(0,1) noise, 255 bins, 255 leaves, quantized gradients (4 bins), 200 trees in a full job.
`--config` selects another configuration: c1 (configs[0]: 1M x 28 L2, 63 leaves, 100 trees), c2 (configs[1]:
10M x 100 binary, 255 leaves, 500 trees), c3 (configs[2]: 2M x 136 lambdarank over queries of Poisson(120) rows,
127 leaves, 300 trees) or c5 (configs[4]: 5M x 2000 binary, 63 bins, 80% of the features 95% zeros, 31 leaves,
200 trees). A "step" is one boosting iteration: gradients, quantization, a tree grown
split by split on the device (partition, smaller-child histogram, sibling subtraction, split scan, leaf choice),
leaf renewal and the score update.

Data are synthetic (BASELINE names no public dataset): every feature value is a pure function of (seed, global row,
feature) from silvic's counter hash, generated on the GPU, so any rank regenerates its own rows. Bin bounds are
equal-frequency cuts of the first 200,000 rows (bin_construct_sample_cnt's default sample size); the rows are binned
by the product's device binning (sb2_bin_dense, data::binning::bin_rows) into silvic's group layout (32 features of
255 bins per group). The binned matrix (c4: 25.6 GB; c2: 1 GB) is larger than the 126 MB L2, so no L2 flush is
needed between timed iterations.

Arms:
  default            the B200 backend. `value` = iterations/s from CUDA events around each iteration of the
                     device-resident trainer (inputs resident in HBM), max over ranks. `e2e` = the same metric for a
                     whole job through the reference-facing C ABI with host buffers: a fresh handle, sb2_load (the
                     host->device copy of the binned data), sb2_join_ranks (N>1), sb2_train of the config's full tree
                     count and the trees read back, wall clock, max over ranks; its one-time setup is reported apart.
                     `parity`: the first trees of the timed run against the CPU oracle's trees of the same dataset
                     (the whole dataset, on rank 0, at every N), field by field and as LightGBM model text.
  --impl reference   the CPU restatement of silvic-core's trainer (oracle/, "port") on this box's host cores.

Multi-GPU: one process per GPU (torchrun). Rows are sharded contiguously (strong scaling: the job is fixed); the
split steps exchange histograms inside the tree kernel over NVLink.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 20261107
SAMPLE_ROWS = 200_000
METRIC = "boosting iters/sec + histogram rows·feats/sec (HBM % peak) at 1/2/4/8 B200"
PARITY_TREES = 2  # trees of the timed run checked against the oracle's


@dataclass
class Config:
    name: str
    index: int            # position in BASELINE.json's configs
    rows: int
    objective: str
    max_bin: int
    num_leaves: int
    trees: int            # trees of the full job (the e2e run)
    kinds: list = field(default_factory=list)  # per feature: its synthetic distribution (column())
    # DRAM bytes (read + write) the tree kernel moved per training row in one launch, from an ncu capture of a
    # smaller case of the same workload (the traffic grows with the rows); None: not captured
    traffic_per_row: float | None = None

    @property
    def features(self) -> int:
        return len(self.kinds)

    def describe(self, rows: int) -> str:
        size = f"{rows:,} rows" + ("" if rows == self.rows else " (reduced)")
        return (f"configs[{self.index}]: {self.objective} {size} x {self.features}, {self.max_bin} bins, "
                f"{self.num_leaves} leaves")


CONFIGS = {
    "c1": Config("c1", 0, 1_000_000, "regression", 255, 63, 100, ["gauss"] * 28),
    "c2": Config("c2", 1, 10_000_000, "binary", 255, 255, 500, ["gauss"] * 70 + ["unif"] * 30, 1207.0),
    "c3": Config("c3", 2, 2_000_000, "lambdarank", 255, 127, 300,
                 ["gauss"] * 60 + ["lognormal"] * 40 + ["zeros30"] * 36),
    "c4": Config("c4", 3, 100_000_000, "regression", 255, 255, 200, ["gauss"] * 256, 1797.0),
    # 80% of the features zero-dominant (every fifth feature is N(0,1), the rest 95% zeros)
    "c5": Config("c5", 4, 5_000_000, "binary", 63, 31, 200,
                 ["gauss" if f % 5 == 0 else "sparse95" for f in range(2000)]),
}
CFG = CONFIGS["c4"]
ROWS = CFG.rows


def set_config(name: str):
    global CFG, ROWS
    CFG = CONFIGS[name]
    ROWS = CFG.rows


def set_rows(rows: int):
    global ROWS
    ROWS = rows


def params_dict(num_iterations: int) -> dict:
    return dict(objective=CFG.objective, num_leaves=CFG.num_leaves, learning_rate=0.1, num_grad_quant_bins=4,
                num_iterations=num_iterations)


# ---- synthetic data (torch on the GPU as plumbing) ------------------------------------------------------------

def _mul32(x, c: int):
    """x * c mod 2^32 for x < 2^32 held in int64, without overflowing int64."""
    lo, hi = x & 0xFFFF, x >> 16
    return (lo * c + (((hi * c) & 0xFFFF) << 16)) & 0xFFFFFFFF


def _mix32(x):
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    return x ^ (x >> 16)


def _unit(stream: int, rows):
    """24-bit uniform in [0, 1) from (SEED, stream, row): silvic's counter hash (quantize.rs:16-31)."""
    import torch

    h = _mix32(_mix32(rows) ^ _mix32(torch.full_like(rows, (SEED ^ stream) & 0xFFFFFFFF)))
    return (h >> 8).to(torch.float64) / 16777216.0


def _gauss(stream: int, rows):
    """N(0, 1) by Box-Muller from two counter-hash uniforms (streams `stream`, `stream` + 1)."""
    import torch

    u1 = 1.0 - _unit(stream, rows)
    u2 = _unit(stream + 1, rows)
    return torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * torch.pi * u2)


def column(f: int, rows):
    """Feature f of `rows` (f64): kind "gauss" ~ N(0,1) (streams 2f, 2f+1), "unif" ~ U[0,1) (stream 1000 + f),
    "lognormal" = exp(N(0,1)), "zeros30" / "sparse95" = N(0,1) with 30% / 95% of the rows exactly 0 (stream
    3000 + f)."""
    kind = CFG.kinds[f]
    if kind == "gauss":
        return _gauss(2 * f, rows)
    if kind == "unif":
        return _unit(1000 + f, rows)
    if kind == "lognormal":
        import torch

        return torch.exp(_gauss(2 * f, rows))
    if kind == "zeros30":
        return _gauss(2 * f, rows) * (_unit(3000 + f, rows) >= 0.3)
    if kind == "sparse95":
        return _gauss(2 * f, rows) * (_unit(3000 + f, rows) >= 0.95)
    raise ValueError(kind)


_QUERIES: dict = {}


def query_boundaries() -> np.ndarray:
    """c3's queries over rows 0..ROWS: sizes ~ Poisson(120) clipped to [1, 1000] from a seeded generator, in order,
    the last one cut at the last row (num_queries + 1 boundaries)."""
    if ROWS not in _QUERIES:
        g = np.random.default_rng(SEED + 3)
        sizes = np.clip(g.poisson(120.0, size=ROWS // 100 + 16), 1, 1000)
        while sizes.sum() < ROWS:
            sizes = np.concatenate([sizes, np.clip(g.poisson(120.0, size=1024), 1, 1000)])
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        last = int(np.searchsorted(bounds, ROWS))
        bounds = bounds[: last + 1]
        bounds[-1] = ROWS
        _QUERIES[ROWS] = bounds.astype(np.int64)
    return _QUERIES[ROWS]


def shard_rows(rank: int, world: int) -> tuple[int, int]:
    """Rank's contiguous rows; with queries, cut at the query boundary nearest to an even split (a query stays on
    one rank)."""
    cut = lambda r: ROWS * r // world  # noqa: E731
    if CFG.objective != "lambdarank":
        return cut(rank), cut(rank + 1)
    qb = query_boundaries()
    snap = lambda r: 0 if r == 0 else ROWS if r == world else int(qb[np.abs(qb - cut(r)).argmin()])  # noqa: E731
    return snap(rank), snap(rank + 1)


def features_of(rows, device):
    """[len(rows), features] f32."""
    import torch

    out = torch.empty((rows.numel(), CFG.features), dtype=torch.float32, device=device)
    for f in range(CFG.features):
        out[:, f] = column(f, rows).to(torch.float32)
    return out


def labels_of(rows):
    """The config's label, computing only the features it depends on.
    c1: 8 random-weight features + 0.5 x0 x1 + N(0, 0.1); c2: Bernoulli(sigmoid(sparse linear in 12 features + 3
    pairwise interactions)); c3: relevance 0..4 (_relevance); c4: a linear function of 32 random features + N(0, 1);
    c5: Bernoulli(sigmoid(linear in 50 random features))."""
    import torch

    x = lambda f: column(int(f), rows).to(torch.float32).double()  # noqa: E731  (the f32 feature, as binned)
    if CFG.name == "c3":
        return _relevance(rows, x)
    if CFG.name == "c5":
        g = np.random.default_rng(SEED + 5)
        picked = g.choice(CFG.features, size=50, replace=False)
        weights = g.normal(0.0, 1.0, size=50)
        logit = torch.zeros(rows.numel(), dtype=torch.float64, device=rows.device)
        for f, w in zip(picked, weights):
            logit += float(w) * x(f)
        return (_unit(5000, rows) < torch.sigmoid(logit)).to(torch.float32)
    if CFG.name == "c1":
        g = np.random.default_rng(SEED + 1)
        picked = g.choice(CFG.features, size=8, replace=False)
        weights = g.normal(0.0, 1.0, size=8)
        y = torch.zeros(rows.numel(), dtype=torch.float64, device=rows.device)
        for f, w in zip(picked, weights):
            y += float(w) * x(f)
        y += 0.5 * x(0) * x(1) + 0.1 * _gauss(6000, rows)
        return y.to(torch.float32)
    g = np.random.default_rng(SEED)
    if CFG.name == "c4":
        picked = g.choice(CFG.features, size=32, replace=False)
        weights = g.normal(0.0, 1.0, size=32)
        y = torch.zeros(rows.numel(), dtype=torch.float64, device=rows.device)
        for f, w in zip(picked, weights):
            y += float(w) * x(f)
        y += _gauss(6000, rows)
        return y.to(torch.float32)
    picked = g.choice(CFG.features, size=12, replace=False)
    weights = g.normal(0.0, 1.0, size=12)
    pairs = g.choice(CFG.features, size=(3, 2), replace=False)
    logit = torch.zeros(rows.numel(), dtype=torch.float64, device=rows.device)
    for f, w in zip(picked, weights):
        logit += float(w) * x(f)
    for a, b in pairs:
        logit += 0.8 * x(a) * x(b)
    p = torch.sigmoid(logit)
    return (_unit(5000, rows) < p).to(torch.float32)


_RELEVANCE_CUTS: dict = {}


def _relevance(rows, x):
    """c3's integer relevance 0..4: a noisy linear score in 20 random features, cut at its 50/75/90/97th percentiles
    over the first SAMPLE_ROWS rows (the same cuts on every rank)."""
    import torch

    g = np.random.default_rng(SEED + 2)
    picked = g.choice(CFG.features, size=20, replace=False)
    weights = g.normal(0.0, 1.0, size=20)

    def score(r, xf):
        y = torch.zeros(r.numel(), dtype=torch.float64, device=r.device)
        for f, w in zip(picked, weights):
            y += float(w) * torch.tanh(xf(f))
        return y + 0.5 * _gauss(7000, r)

    key = (ROWS, SAMPLE_ROWS)
    if key not in _RELEVANCE_CUTS:
        sample = torch.arange(min(SAMPLE_ROWS, ROWS), dtype=torch.int64, device=rows.device)
        s = score(sample, lambda f: column(int(f), sample).to(torch.float32).double())
        _RELEVANCE_CUTS[key] = torch.quantile(s.float(), torch.tensor([0.5, 0.75, 0.9, 0.97], device=s.device)).double()
    cuts = _RELEVANCE_CUTS[key].to(rows.device)
    return torch.bucketize(score(rows, x), cuts, right=True).to(torch.float32)


def bin_mappers(device):
    """Per feature: equal-frequency upper bounds (ascending, duplicates dropped, the last +inf) from the first
    SAMPLE_ROWS rows, and the sample's min and max."""
    import torch

    n = min(SAMPLE_ROWS, max(ROWS, 1))
    rows = torch.arange(n, dtype=torch.int64, device=device)
    k = torch.arange(1, CFG.max_bin, device=device)
    cut = (k * n) // CFG.max_bin
    out = []
    for f in range(CFG.features):
        srt, _ = torch.sort(column(f, rows).to(torch.float32).double())
        bounds = ((srt[cut - 1] + srt[cut]) / 2.0).cpu().numpy()
        bounds = np.unique(bounds[np.isfinite(bounds)])
        out.append((np.append(bounds, np.inf), float(srt[0]), float(srt[-1])))
    return out


def feature_metas(mappers):
    """The config's numerical mappers ((upper bounds, min, max) per feature) as FeatureMeta, named as LightGBM names
    unnamed columns."""
    from silvic_b200.dataset import FeatureMeta

    return [FeatureMeta(name=f"Column_{f}", num_bins=len(ub), upper_bounds=ub, min_value=lo, max_value=hi)
            for f, (ub, lo, hi) in enumerate(mappers)]


def dataset_layout(mappers):
    """silvic's group layout of the config's features (silvic_b200.dataset.layout, data/build.rs:336-382)."""
    from silvic_b200.dataset import layout

    return layout(feature_metas(mappers))


def build_dataset(begin: int, end: int, device, chunk: int = 2_000_000):
    """Rows begin..end in silvic's group layout, in page-locked host memory (the load's host-to-device copies run at
    DMA speed and count in the e2e time). On a GPU the rows are binned by the product (sb2_bin_dense); without one
    (the CPU tests of the bench's sharding) by torch.bucketize, which counts the same bounds."""
    import torch

    from silvic_b200.dataset import BinnedDataset, FeatureGroup

    mappers = bin_mappers(device)
    features, shells, total_bins = dataset_layout(mappers)
    n = end - begin
    pin = torch.cuda.is_available()
    pinned = [torch.empty((n, g.row_stride), dtype=torch.uint8, pin_memory=pin) for g in shells]
    pinned.append(torch.empty(n, dtype=torch.float32, pin_memory=pin))
    host = [t.numpy() for t in pinned[:-1]]
    label = pinned[-1].numpy()
    binner = None
    if device.type == "cuda":
        from silvic_b200 import B200Backend

        binner = B200Backend(device.index or 0)
    def chunks():
        # the chunk's raw features made on the device, its labels into the label array on the way
        for lo in range(0, n, chunk):
            hi = min(n, lo + chunk)
            rows = torch.arange(begin + lo, begin + hi, dtype=torch.int64, device=device)
            label[lo:hi] = labels_of(rows).cpu().numpy()
            yield lo, features_of(rows, device)

    try:
        if binner is not None:
            # streaming construction through the product: each chunk binned on the device into the pinned rows
            data = BinnedDataset.from_chunks(chunks(), n, feature_metas(mappers), label, binner, row_offset=begin,
                                             out=host)
        else:
            for lo, x in chunks():
                for gi, g in enumerate(shells):
                    blk = torch.zeros((x.shape[0], g.row_stride), dtype=torch.uint8)
                    for col, f in enumerate(g.features):
                        ub = torch.from_numpy(features[f].upper_bounds).to(torch.float64)
                        blk[:, col] = torch.bucketize(x[:, f].double(), ub, right=False).to(torch.uint8)
                    host[gi][lo:lo + x.shape[0]] = blk.numpy()
            groups = [FeatureGroup(g.features, g.row_stride, g.hist_offset, g.total_bins, host[gi])
                      for gi, g in enumerate(shells)]
            data = BinnedDataset(n, begin, features, groups, total_bins, label)
    finally:
        if binner is not None:
            binner.close()
    if CFG.objective == "lambdarank":
        qb = query_boundaries()
        lo, hi = np.searchsorted(qb, [begin, end])
        assert qb[lo] == begin and qb[hi] == end, "a shard must hold whole queries"
        data.query_boundaries = (qb[lo:hi + 1] - begin).astype(np.uint32)
    data._keep.extend(pinned)
    return data


def all_labels(device):
    """Every rank's labels (rows 0..ROWS in row order) for the initial score."""
    import torch

    out = np.empty(ROWS, dtype=np.float32)
    for lo in range(0, ROWS, 4_000_000):
        hi = min(ROWS, lo + 4_000_000)
        out[lo:hi] = labels_of(torch.arange(lo, hi, dtype=torch.int64, device=device)).cpu().numpy()
    return out


# ---- clocks --------------------------------------------------------------------------------------------------

class Clocks:
    """nvidia-smi samples of one GPU's clocks and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.lines, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- arms ----------------------------------------------------------------------------------------------------

def measured_peak_hbm() -> tuple[float, str]:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def tree_algorithmic_bytes(tree, n_rows: int, row_bytes: int, total_bins: int, max_leaves: int, world: int = 1) -> int:
    """Bytes one GPU's tree kernel must move at the least to grow `tree` (`n_rows` rows of `row_bytes` bin bytes on
    this GPU; with `world` ranks the tree's node counts are global, and each rank holds 1/world of every leaf).

    The root histogram reads every row's bins and packed gradient (its rows are in row order: no row ids) and writes
    a histogram of `total_bins` [g, h] int32 pairs. Split k of a parent of P rows reads each row's id (not for the
    root's rows), packed gradient and byte of the split feature, and writes id and gradient to the other partition
    buffer (n·(4+1+4) read, 8 written); while more splits may follow (k + 2 < max_leaves) it also histograms the
    smaller child's B rows: their ids, gradients and bins, and the histogram out. Split k is internal node k (nodes
    are numbered in split order).
    """
    def count(c: int) -> int:
        return (int(tree.internal_count[c]) if c >= 0 else int(tree.leaf_count[~c])) // world

    total = n_rows * (row_bytes + 4) + 8 * total_bins
    for k in range(len(tree.internal_count)):
        parent = int(tree.internal_count[k]) // world
        total += parent * ((0 if k == 0 else 4) + 4 + 1) + parent * 8
        if k + 2 < max_leaves:
            built = min(count(int(tree.left_child[k])), count(int(tree.right_child[k])))
            total += built * (row_bytes + 8) + 8 * total_bins
    return total


def oracle_params(num_iterations: int):
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as orc
    from silvic_b200 import _abi

    objective = {"regression": _abi.REGRESSION, "binary": _abi.BINARY, "lambdarank": _abi.LAMBDARANK}[CFG.objective]
    return orc.default_params(objective=objective, num_leaves=CFG.num_leaves, learning_rate=0.1,
                              num_grad_quant_bins=4, num_iterations=num_iterations)


def oracle_train(data, iterations: int):
    """The CPU oracle's trainer on `data` (test infrastructure: the bench's CPU legs only)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as orc

    m = orc.train([data], oracle_params(iterations))
    return m, orc.lib().orc_num_threads()


def parity_of(model, ref, data) -> dict:
    """The device model's first trees against the oracle's trees of the same dataset: every tree field bit for bit,
    the initial score, and the LightGBM model text of those trees byte for byte."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as orc
    from silvic_b200.backend import Model

    k = len(ref.trees)
    mine = model.trees[:k]
    differs = [f"tree {i}: {','.join(d)}" for i, (t, r) in enumerate(zip(mine, ref.trees))
               if (d := orc.trees_equal(t, r))]
    p = oracle_params(k)
    text_dev = Model(mine, model.init_score, []).to_lightgbm_string(data, p)
    text_ref = Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)
    return {"trees": k, "trees_identical": len(mine) == k and not differs,
            "init_score_identical": model.init_score == ref.init_score,
            "model_text_identical": text_dev == text_ref, "differences": differs[:5],
            "against": "CPU oracle (oracle/oracle.cpp) on the whole dataset"}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import torch

    data = build_dataset(0, ROWS, torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu"))
    # Warm-up iteration, then as many timed iterations (up to --steps) as fit a ~60 s CPU budget.
    warm, _ = oracle_train(data, 1)
    per_iter = max(warm.iteration_seconds)
    k = int(max(1, min(args.steps, 60.0 // max(per_iter, 1e-3))))
    m, cores = oracle_train(data, k)
    secs = m.iteration_seconds
    rate = len(secs) / sum(secs)
    sample = f"{len(secs)} boosting iterations of the full {ROWS:,} x {CFG.features} set on {cores} threads"
    by_op = {k_: v / len(secs) for k_, v in m.op_seconds.items()}
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": "iters/s", "n_gpus": world,
            "steps": args.steps, "timed_steps": len(secs), "warmup": args.warmup,
            "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int32 histograms / f64 split search", "data": "synthetic",
            "config": {"workload": CFG.describe(ROWS), "rows": ROWS, "features": CFG.features,
                       "num_leaves": CFG.num_leaves},
            "cpu_baseline": {"value": rate, "unit": "iters/s", "cores": cores, "kind": "port", "sample": sample,
                             "seconds_by_op": by_op},
            "e2e": {"value": rate, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _max_over_ranks(values: list[float], world: int, dev) -> list[float]:
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


DOMINANT_SHARE: float | None = None  # --dominant-share: sb2_set_dominant_share before every load (None: default)


def _joined_backend(local: int, data, params, rank: int, world: int) -> tuple[object, float, float]:
    """A fresh handle with `data` loaded and, with ranks, joined: (backend, load seconds, join seconds)."""
    import torch.distributed as dist

    from silvic_b200 import B200Backend

    t0 = time.perf_counter()
    b = B200Backend(local)
    if DOMINANT_SHARE is not None:
        b.set_dominant_share(DOMINANT_SHARE)
    b.load(data, params.objective, params.sigmoid, params)
    t1 = time.perf_counter()
    if world > 1:
        uid = [B200Backend.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        b.join_ranks(uid[0], world, rank)
    return b, t1 - t0, time.perf_counter() - t1


def run_b200(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from silvic_b200 import init_score, params_from_dict

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    begin, end = shard_rows(rank, world)
    data = build_dataset(begin, end, dev)
    labels = all_labels(dev) if world > 1 else data.label
    torch.cuda.synchronize()
    params = params_from_dict(params_dict(args.warmup + args.steps))
    score0 = init_score(params, labels)

    # Device-timed run: per-iteration CUDA events; the last `steps` iterations are the timed region.
    backend, _, _ = _joined_backend(local, data, params, rank, world)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        model = backend.train(params, score0)
    torch.cuda.synchronize()
    secs = model.iteration_seconds
    timed = float(sum(secs[args.warmup:args.warmup + args.steps]))
    # The tree kernel's own launches in the timed region (one cooperative launch per tree, CUDA events on the
    # backend's stream around each).
    tree_s = model.tree_seconds[args.warmup:args.warmup + args.steps]
    timed_trees = model.trees[args.warmup:args.warmup + args.steps]
    # The standalone root histogram (every row, every feature).
    hist_s = backend.time_histogram(10)
    # What bounds it: red.shared.add.u32 alone at the histogram's address pattern (lane adds per second).
    adds_alone = backend.time_shared_adds(0)[0]
    backend.close()
    launches_persistent = bool(model.tree_seconds)
    timed, hist_s = _max_over_ranks([timed, hist_s], world, dev)

    # End to end through the C ABI with host buffers: a whole job of the config's trees, setup included.
    e2e_params = params_from_dict(params_dict(args.trees or CFG.trees))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    b2, load_s, join_s = _joined_backend(local, data, e2e_params, rank, world)
    t1 = time.perf_counter()
    m2 = b2.train(e2e_params, score0)
    e2e_s = time.perf_counter() - t0
    train_s = time.perf_counter() - t1
    b2.close()
    e2e_s, load_s, join_s, train_s = _max_over_ranks([e2e_s, load_s, join_s, train_s], world, dev)
    e2e_trees = len(m2.trees)
    h2d = sum(g.data.nbytes for g in data.groups) + data.label.nbytes
    d2h = sum(sum(getattr(t_, f).nbytes for f in t_.FIELDS) for t_ in m2.trees)
    del m2
    # Every collective is done: the other ranks leave while rank 0 checks parity on the CPU.
    if rank != 0:
        return
    n_local = end - begin
    S = sum(g.row_stride for g in data.groups)
    T = data.total_bins
    bytes_root = n_local * (S + 4) + 8 * T  # algorithmic bytes of one root histogram launch (rows in row order)
    peak, peak_kind = measured_peak_hbm()
    hist_roofline = {"kernel": "histogram_kernel + slab reduction (root: every row, every feature)",
                     "achieved": bytes_root / hist_s / 1e9, "launch_ms": hist_s * 1000.0,
                     "algorithmic_bytes": bytes_root}
    hist_roofline["frac"] = hist_roofline["achieved"] / peak
    # One shared atomic per (row, feature): the histogram's atomic rate against the atomic unit's rate alone.
    hist_roofline["shared_adds"] = {"histogram_per_s": n_local * CFG.features / hist_s, "alone_per_s": adds_alone,
                                    "frac": n_local * CFG.features / hist_s / adds_alone}
    if tree_s and len(tree_s) == len(timed_trees):
        # The dominant kernel: the persistent tree kernel, one launch per tree.
        tree_bytes = [tree_algorithmic_bytes(tr, n_local, S, T, CFG.num_leaves, world) for tr in timed_trees]
        launch_s = sum(tree_s) / len(tree_s)
        per_launch = sum(tree_bytes) / len(tree_bytes)
        roofline = {"bound": "hbm", "achieved": per_launch / launch_s / 1e9, "peak": peak, "unit": "GB/s",
                    "peak_kind": peak_kind,
                    "traffic": None if CFG.traffic_per_row is None else CFG.traffic_per_row * n_local,
                    "kernel": "grow_tree_kernel (one cooperative launch grows one tree)",
                    "launch_ms": launch_s * 1000.0, "algorithmic_bytes": per_launch,
                    "share_of_step": sum(tree_s) / timed if world == 1 else None, "root_histogram": hist_roofline}
    else:
        roofline = {"bound": "hbm", "achieved": hist_roofline["achieved"], "peak": peak, "unit": "GB/s",
                    "peak_kind": peak_kind, "traffic": None, "kernel": hist_roofline["kernel"],
                    "launch_ms": hist_roofline["launch_ms"], "algorithmic_bytes": bytes_root}
    roofline["frac"] = roofline["achieved"] / peak
    line = {
        "metric": METRIC,
        "value": args.steps / timed,
        "unit": "iters/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * timed / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int32 histograms / f64 split search",
        "data": "synthetic (counter-hash features; equal-frequency bins of the first 200,000 rows)",
        "config": {"workload": CFG.describe(ROWS), "rows": ROWS, "features": CFG.features,
                   "num_leaves": CFG.num_leaves, "parallelism": f"rows sharded over {world} GPU(s)",
                   "l2": f"inputs ({n_local * S / 1e9:.1f} GB binned per GPU) larger than L2; no flush",
                   **({"dominant_share": DOMINANT_SHARE} if DOMINANT_SHARE is not None else {})},
        "trees": len(model.trees),
        "hist_rows_feats_per_s": n_local * CFG.features / hist_s * world,
        "roofline": roofline,
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_trees / e2e_s, "unit": "iters/s", "trees": e2e_trees, "seconds": e2e_s,
                "h2d_bytes_per_step": h2d // e2e_trees, "d2h_bytes_per_step": d2h // e2e_trees,
                "setup_seconds": {"load": load_s, "join_ranks": join_s}, "train_seconds": train_s},
        # Our kernels per iteration: gradients, iteration start (quantize), the tree (one persistent launch, or
        # histogram + reduction + search for the root and partition flags + scatter + histogram + reduction + search
        # per split with NCCL ranks), leaf map + leaf sums, finalize, score update.
        "gpu_launches": args.steps * (7 if launches_persistent else 3 + 3 + 5 * (CFG.num_leaves - 1) + 4),
    }
    if not args.no_parity:
        # The oracle trains the first trees of the same job on the whole dataset (on one rank: the same data; with
        # ranks, rank 0 builds every rank's rows). Its time is also the CPU baseline at N = 1.
        full = data if world == 1 else build_dataset(0, ROWS, dev)
        ref, cores = oracle_train(full, PARITY_TREES)
        line["parity"] = parity_of(model, ref, full)
        if world == 1:
            secs_ref = ref.iteration_seconds
            line["cpu_baseline"] = {"value": len(secs_ref) / sum(secs_ref), "unit": "iters/s", "cores": cores,
                                    "kind": "port",
                                    "sample": f"{len(secs_ref)} boosting iterations of the same {ROWS:,} x "
                                              f"{CFG.features} dataset, {sum(secs_ref):.1f} s on {cores} threads",
                                    # the reference's `Timed` split (tests/train_cpu.rs:434-484), seconds per iteration
                                    "seconds_by_op": {k: v / len(secs_ref) for k, v in ref.op_seconds.items()}}
    print(json.dumps(line), flush=True)


def run_binning(args):
    """The device binning of a dense matrix (`sb2_bin_dense`, data/binning.rs bin_rows) on the config's raw
    features: a device-resident f32 matrix into the dataset's groups, timed from the call until the group rows are
    in host memory (wall clock: the copy of the rows back is part of the job). One line of JSON."""
    import torch

    from silvic_b200.backend import B200Backend

    dev = torch.device("cuda", 0)
    rows = min(ROWS, 10_000_000)
    features, groups, _ = dataset_layout(bin_mappers(dev))
    x = features_of(torch.arange(rows, dtype=torch.int64, device=dev), dev)
    b = B200Backend(0)
    times = []
    for it in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        b.bin_dense(x, features, groups)
        if it >= args.warmup:
            times.append(time.perf_counter() - t0)
    b.close()
    s = sum(times) / len(times)
    print(json.dumps({"binning": {"rows": rows, "features": CFG.features, "ms": s * 1e3,
                                  "values_per_s": rows * CFG.features / s, "input": "device f32 row-major",
                                  "output": "host group rows", "steps": args.steps, "warmup": args.warmup}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle's trees (parity and, at N = 1, the CPU baseline)")
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS),
                    help="c4 (default): BASELINE configs[3], 100M rows; c1, c2, c3, c5: configs[0], [1], [2], [4]")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows of the synthetic set (a smaller case for profiling; default: the config's)")
    ap.add_argument("--trees", type=int, default=0,
                    help="trees of the end-to-end job (default: the config's full count)")
    ap.add_argument("--binning", action="store_true",
                    help="time the device binning of the config's raw features instead of training (one GPU)")
    ap.add_argument("--dominant-share", type=float, default=None,
                    help="sb2_set_dominant_share before each load: tiles whose features hold this share of the rows "
                         "in their most frequent bins skip them in the tree kernel's histogram (default: off)")
    args = ap.parse_args()
    set_config(args.config)
    if args.dominant_share is not None:
        global DOMINANT_SHARE
        DOMINANT_SHARE = args.dominant_share
    if args.rows:
        set_rows(args.rows)
    if args.binning:
        run_binning(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_b200(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
