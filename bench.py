"""Benchmark: boosting iterations/s of silvic's quantized-histogram training on B200, BASELINE config 2.

Workload: binary classification, 10,000,000 rows x 100 f32 features (70 N(0,1),
30 U[0,1)), label ~ Bernoulli(sigmoid(sparse random linear + 3 pairwise interactions)), 255 bins, 255 leaves,
quantized gradients (4 bins). A "step" is one boosting iteration: gradients, quantization, a 255-leaf tree grown
split by split on the device (partition, smaller-child histogram, sibling subtraction, split scan), leaf renewal
and the score update.

Data are synthetic: every feature value is a pure function of (seed, global row, feature) from silvic's counter
hash, generated on the GPU, so any rank regenerates its own rows. Bin bounds are equal-frequency cuts of the first
200,000 rows (bin_construct_sample_cnt's default sample size), bins the rows with them, and pack the features into
silvic's group layout (32 features of 255 bins per group). The binned matrix (1 GB) is larger than the 126 MB L2,
so no L2 flush is needed between timed iterations.

Arms:
  default            the B200 backend; `value` = iterations/s from CUDA events around each iteration of the
                     device-resident trainer (inputs resident in HBM), max over ranks; `e2e` = the same metric
                     through the reference-facing C ABI with host buffers: sb2_load (host->device copy of the binned
                     data) + sb2_train + the trees read back, wall clock.
  --impl reference   the CPU restatement of silvic-core's trainer (oracle/, "port") on this box's host cores.

Multi-GPU: one process per GPU (torchrun). Rows are sharded contiguously (strong scaling: the 10M-row job is fixed)
and every split's histogram is allreduced over NCCL inside the backend.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 20261107
CONFIG = "c2"
ROWS = 10_000_000
GAUSSIAN, UNIFORM = 70, 30
FEATURES = GAUSSIAN + UNIFORM
MAX_BIN = 255
SAMPLE_ROWS = 200_000
PARAMS = dict(objective="binary", num_leaves=255, learning_rate=0.1, num_grad_quant_bins=4)


def set_config(name: str):
    """c2 (the default) or c4 (configs[3], the multi-GPU scaling config: 100,000,000 rows
    x 256 N(0,1) features, target = a random 32-feature linear function + N(0,1) noise, L2 regression, 255 bins,
    255 leaves)."""
    global CONFIG, ROWS, GAUSSIAN, UNIFORM, FEATURES, PARAMS
    CONFIG = name
    if name == "c4":
        ROWS, GAUSSIAN, UNIFORM = 100_000_000, 256, 0
        PARAMS = dict(objective="regression", num_leaves=255, learning_rate=0.1, num_grad_quant_bins=4)
    else:
        ROWS, GAUSSIAN, UNIFORM = 10_000_000, 70, 30
        PARAMS = dict(objective="binary", num_leaves=255, learning_rate=0.1, num_grad_quant_bins=4)
    FEATURES = GAUSSIAN + UNIFORM
METRIC = "boosting iters/sec + histogram rows·feats/sec (HBM % peak) at 1/2/4/8 B200"
# DRAM bytes (read + write) the tree kernel moved per training row in one launch, from an ncu capture of a smaller
# case of the same workload (2M rows; the traffic grows with the rows): profiles/grow_tree_kernel_2m.md. Per config;
# none captured for c4.
TREE_TRAFFIC_PER_ROW = {"c2": 885, "c4": None}


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


def features_of(rows, device):
    """[len(rows), 100] f32: features 0..69 ~ N(0,1) (Box-Muller), 70..99 ~ U[0,1)."""
    import torch

    out = torch.empty((rows.numel(), FEATURES), dtype=torch.float32, device=device)
    for f in range(GAUSSIAN):
        u1 = 1.0 - _unit(2 * f, rows)
        u2 = _unit(2 * f + 1, rows)
        out[:, f] = (torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * torch.pi * u2)).to(torch.float32)
    for f in range(GAUSSIAN, FEATURES):
        out[:, f] = _unit(1000 + f, rows).to(torch.float32)
    return out


def labels_of(rows, x):
    """c2: Bernoulli(sigmoid(sparse linear in 12 features + 3 pairwise interactions)); c4: a linear function of 32
    random features + N(0,1) noise."""
    import torch

    g = np.random.default_rng(SEED)
    if CONFIG == "c4":
        picked = g.choice(FEATURES, size=32, replace=False)
        weights = g.normal(0.0, 1.0, size=32)
        y = torch.zeros(rows.numel(), dtype=torch.float64, device=x.device)
        for f, w in zip(picked, weights):
            y += float(w) * x[:, int(f)].double()
        u1, u2 = 1.0 - _unit(6000, rows), _unit(6001, rows)
        y += torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * torch.pi * u2)
        return y.to(torch.float32)
    picked = g.choice(FEATURES, size=12, replace=False)
    weights = g.normal(0.0, 1.0, size=12)
    pairs = g.choice(FEATURES, size=(3, 2), replace=False)
    logit = torch.zeros(rows.numel(), dtype=torch.float64, device=x.device)
    for f, w in zip(picked, weights):
        logit += float(w) * x[:, int(f)].double()
    for a, b in pairs:
        logit += 0.8 * x[:, int(a)].double() * x[:, int(b)].double()
    p = torch.sigmoid(logit)
    return (_unit(5000, rows) < p).to(torch.float32)


def bin_bounds(device):
    """Equal-frequency upper bounds per feature from the first SAMPLE_ROWS rows (ascending, last +inf)."""
    import torch

    rows = torch.arange(SAMPLE_ROWS, dtype=torch.int64, device=device)
    x = features_of(rows, device).double()
    srt, _ = torch.sort(x, dim=0)
    k = torch.arange(1, MAX_BIN, device=device)
    cut = (k * SAMPLE_ROWS) // MAX_BIN
    bounds = (srt[cut - 1] + srt[cut]) / 2.0
    bounds = torch.cat([bounds, torch.full((1, FEATURES), float("inf"), device=device, dtype=torch.float64)])
    return bounds.T.contiguous()  # [FEATURES, MAX_BIN]


def build_dataset(begin: int, end: int, device, chunk: int = 2_000_000):
    """Rows begin..end binned into silvic's group layout on the GPU, returned as host arrays."""
    import torch

    from silvic_b200.dataset import BinnedDataset, FeatureGroup, FeatureMeta

    bounds = bin_bounds(device)
    n = end - begin
    per_group = 8192 // MAX_BIN  # 32 features of 255 bins per group (data/build.rs:336-382)
    group_feats = [list(range(s, min(s + per_group, FEATURES))) for s in range(0, FEATURES, per_group)]
    strides = [(len(g) + 3) // 4 * 4 for g in group_feats]
    # Page-locked host arrays: the load's host-to-device copies run at DMA speed (and count in the e2e time).
    pin = torch.cuda.is_available()
    pinned = [torch.empty((n, s), dtype=torch.uint8, pin_memory=pin) for s in strides]
    pinned.append(torch.empty(n, dtype=torch.float32, pin_memory=pin))
    host = [t.numpy() for t in pinned[:-1]]
    label = pinned[-1].numpy()
    b32 = bounds.to(torch.float32)
    for lo in range(0, n, chunk):
        hi = min(n, lo + chunk)
        rows = torch.arange(begin + lo, begin + hi, dtype=torch.int64, device=device)
        x = features_of(rows, device)
        label[lo:hi] = labels_of(rows, x).cpu().numpy()
        xt = x.T.contiguous()
        binned = torch.empty((FEATURES, hi - lo), dtype=torch.uint8, device=device)
        for f in range(FEATURES):
            # the first bin whose upper bound is >= value (BinMapper::value_to_bin, data/bin_mapper.rs:344-360)
            binned[f] = torch.bucketize(xt[f], b32[f], right=False).to(torch.uint8)
        for gi, feats in enumerate(group_feats):
            blk = torch.zeros((hi - lo, strides[gi]), dtype=torch.uint8, device=device)
            blk[:, : len(feats)] = binned[feats].T
            host[gi][lo:hi] = blk.cpu().numpy()
    features, groups, offset = [], [], 0
    ub = bounds.cpu().numpy()
    for gi, feats in enumerate(group_feats):
        hist_offset = offset
        for col, f in enumerate(feats):
            features.append(FeatureMeta(name=f"Column_{f}", num_bins=MAX_BIN, upper_bounds=ub[f].copy(),
                                        min_value=float(ub[f][0]), max_value=float(ub[f][-2]), group=gi,
                                        column=col, hist_offset=offset))
            offset += MAX_BIN
        groups.append(FeatureGroup(feats, strides[gi], hist_offset, len(feats) * MAX_BIN, host[gi]))
    data = BinnedDataset(n, begin, features, groups, offset, label)
    data._keep.extend(pinned)
    return data


def all_labels(device):
    """Every rank's labels (rows 0..ROWS in row order) for the initial score."""
    import torch

    out = np.empty(ROWS, dtype=np.float32)
    for lo in range(0, ROWS, 2_000_000):
        hi = min(ROWS, lo + 2_000_000)
        rows = torch.arange(lo, hi, dtype=torch.int64, device=device)
        out[lo:hi] = labels_of(rows, features_of(rows, device)).cpu().numpy()
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
    buffer; while more splits may follow (k + 2 < max_leaves) it also histograms the smaller child's B rows: their ids,
    gradients and bins, and the histogram out. Split k is internal node k (nodes are numbered in split order).
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


def oracle_rate(data, iterations: int, params) -> tuple[float, list[float], int]:
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as orc

    p = orc.default_params(**params)
    p.num_iterations = iterations
    m = orc.train([data], p)
    secs = m.iteration_seconds
    return len(secs) / sum(secs), secs, orc.lib().orc_num_threads()


def oracle_params():
    from silvic_b200 import _abi

    objective = _abi.REGRESSION if PARAMS["objective"] == "regression" else _abi.BINARY
    return dict(objective=objective, num_leaves=255, learning_rate=0.1, num_grad_quant_bins=4)


def set_rows(rows: int):
    global ROWS
    ROWS = rows


def workload() -> str:
    if CONFIG == "c4":
        size = "100M" if ROWS == 100_000_000 else f"{ROWS:,} rows (reduced)"
        return f"configs[3]: L2 regression {size} x 256, 255 bins, 255 leaves"
    size = "10M" if ROWS == 10_000_000 else f"{ROWS:,} rows (reduced)"
    return f"configs[1]: binary {size} x 100, 255 bins, 255 leaves"


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import torch

    data = build_dataset(0, ROWS, torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu"))
    # Warm-up iteration, then as many timed iterations (up to --steps) as fit a ~60 s CPU budget.
    warm_rate, warm_secs, cores = oracle_rate(data, max(1, min(args.warmup, 1)), oracle_params())
    per_iter = max(warm_secs)
    k = int(max(1, min(args.steps, 60.0 // max(per_iter, 1e-3))))
    rate, secs, cores = oracle_rate(data, k, oracle_params())
    sample = f"{len(secs)} boosting iterations of the full {ROWS:,} x 100 set on {cores} threads"
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": "iters/s", "n_gpus": world,
            "steps": args.steps, "timed_steps": len(secs), "warmup": args.warmup,
            "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int32 histograms / f64 split search", "data": "synthetic",
            "config": {"workload": workload(), "rows": ROWS,
                       "features": FEATURES, "num_leaves": 255},
            "cpu_baseline": {"value": rate, "unit": "iters/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from silvic_b200 import B200Backend, init_score, params_from_dict

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    begin, end = ROWS * rank // world, ROWS * (rank + 1) // world
    data = build_dataset(begin, end, dev)
    labels = all_labels(dev) if world > 1 else data.label
    torch.cuda.synchronize()
    params = params_from_dict(dict(PARAMS, num_iterations=args.warmup + args.steps))
    score0 = init_score(params, labels)

    def make_backend():
        b = B200Backend(local)
        b.load(data, params.objective, params.sigmoid)
        if world > 1:
            uid = [B200Backend.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            b.join_ranks(uid[0], world, rank)
        return b

    # Device-timed run: per-iteration CUDA events; the last `steps` iterations are the timed region.
    backend = make_backend()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        model = backend.train(params, score0)
    torch.cuda.synchronize()
    secs = model.iteration_seconds
    timed = float(sum(secs[args.warmup:args.warmup + args.steps]))
    trees = len(model.trees)
    # The tree kernel's own launches in the timed region (one GPU: one cooperative launch per tree, CUDA events on
    # the backend's stream around each).
    tree_s = model.tree_seconds[args.warmup:args.warmup + args.steps]
    timed_trees = model.trees[args.warmup:args.warmup + args.steps]
    # The standalone root histogram (every row, every feature), the kernel the multi-GPU path runs per split.
    hist_s = backend.time_histogram(10)
    backend.close()
    launches_persistent = bool(model.tree_seconds)  # each tree in one cooperative launch (per GPU)
    t = torch.tensor([timed, hist_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    timed, hist_s = float(t[0]), float(t[1])

    # End to end through the C ABI with host buffers: load (host -> device) + train + trees back.
    e2e_params = params_from_dict(dict(PARAMS, num_iterations=args.steps))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    b2 = B200Backend(local)
    b2.load(data, e2e_params.objective, e2e_params.sigmoid)
    if world > 1:
        uid = [B200Backend.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        b2.join_ranks(uid[0], world, rank)
    m2 = b2.train(e2e_params, score0)
    e2e_s = time.perf_counter() - t0
    b2.close()
    e = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
    e2e_s = float(e[0])
    h2d = sum(g.data.nbytes for g in data.groups) + data.label.nbytes
    d2h = sum(sum(getattr(t_, f).nbytes for f in t_.FIELDS) for t_ in m2.trees)

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
    if tree_s and len(tree_s) == len(timed_trees):
        # The dominant kernel: the persistent tree kernel, one launch per tree.
        tree_bytes = [tree_algorithmic_bytes(tr, n_local, S, T, PARAMS["num_leaves"], world) for tr in timed_trees]
        launch_s = sum(tree_s) / len(tree_s)
        per_launch = sum(tree_bytes) / len(tree_bytes)
        roofline = {"bound": "hbm", "achieved": per_launch / launch_s / 1e9, "peak": peak, "unit": "GB/s",
                    "peak_kind": peak_kind,
                    "traffic": None if TREE_TRAFFIC_PER_ROW[CONFIG] is None else TREE_TRAFFIC_PER_ROW[CONFIG] * n_local,
                    "kernel": "grow_tree_kernel (one cooperative launch grows one tree)",
                    "launch_ms": launch_s * 1000.0, "algorithmic_bytes": per_launch,
                    "share_of_step": sum(tree_s) / timed, "root_histogram": hist_roofline}
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
        "data": "synthetic",
        "config": {"workload": workload(), "rows": ROWS,
                   "features": FEATURES, "num_leaves": 255, "parallelism": f"rows sharded over {world} GPU(s)",
                   "l2": f"inputs ({n_local * S / 1e9:.1f} GB binned per GPU) larger than L2; no flush"},
        "trees": trees,
        "hist_rows_feats_per_s": n_local * FEATURES / hist_s * world,
        "roofline": roofline,
        "clocks": clocks.summary(),
        "e2e": {"value": args.steps / e2e_s, "unit": "iters/s", "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        # Our kernels per iteration: gradients, iteration start (quantize), the tree (one persistent launch, or
        # histogram + reduction + search for the root and partition flags + scatter + histogram + reduction + search
        # per split with NCCL ranks), leaf map + leaf sums, finalize, score update.
        "gpu_launches": args.steps * (7 if launches_persistent else 3 + 3 + 5 * (PARAMS["num_leaves"] - 1) + 4),
    }
    if world == 1 and not args.no_cpu_baseline:
        rate, secs, cores = oracle_rate(data, 2, oracle_params())
        line["cpu_baseline"] = {"value": rate, "unit": "iters/s", "cores": cores, "kind": "port",
                                "sample": f"2 boosting iterations of the same {ROWS:,} x {FEATURES} dataset, "
                                          f"{sum(secs):.1f} s on {cores} threads"}
    print(json.dumps(line), flush=True)


def run_binning(args):
    """The device binning of a dense matrix (`sb2_bin_dense`, data/binning.rs bin_rows) on the config's raw
    features: a device-resident f32 matrix into the dataset's groups of 32 features, timed from the call until the
    group rows are in host memory (wall clock: the copy of the rows back is part of the job). One line of JSON."""
    import torch

    from silvic_b200.backend import B200Backend
    from silvic_b200.dataset import FeatureGroup, FeatureMeta

    dev = torch.device("cuda", 0)
    bounds = bin_bounds(dev).cpu().numpy()
    x = features_of(torch.arange(ROWS, dtype=torch.int64, device=dev), dev)
    per_group = 8192 // MAX_BIN
    feats, groups = [], []
    for gi, start in enumerate(range(0, FEATURES, per_group)):
        members = list(range(start, min(FEATURES, start + per_group)))
        groups.append(FeatureGroup(members, (len(members) + 3) // 4 * 4, 0, 0, np.zeros((0, 4), np.uint8)))
        for col, f in enumerate(members):
            feats.append(FeatureMeta(name=f"Column_{f}", num_bins=MAX_BIN, upper_bounds=bounds[f].copy(), group=gi,
                                     column=col))
    b = B200Backend(0)
    times = []
    for it in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        b.bin_dense(x, feats, groups)
        if it >= args.warmup:
            times.append(time.perf_counter() - t0)
    b.close()
    s = sum(times) / len(times)
    print(json.dumps({"binning": {"rows": ROWS, "features": FEATURES, "ms": s * 1e3,
                                  "values_per_s": ROWS * FEATURES / s, "input": "device f32 row-major",
                                  "output": "host group rows", "steps": args.steps, "warmup": args.warmup}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="c2", choices=["c2", "c4"],
                    help="c2 (default): BASELINE configs[1]; c4: configs[3], the 100M-row scaling config")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows of the synthetic set (a smaller case for profiling; default: the config's)")
    ap.add_argument("--binning", action="store_true",
                    help="time the device binning of the config's raw features instead of training (one GPU)")
    args = ap.parse_args()
    set_config(args.config)
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
