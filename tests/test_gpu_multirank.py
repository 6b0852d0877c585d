"""Two ranks grow the trees of one GPU (the reference pins this as `two_ranks_grow_the_tree_of_one`,
crates/silvic-core/src/learner.rs:709-722, and `two_ranks_train_the_model_of_one`,
crates/silvic-core/tests/train_cpu.rs:270-286).

Two processes (torchrun, one per GPU) each hold a contiguous row shard and join with sb2_join_ranks; their trees must
equal, field by field, the trees one GPU grows on the whole dataset and the CPU oracle's. Both exchanges run: the
tree kernel's own over NVLink (the default) and the NCCL fallback (per-step launches with an ncclAllReduce of each
split's histogram). Four and eight ranks run the NVLink exchange alike when that many GPUs are visible. Skipped with
fewer GPUs. NVLS is off (NCCL_NVLS_ENABLE=0): the exchange uses plain peer stores and NCCL only small reductions."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
WORKER = Path(__file__).resolve().parent / "multirank_worker.py"


# config c2's shape (100 features, binary) at 1M rows: 255-leaf trees run grid steps of eight splits; c5's (2,000
# features, 80% of them 95% zeros) at 200K rows with the dominant-bin skip: every rank skips its own most frequent
# bins and recovers them from its own totals before the exchange; categorical features, whose candidates carry their
# left bins through the exchange; c4's (256 features in two histogram units, L2 with a constant hessian)
CASES = [("c2", 1_000_000, 3, 255, None), ("c5", 200_000, 3, 31, 0.125), ("categorical", 400_000, 3, 63, None),
         ("c4", 2_000_000, 2, 255, None)]


def run_ranks(world, mode, config, rows, trees, leaves, share, tmp_path, port):
    out = tmp_path / "result.json"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", f"--master-port={port}", str(WORKER), str(out),
           mode, config, str(rows), str(trees), str(leaves)] + ([str(share)] if share is not None else [])
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    run = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    assert run.returncode == 0, (run.stdout[-4000:], run.stderr[-4000:])
    return json.loads(out.read_text())


@pytest.mark.parametrize("config,rows,trees,leaves,share", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("mode", ["auto", "nccl"])
def test_two_ranks_grow_the_trees_of_one_gpu(device, mode, config, rows, trees, leaves, share, tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    port = 29500 + (os.getpid() + (0 if mode == "auto" else 7) + 13 * [c[0] for c in CASES].index(config)) % 2000
    res = run_ranks(2, mode, config, rows, trees, leaves, share, tmp_path, port)
    assert res["world"] == 2 and res["trees"] == trees
    assert res["tree_kernel_exchange"] == (mode == "auto"), res
    assert res["identical_to_one_gpu"], res["differences"]
    assert res["identical_to_oracle"], res["differences"]


@pytest.mark.parametrize("world", [4, 8])
def test_more_ranks_grow_the_trees_of_one_gpu(device, world, tmp_path):
    """The NVLink exchange at 4 and 8 ranks (every feature's owner f mod world, a rank's pushes to every other), on
    config 2's shape: the trees of one GPU and of the oracle."""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = 29500 + (os.getpid() + 101 + world) % 2000
    res = run_ranks(world, "auto", "c2", 1_000_000, 3, 255, None, tmp_path, port)
    assert res["world"] == world and res["trees"] == 3
    assert res["tree_kernel_exchange"], res
    assert res["identical_to_one_gpu"], res["differences"]
    assert res["identical_to_oracle"], res["differences"]
