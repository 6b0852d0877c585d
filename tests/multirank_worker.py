"""One rank of tests/test_gpu_multirank.py, launched by torchrun (one process per GPU).

Every rank builds its contiguous row shard of a bench configuration (bench.py's synthetic data, binned by
sb2_bin_dense), joins the ranks with the chosen exchange (NVLink inside the tree kernel, or the NCCL fallback) and
trains. Rank 0 then trains the whole dataset on its one GPU and with the CPU oracle, and writes whether the N-rank
trees equal both, field by field, as JSON to the output path.

usage: torchrun ... multirank_worker.py <output.json> <auto|nccl> <config> <rows> <trees> <num_leaves> [share]

<config> is a bench configuration, or `categorical` for tests/synth.py's categorical dataset.

With `share`, every handle skips the dominant bins of the tiles that share picks (sb2_set_dominant_share).
"""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main():
    out_path, mode, config, rows, trees, leaves = sys.argv[1], sys.argv[2], sys.argv[3], *map(int, sys.argv[4:7])
    share = float(sys.argv[7]) if len(sys.argv) > 7 else None
    import torch
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        import bench
        import oracle_lib as orc
        from silvic_b200 import B200Backend, _abi, init_score, params_from_dict

        dev = torch.device("cuda", local)
        lo, hi = rows * rank // world, rows * (rank + 1) // world
        if config == "categorical":
            # two categorical features (one-hot and sorted scans) beside four numerical ones (tests/synth.py)
            from synth import categorical_binned

            whole = categorical_binned(rows, seed=17, label_kind="binary")
            p = params_from_dict(dict(objective="binary", num_iterations=trees, num_leaves=leaves,
                                      min_data_per_group=50, max_cat_threshold=16))
            s0 = init_score(p, whole.label)
            data = whole.shard(lo, hi)
        else:
            bench.set_config(config)
            bench.set_rows(rows)
            p = params_from_dict(dict(bench.params_dict(trees), num_leaves=leaves))
            s0 = init_score(p, bench.all_labels(dev))
            data = bench.build_dataset(lo, hi, dev)
        b = B200Backend(local)
        if share is not None:
            b.set_dominant_share(share)
        b.load(data, p.objective, p.sigmoid)
        b.set_rank_exchange(_abi.EXCHANGE_NCCL if mode == "nccl" else _abi.EXCHANGE_AUTO)
        uid = [B200Backend.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        b.join_ranks(uid[0], world, rank)
        model = b.train(p, s0)
        persistent = bool(model.tree_seconds)  # one tree-kernel launch per tree: the NVLink exchange ran
        b.close()
        dist.barrier()
        if rank == 0:
            full = whole if config == "categorical" else bench.build_dataset(0, rows, dev)
            one = B200Backend(local)
            if share is not None:
                one.set_dominant_share(share)
            one.load(full, p.objective, p.sigmoid)
            single = one.train(p, s0)
            one.close()
            ref = orc.train([full], p if config == "categorical" else
                            orc.default_params(objective=p.objective, num_leaves=leaves, num_iterations=trees,
                                               learning_rate=p.learning_rate,
                                               num_grad_quant_bins=p.num_grad_quant_bins))

            def differences(a, b_):
                if len(a) != len(b_):
                    return [f"{len(a)} trees vs {len(b_)}"]
                return [f"tree {k}: {','.join(d)}" for k, (x, y) in enumerate(zip(a, b_)) if (d := orc.trees_equal(x, y))]

            d_one = differences(model.trees, single.trees)
            d_ref = differences(model.trees, ref.trees)
            Path(out_path).write_text(json.dumps({
                "world": world, "mode": mode, "tree_kernel_exchange": persistent, "trees": len(model.trees),
                "leaves": [t.num_leaves for t in model.trees], "identical_to_one_gpu": not d_one,
                "identical_to_oracle": not d_ref, "differences": (d_one + d_ref)[:10]}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
