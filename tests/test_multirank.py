"""The multi-rank host logic of the bench on CPU: two `gloo` ranks (world_size 2) shard the synthetic dataset the way
`bench.py --gpus 2` does under torchrun, share a handle id the way the NCCL unique id is shared, and reduce their
timings with the max over ranks. The shards must tile the single-process dataset exactly (the device path's
row_offset keys quantization by global row), and every rank must see the same labels for the initial score; the
oracle's two-rank training equals the one-rank one (test_oracle.py::test_two_ranks_grow_the_tree_of_one)."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
ROWS = 3001  # odd, so the two shards differ in size
SAMPLE = 2000  # rows the bin boundaries are cut from (the bench's 200,000 would only slow the test)


def _rank(rank: int, world: int, port: int, out):
    sys.path.insert(0, str(ROOT))
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.set_rows(ROWS)
        bench.SAMPLE_ROWS = SAMPLE
        dev = torch.device("cpu")
        begin, end = bench.ROWS * rank // world, bench.ROWS * (rank + 1) // world
        data = bench.build_dataset(begin, end, dev)
        # the handle id travels as in bench.py (rank 0's bytes, broadcast)
        uid = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        # the timing: max over ranks
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        labels = bench.all_labels(dev)
        shards = [None] * world
        dist.all_gather_object(shards, (begin, end, data.row_offset, [g.data.copy() for g in data.groups],
                                        data.label.copy(), labels))
        if rank == 0:
            out.put((uid[0], float(t[0]), shards))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_tile_the_dataset():
    sys.path.insert(0, str(ROOT))
    import bench

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    uid, tmax, shards = out.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert uid == bytes(range(128))
    assert tmax == 2.0
    (b0, e0, off0, g0, l0, all0), (b1, e1, off1, g1, l1, all1) = shards
    assert (b0, e0, b1, e1) == (0, ROWS // 2, ROWS // 2, ROWS)
    assert (off0, off1) == (b0, b1)  # row_offset = rows of lower ranks
    bench.set_rows(ROWS)
    bench.SAMPLE_ROWS = SAMPLE
    full = bench.build_dataset(0, ROWS, torch.device("cpu"))
    for k, g in enumerate(full.groups):
        assert np.array_equal(np.concatenate([g0[k], g1[k]]), g.data)
    assert np.array_equal(np.concatenate([l0, l1]), full.label)
    assert np.array_equal(all0, all1) and np.array_equal(all0, full.label)
