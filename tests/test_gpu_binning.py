"""Device binning (`sb2_bin_dense`) against the oracle's bin_rows (data/binning.rs:71-135), byte for byte: the
reference's generated columns with LightGBM's thresholds, hashed matrices with NaN, signed zeros, infinities and
values on the bounds, f32 and f64, row- and column-major, host and device inputs, a matrix larger than one
256 MB chunk, and categorical columns."""

from __future__ import annotations

import numpy as np
import pytest

import oracle_lib as orc
from binning_cases import hashed_case, lightgbm_case
from silvic_b200 import _abi
from silvic_b200.backend import B200Backend

pytestmark = pytest.mark.gpu


def check(b, values, feats, groups):
    want = orc.bin_rows(values, feats, groups)
    got = b.bin_dense(values, feats, groups)
    for g, (x, y) in enumerate(zip(got, want)):
        assert np.array_equal(x, y), f"group {g}: {int((x != y).sum())} bytes differ"
    return got


def test_lightgbm_columns(device):
    b = B200Backend(0)
    values, feats, groups = lightgbm_case()
    for v in (values, np.asfortranarray(values), values.astype(np.float32), np.asfortranarray(values.astype(np.float32))):
        check(b, v, feats, groups)
    b.close()


def test_hashed_matrices(device):
    b = B200Backend(0)
    for dtype in (np.float32, np.float64):
        for per_group in (1, 5, 32):
            values, feats, groups = hashed_case(3_001, 37, seed=7, dtype=dtype, per_group=per_group)
            check(b, values, feats, groups)
            check(b, np.asfortranarray(values), feats, groups)
    b.close()


def test_device_input_written_by_a_late_kernel(device):
    """A CUDA tensor whose last write is still queued on torch's stream when bin_dense is called: the values are
    binned as written, not as the memory held before (the library's stream is not ordered after torch's; the
    binding waits for the tensor's device). The write is held back by a spin on torch's stream."""
    import torch

    b = B200Backend(0)
    values, feats, groups = hashed_case(50_000, 24, seed=21, dtype=np.float32, per_group=8)
    want = orc.bin_rows(values, feats, groups)
    src = torch.from_numpy(values).cuda()
    for _ in range(2):
        t = torch.full_like(src, float("nan"))
        torch.cuda.synchronize()
        torch.cuda._sleep(200_000_000)  # about 0.1 s of SM cycles on torch's stream before the copy
        t.copy_(src)
        got = b.bin_dense(t, feats, groups)
        assert all(np.array_equal(x, y) for x, y in zip(got, want))
    b.close()


def test_device_input_and_chunks(device):
    """A CUDA tensor as input (row-major and its transpose), and 600,000 × 128 f32 values: two chunks."""
    import torch

    b = B200Backend(0)
    values, feats, groups = hashed_case(20_000, 24, seed=11, dtype=np.float32, per_group=8)
    want = orc.bin_rows(values, feats, groups)
    t = torch.from_numpy(values).cuda()
    for tensor in (t, t.t().contiguous().t()):
        got = b.bin_dense(tensor, feats, groups)
        assert all(np.array_equal(x, y) for x, y in zip(got, want))
    rng = np.random.default_rng(3)
    big = rng.standard_normal((600_000, 128), dtype=np.float32) * 5.0
    big[rng.random(big.shape) < 0.02] = np.nan
    _, feats_b, groups_b = hashed_case(4, 128, seed=13, dtype=np.float32, per_group=32)
    check(b, big, feats_b, groups_b)
    b.close()


def categorical_case(rows, seed, dtype):
    """hashed_case with every third feature categorical: categories listed in frequency order (not sorted), values
    that hit them, miss them, are negative, NaN, fractional (truncated) or beyond the i32 range."""
    from silvic_b200.dataset import FeatureMeta

    values, feats, groups = hashed_case(rows, 12, seed=seed, dtype=dtype, per_group=6)
    rng = np.random.default_rng(seed)
    out = []
    for f, m in enumerate(feats):
        if f % 3 != 1:
            out.append(m)
            continue
        cats = [int(c) for c in rng.choice(np.arange(0, 400), size=int(rng.integers(1, 200)), replace=False)]
        pick = rng.integers(0, 8, size=rows)
        col = np.where(pick < 5, np.array(cats)[rng.integers(0, len(cats), size=rows)] + rng.random(rows) * 0.99,
                       np.select([pick == 5, pick == 6], [np.nan, -rng.random(rows) * 5.0],
                                 rng.choice([1e12, -1e12, 401.0, 3.5e9], size=rows)))
        values[:, f] = col.astype(dtype)
        out.append(FeatureMeta(name=m.name, kind=_abi.CATEGORICAL, num_bins=len(cats) + 1, categories=cats,
                               group=m.group, column=m.column, hist_offset=m.hist_offset))
    return values, out, groups


def test_categorical_columns(device):
    """categorical_bin (data/bin_mapper.rs:379-391) on the device against the oracle's, f32 and f64, both layouts."""
    b = B200Backend(0)
    for dtype in (np.float32, np.float64):
        values, feats, groups = categorical_case(5_003, seed=21, dtype=dtype)
        got = check(b, values, feats, groups)
        check(b, np.asfortranarray(values), feats, groups)
        col = feats[1].column
        assert len(np.unique(got[feats[1].group][:, col])) > 10  # the categories are hit
    b.close()


def test_bad_categories_are_rejected(device):
    b = B200Backend(0)
    values, feats, groups = categorical_case(100, seed=2, dtype=np.float64)
    feats[1].categories = feats[1].categories[:1] * 2
    feats[1].num_bins = 3
    with pytest.raises(_abi.SilvicError, match="twice"):
        b.bin_dense(values, feats, groups)
    b.close()


def test_streaming_construction(device):
    """BinnedDataset.from_chunks: chunks of rows (uneven, host and device) binned into one dataset equal to the
    oracle's bin_rows of the whole matrix, with the layout of from_bins."""
    import torch

    from silvic_b200.dataset import BinnedDataset, layout

    values, feats, _ = categorical_case(10_007, seed=5, dtype=np.float32)
    mappers = [m for m in feats]
    _, shells, _ = layout(mappers)
    want = orc.bin_rows(values, layout(mappers)[0], shells)
    cuts = [0, 1, 4_000, 4_128, 9_999, 10_007]
    chunks = [(lo, values[lo:hi] if k % 2 else torch.from_numpy(values[lo:hi]).cuda())
              for k, (lo, hi) in enumerate(zip(cuts, cuts[1:]))]
    b = B200Backend(0)
    data = BinnedDataset.from_chunks(iter(chunks), len(values), mappers, np.zeros(len(values)), b)
    b.close()
    assert len(data.groups) == len(want)
    for g, (x, y) in enumerate(zip(data.groups, want)):
        assert np.array_equal(x.data, y), f"group {g}"
    with pytest.raises(ValueError, match="start at"):
        BinnedDataset.from_chunks(iter([(5, values[:10])]), 10, mappers, np.zeros(10), None)
