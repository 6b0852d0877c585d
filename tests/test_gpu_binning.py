"""Device binning (`sb2_bin_dense`) against the oracle's bin_rows (data/binning.rs:71-135), byte for byte: the
reference's generated columns with LightGBM's thresholds, hashed matrices with NaN, signed zeros, infinities and
values on the bounds, f32 and f64, row- and column-major, host and device inputs, and a matrix larger than one
256 MB chunk."""

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


def test_categorical_is_unsupported(device):
    b = B200Backend(0)
    values, feats, groups = hashed_case(100, 4, seed=1)
    feats[2].kind = _abi.CATEGORICAL
    with pytest.raises(_abi.SilvicError):
        b.bin_dense(values, feats, groups)
    b.close()
