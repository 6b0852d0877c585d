"""The measurement entry points that explain the histogram's roofline: the shared-memory atomic rate alone, at the
histogram's address patterns, and the standalone histogram's rate against it."""

from __future__ import annotations

import math

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend
import oracle_lib as orc
from synth import random_binned

pytestmark = pytest.mark.gpu


def test_shared_add_rate_is_measured(device):
    b = B200Backend(0)
    try:
        for pattern in (0, 1):
            per_s, per_clk = b.time_shared_adds(pattern)
            assert math.isfinite(per_s) and per_s > 1e11, (pattern, per_s)
            # at most one lane add per bank per SM clock
            assert 0.0 < per_clk <= 32.0, (pattern, per_clk)
            print(f"pattern {pattern}: {per_s:.3e} lane adds/s, {per_clk:.2f} per SM clock")
        with pytest.raises(_abi.SilvicError):
            b.time_shared_adds(2)
    finally:
        b.close()


def test_root_histogram_rate_below_the_atomic_rate(device):
    """The root histogram adds one packed gradient per (row, feature): its atomic rate cannot pass the rate of the
    adds alone, and the histogram it times is the oracle's."""
    data = random_binned(400_000, [255] * 128, seed=11)
    b = B200Backend(0)
    try:
        b.load(data, _abi.REGRESSION, 1.0)
        r = np.arange(data.num_rows)
        grad = ((r * 7) % 13).astype(np.float32) / 4.0 - 1.5
        hess = np.ones(data.num_rows, dtype=np.float32)
        b.write_gradients(grad, hess)
        spec = orc.quant_spec(1.5, 1.0, None, 4, True, 3, 0)
        b.quantize(spec)
        n = b.reset_partition()
        want = orc.histogram(data, b.read_packed(), np.arange(n))
        assert np.array_equal(b.histogram(0, n), want)
        secs = b.time_histogram(5)
        alone = b.time_shared_adds(0)[0]
        rate = data.num_rows * 128 / secs
        assert rate < 1.05 * alone, (rate, alone)
    finally:
        b.close()
