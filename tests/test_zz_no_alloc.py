"""sb2_find_best_split_noalloc, the split search for callers that cannot let a call allocate device memory: its
results, taken through the C ABI from device buffers the test owns, equal sb2_find_best_split's on the same inputs,
on two calls in a row (the second reuses the scratch the first left behind), and the CPU oracle's find_best_split
(a restatement of crates/silvic-core/src/split.rs:919-961 that shares no code with the device search). It has no
counterpart in the reference. Collected last so it also runs after every other test in one process."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend
import oracle_lib as orc
from synth import random_binned

pytestmark = pytest.mark.gpu

MAX_FEATURES = 4096  # the scratch's limit, as the header states


def random_hist(rng, data):
    """Integer-valued quantized histograms with positive hessians."""
    h = np.zeros(2 * data.total_bins)
    for m in data.features:
        n = rng.integers(0, 40, size=m.num_bins)
        h[2 * m.hist_offset: 2 * (m.hist_offset + m.num_bins): 2] = rng.integers(-2 * n, 2 * n + 1)
        h[2 * m.hist_offset + 1: 2 * (m.hist_offset + m.num_bins): 2] = n * 4
    return h


def leaf_sums(data, hist):
    m0 = data.features[0]
    g = hist[2 * m0.hist_offset: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    h = hist[2 * m0.hist_offset + 1: 2 * (m0.hist_offset + m0.num_bins): 2].sum()
    return g, h, int(h // 4)


def noalloc_search(b, hist, evaluate, sums, scale, cfg):
    """sb2_find_best_split_noalloc over device copies of `hist` (as int32) and `evaluate`."""
    import torch

    dev = torch.device("cuda", 0)
    d_hist = torch.from_numpy(hist.astype(np.int32)).to(dev)
    d_eval = torch.from_numpy(evaluate.astype(np.uint8)).to(dev)
    d_out = torch.zeros(C.sizeof(_abi.SplitInfo), dtype=torch.uint8, device=dev)
    d_spl = torch.zeros(len(evaluate), dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()  # the inputs are written before the call reads them on its own stream
    rc = b._lib.sb2_find_best_split_noalloc(
        b._h, C.c_void_p(d_hist.data_ptr()), len(hist), C.c_void_p(d_eval.data_ptr()), sums[0], sums[1], sums[2],
        scale[0], scale[1], C.byref(cfg), C.c_void_p(d_out.data_ptr()), C.c_void_p(d_spl.data_ptr()))
    b._check(rc)
    info = _abi.SplitInfo.from_buffer_copy(d_out.cpu().numpy().tobytes())
    return info, d_spl.cpu().numpy()


def test_noalloc_split_matches_find_best_split(device):
    rng = np.random.default_rng(7)
    nb = [int(x) for x in rng.integers(2, 256, size=45)]
    nan = [bool(x) for x in rng.integers(0, 2, size=len(nb))]
    data = random_binned(64, nb, nan_bins=nan, seed=5)
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    try:
        cases = [
            (_abi.SplitConfig(5, 1e-3, 0.5, 2.0, 0.0), (0.37, 0.25)),
            (_abi.SplitConfig(20, 0.0, 0.0, 10.0, 0.1), (1.5, 0.5)),
        ]
        for k, (cfg, scale) in enumerate(cases):  # two calls in a row on one handle and one scratch
            hist = random_hist(rng, data)
            evaluate = (rng.random(len(nb)) < 0.8).astype(np.uint8)
            sums = leaf_sums(data, hist)
            want, want_spl = b.find_best_split(hist, evaluate, sums, scale, cfg)
            got, got_spl = noalloc_search(b, hist, evaluate, sums, scale, cfg)
            # The same kernel on the same integer histogram: equal bit for bit (the tolerance is zero).
            assert got.as_tuple() == want.as_tuple(), f"call {k}"
            assert np.array_equal(got_spl, want_spl), f"call {k}"
            assert want.found, f"call {k} should find a split"
            # And the CPU oracle's search on the same histogram: the same split, bit for bit.
            ref, ref_spl = orc.find_best_split(data, hist, evaluate, sums, scale, cfg)
            assert got.as_tuple() == ref.as_tuple(), f"call {k} differs from the oracle"
            assert np.array_equal(got_spl, ref_spl), f"call {k}: splittable differs from the oracle"
    finally:
        b.close()


def test_noalloc_split_rejects_host_buffers(device):
    data = random_binned(64, [31, 7], seed=1)
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    try:
        hist = np.zeros(2 * data.total_bins, dtype=np.int32)
        flags = np.ones(2, dtype=np.uint8)
        info = _abi.SplitInfo()
        rc = b._lib.sb2_find_best_split_noalloc(
            b._h, hist.ctypes.data_as(C.c_void_p), len(hist), flags.ctypes.data_as(C.c_void_p), 0.0, 0.0, 0, 1.0,
            1.0, C.byref(_abi.SplitConfig(1, 0.0, 0.0, 0.0, 0.0)), C.cast(C.byref(info), C.c_void_p),
            flags.ctypes.data_as(C.c_void_p))
        assert rc == 4  # SB2_EDEVICE
        buf = C.create_string_buffer(512)
        b._lib.sb2_last_error(b._h, buf, len(buf))
        assert b"is not memory of device" in buf.value
    finally:
        b.close()


def test_noalloc_split_rejects_too_many_features(device):
    data = random_binned(32, [2] * (MAX_FEATURES + 1), seed=2)
    b = B200Backend(0)
    b.load(data, _abi.REGRESSION, 1.0)
    try:
        rc = b._lib.sb2_find_best_split_noalloc(
            b._h, None, 2 * data.total_bins, None, 0.0, 0.0, 0, 1.0, 1.0,
            C.byref(_abi.SplitConfig(1, 0.0, 0.0, 0.0, 0.0)), None, None)
        assert rc == 7  # SB2_EUNSUPPORTED
        buf = C.create_string_buffer(512)
        b._lib.sb2_last_error(b._h, buf, len(buf))
        assert f"its scratch holds {MAX_FEATURES}".encode() in buf.value
    finally:
        b.close()
