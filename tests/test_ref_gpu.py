"""The reference's own GPU kernels beside this build's and the CPU oracle's.

oracle/_ref/libref_gpu.so holds silvic-gpu's kernels compiled from the reference's kernel text, driven with the
reference's launch math (oracle/ref_gpu.cu; built by `make -C oracle ref REF=<checkout>` where the reference checkout
is present, and carried to the GPU box with the repository). On the same inputs:
  - the reference's `hist_quant` and this build's root histogram are identical integers, and both are timed at the
    bench's config-2 size (`pytest -s` prints them);
  - the reference's quantize, grad_regression, partition (count/scan/scatter), bagging, leaf_sums and add_tree
    kernels equal the CPU oracle bit for bit, pinning those parts of the oracle on outputs the reference itself
    produced; grad_binary, which the reference computes in f32 (expf) where its CPU path uses f64, is compared within
    f32 rounding and its bit mismatches are counted."""

import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "oracle" / "_ref" / "libref_gpu.so"

pytestmark = pytest.mark.gpu


def _ref():
    if not LIB.exists():
        pytest.skip("the reference's GPU histogram is not built (make -C oracle ref, where the reference is present)")
    lib = C.CDLL(str(LIB))
    lib.ref_hist_create.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]
    lib.ref_hist_run.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_double), C.c_void_p]
    lib.ref_hist_destroy.argtypes = [C.c_void_p]
    lib.ref_gpu_last_error.restype = C.c_char_p
    return lib


def _packed_rows_cap(spec) -> int:
    """packed_block_rows (crates/silvic-gpu/src/backend.rs:622-632)."""
    if spec.constant_hessian:
        return max(32767 // max(spec.grad_max_q, 1), 1)
    return max(32767 // max(spec.grad_max_q, spec.hess_max_q), 1)


def _both(data, spec_args, repeats=0):
    """Our root histogram and the reference kernel's on `data` with the same packed gradients; their seconds."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle_lib as orc
    from test_gpu_parity import loaded, set_gradients

    lib = _ref()
    b = loaded(data)
    set_gradients(b, data)
    spec = orc.quant_spec(*spec_args)
    b.quantize(spec)
    packed = np.ascontiguousarray(b.read_packed())
    n = b.reset_partition()
    ours = b.histogram(0, n)
    ours_s = b.time_histogram(repeats) if repeats else 0.0
    b.close()
    d = data.c_struct()
    h = C.c_void_p()
    assert lib.ref_hist_create(C.addressof(d), packed.ctypes.data, _packed_rows_cap(spec), C.byref(h)) == 0, \
        lib.ref_gpu_last_error()
    try:
        out = np.zeros(2 * data.total_bins, dtype=np.int32)
        secs = C.c_double()
        assert lib.ref_hist_run(h, max(repeats, 1), C.byref(secs), out.ctypes.data) == 0, lib.ref_gpu_last_error()
    finally:
        lib.ref_hist_destroy(h)
    return ours, out, ours_s, secs.value


@pytest.mark.parametrize("quant_bins", [4, 16])
def test_reference_gpu_histogram_equals_ours(device, quant_bins):
    from synth import random_binned

    data = random_binned(100_000, [255] * 40 + [63] * 20 + [5, 2], seed=7)
    ours, ref, _, _ = _both(data, (1.5, 0.75, None, quant_bins, True, 9, 3))
    for m in data.features:
        sl = slice(2 * m.hist_offset, 2 * (m.hist_offset + m.num_bins))
        assert np.array_equal(ours[sl], ref[sl].astype(np.float64)), m.name


def test_reference_gpu_histogram_timing(device):
    """The bench's dataset (configs[1], 10M x 100, 4 quant bins): both root histograms timed on this GPU."""
    import torch

    sys.path.insert(0, str(ROOT))
    import bench

    bench.set_config("c2")
    try:
        data = bench.build_dataset(0, bench.ROWS, torch.device("cuda", 0))
    finally:
        bench.set_config("c4")
    ours, ref, ours_s, ref_s = _both(data, (1.5, 0.75, None, 4, True, 9, 3), repeats=10)
    assert np.array_equal(ours, ref.astype(np.float64))
    n, S = data.num_rows, sum(g.row_stride for g in data.groups)
    bytes_root = n * (S + 4) + 8 * data.total_bins
    print(json.dumps({"rows": n, "features": len(data.features), "ours_ms": ours_s * 1e3, "reference_ms": ref_s * 1e3,
                      "speedup": ref_s / ours_s, "ours_gbs": bytes_root / ours_s / 1e9,
                      "reference_gbs": bytes_root / ref_s / 1e9}))


# ---- the reference's other kernels against the oracle --------------------------------------------------------

def _lib2():
    lib = _ref()
    if not hasattr(lib, "ref_quantize"):
        pytest.skip("oracle/_ref/libref_gpu.so predates the training-kernel harness")
    P = C.c_void_p
    lib.ref_quantize.argtypes = [P, P, P, C.c_uint32, C.c_uint64, P]
    lib.ref_gradients.argtypes = [C.c_int, C.c_float, P, P, P, C.c_uint32, P, P]
    lib.ref_partition.argtypes = [P, P, C.c_uint32, P, P, P]
    lib.ref_bag.argtypes = [C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, C.c_double, P, P]
    lib.ref_leaf_sums.argtypes = [P, P, C.c_uint32, P, P, C.c_uint32, C.c_float, C.c_float, P]
    lib.ref_add_tree.argtypes = [P, P, C.c_uint32, P, C.c_uint32, P]
    return lib


def _gradients(n, seed):
    rng = np.random.default_rng(seed)
    grad = (rng.normal(size=n) * 1.3).astype(np.float32)
    hess = (0.05 + rng.random(n)).astype(np.float32)
    grad[::97] = 0.0  # exact zeros and the extremes
    grad[1] = np.abs(grad).max()
    grad[2] = -np.abs(grad).max()
    return grad, hess


@pytest.mark.parametrize("bins,constant,stochastic,offset", [
    (4, None, True, 0), (16, None, True, 3_000_000), (4, 1.0, True, (1 << 32) - 1000), (64, None, False, 77)])
def test_reference_quantize_equals_oracle(device, bins, constant, stochastic, offset):
    import oracle_lib as orc

    lib = _lib2()
    grad, hess = _gradients(200_003, bins)
    if constant is not None:
        hess[:] = 1.0
    spec = orc.quant_spec(float(np.abs(grad).max()), float(hess.max()), constant, bins, stochastic, 11, 5)
    ref = np.empty(len(grad), dtype=np.int32)
    assert lib.ref_quantize(C.addressof(spec), grad.ctypes.data, hess.ctypes.data, len(grad), offset,
                            ref.ctypes.data) == 0, lib.ref_gpu_last_error()
    assert np.array_equal(ref, orc.quantize(spec, grad, hess, row_offset=offset))


@pytest.mark.parametrize("weighted", [False, True])
def test_reference_gradients_against_oracle(device, weighted):
    """L2: bit for bit. Binary: the reference's GPU kernel is f32 (expf) while its CPU path, which the oracle and this
    build follow, is f64; they agree to f32 rounding and the bits that differ are counted."""
    import oracle_lib as orc

    from silvic_b200 import _abi

    lib = _lib2()
    rng = np.random.default_rng(3)
    n = 100_000
    scores = (rng.normal(size=n) * 2.0).astype(np.float32)
    label_r = rng.normal(size=n).astype(np.float32)
    label_b = (rng.random(n) < 0.4).astype(np.float32)
    weight = (0.5 + rng.random(n)).astype(np.float32) if weighted else None
    wp = None if weight is None else weight.ctypes.data
    g = np.empty(n, np.float32)
    h = np.empty(n, np.float32)
    assert lib.ref_gradients(_abi.REGRESSION, 1.0, scores.ctypes.data, label_r.ctypes.data, wp, n, g.ctypes.data,
                             h.ctypes.data) == 0, lib.ref_gpu_last_error()
    og, oh = orc.gradients(_abi.REGRESSION, scores, label_r, weight)
    assert np.array_equal(g, og) and np.array_equal(h, oh)
    assert lib.ref_gradients(_abi.BINARY, 1.0, scores.ctypes.data, label_b.ctypes.data, wp, n, g.ctypes.data,
                             h.ctypes.data) == 0, lib.ref_gpu_last_error()
    og, oh = orc.gradients(_abi.BINARY, scores, label_b, weight)
    assert np.allclose(g, og, rtol=2e-6, atol=1e-7) and np.allclose(h, oh, rtol=2e-6, atol=1e-7)
    mismatches = int((g.view(np.uint32) != og.view(np.uint32)).sum() + (h.view(np.uint32) != oh.view(np.uint32)).sum())
    print(json.dumps({"grad_binary_bit_mismatches": mismatches, "values": 2 * n, "weighted": weighted}))


def test_reference_partition_and_bagging_equal_oracle(device):
    import oracle_lib as orc
    from synth import random_binned

    from silvic_b200 import _abi

    lib = _lib2()
    data = random_binned(150_000, [255] * 6 + [63] * 40 + [3], seed=12)
    rng = np.random.default_rng(8)
    rows = rng.permutation(data.num_rows).astype(np.uint32)[:123_457]
    d = data.c_struct()
    for f in [0, 3, 10, 45, 46]:
        m = data.features[f]
        split = _abi.BinSplit(m.group, m.column)
        for b_ in rng.choice(m.num_bins, size=max(1, m.num_bins // 2), replace=False):
            split.left_bins[int(b_) // 32] |= 1 << (int(b_) % 32)
        out = np.empty(len(rows), np.uint32)
        left = C.c_uint32()
        assert lib.ref_partition(C.addressof(d), rows.ctypes.data, len(rows), C.addressof(split), out.ctypes.data,
                                 C.addressof(left)) == 0, lib.ref_gpu_last_error()
        want_left, want = orc.partition(data, split, rows)
        assert left.value == want_left and np.array_equal(out, want), f"feature {f}"
    for fraction, offset in [(0.5, 0), (0.1, 12345), (0.9, (1 << 32) + 7)]:
        out = np.empty(data.num_rows, np.uint32)
        count = C.c_uint32()
        assert lib.ref_bag(data.num_rows, offset, 4, 2, fraction, out.ctypes.data, C.addressof(count)) == 0
        want = orc.reset_partition(_abi.BagSpec(1, 4, 2, 0, fraction), data.num_rows, offset)
        assert count.value == len(want) and np.array_equal(out[:count.value], want), fraction


def test_reference_leaf_sums_and_add_tree_equal_oracle(device):
    import oracle_lib as orc
    from synth import random_binned

    from silvic_b200 import _abi

    lib = _lib2()
    data = random_binned(90_001, [255] * 4 + [31] * 8, seed=13)
    n = data.num_rows
    grad, hess = _gradients(n, 5)
    rng = np.random.default_rng(2)
    part = rng.permutation(n).astype(np.uint32)
    cuts = [0, 1, 4096, 4097, 30_000, 77_000, n]
    leaves = [(cuts[i], cuts[i + 1] - cuts[i]) for i in range(len(cuts) - 1)]
    arr = (_abi.LeafRange * len(leaves))(*[_abi.LeafRange(b, c) for b, c in leaves])
    gs = float(orc.lib().orc_fixed_point_scale(float(np.abs(grad).max())))
    hs = float(orc.lib().orc_fixed_point_scale(float(hess.max())))
    out = np.empty(2 * len(leaves), np.int64)
    assert lib.ref_leaf_sums(grad.ctypes.data, hess.ctypes.data, n, part.ctypes.data, C.addressof(arr), len(leaves),
                             gs, hs, out.ctypes.data) == 0, lib.ref_gpu_last_error()
    assert np.array_equal(out.reshape(-1, 2), orc.leaf_sums(grad, hess, part, leaves, gs, hs))
    # a three-node tree on three features, then a single-leaf tree
    d = data.c_struct()
    nodes = []
    for k, f in enumerate([2, 7, 9]):
        m = data.features[f]
        sp = _abi.BinSplit(m.group, m.column)
        for b_ in range(0, m.num_bins // 2):
            sp.left_bins[b_ // 32] |= 1 << (b_ % 32)
        nodes.append(_abi.DeviceNode(sp, k + 1 if k < 2 else ~2, ~k if k < 2 else ~3))
    leaf_values = np.array([0.5, -0.25, 0.125, 1.5], dtype=np.float32)
    scores = rng.normal(size=n).astype(np.float32)
    for tree_nodes, values in [(nodes, leaf_values), ([], leaf_values[:1])]:
        arr = (_abi.DeviceNode * max(len(tree_nodes), 1))(*tree_nodes)
        ref = scores.copy()
        assert lib.ref_add_tree(C.addressof(d), C.addressof(arr), len(tree_nodes), values.ctypes.data, len(values),
                                ref.ctypes.data) == 0, lib.ref_gpu_last_error()
        assert np.array_equal(ref, orc.add_tree(data, tree_nodes, values, scores))
