"""The reference's own GPU histogram beside this build's (SURVEY's "reference GPU bar").

oracle/_ref/libref_gpu.so holds silvic-gpu's `hist_quant` kernel compiled from the reference's kernel text, with
the reference's launch math (oracle/ref_gpu.cu; built by `make -C oracle ref` where the reference checkout is present,
and carried to the GPU box with the repository). On the same rows and packed gradients the two root histograms must
be identical integers; at the bench's size both are timed and printed (`pytest -s`)."""

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

    data = bench.build_dataset(0, bench.ROWS, torch.device("cuda", 0))
    ours, ref, ours_s, ref_s = _both(data, (1.5, 0.75, None, 4, True, 9, 3), repeats=10)
    assert np.array_equal(ours, ref.astype(np.float64))
    n, S = data.num_rows, sum(g.row_stride for g in data.groups)
    bytes_root = n * (S + 4) + 8 * data.total_bins
    print(json.dumps({"rows": n, "features": len(data.features), "ours_ms": ours_s * 1e3, "reference_ms": ref_s * 1e3,
                      "speedup": ref_s / ours_s, "ours_gbs": bytes_root / ours_s / 1e9,
                      "reference_gbs": bytes_root / ref_s / 1e9}))
