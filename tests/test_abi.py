"""The C-ABI library builds, loads without a GPU, and exports every function include/silvic_b200.h declares."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

from silvic_b200 import _abi, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "silvic_b200.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(sb2_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _abi.load_library(build.build())
    names = declared()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_abi.SIGNATURES), set(names) ^ set(_abi.SIGNATURES)


def test_default_params_are_the_reference_defaults():
    lib = _abi.load_library(build.build())
    p = _abi.Params()
    lib.sb2_default_params(C.byref(p))
    assert (p.num_iterations, p.learning_rate, p.num_leaves, p.min_data_in_leaf) == (100, 0.1, 31, 20)
    assert (p.use_quantized_grad, p.num_grad_quant_bins, p.quant_train_renew_leaf, p.stochastic_rounding) == (1, 4, 1, 1)
    assert (p.bagging_seed, p.feature_fraction_seed, p.data_random_seed) == (3, 2, 1)


def test_boost_from_average_in_row_order():
    lib = _abi.load_library(build.build())
    p = _abi.Params()
    lib.sb2_default_params(C.byref(p))
    label = (C.c_float * 3)(1.0, 2.0, 4.0)
    weight = (C.c_float * 3)(1.0, 0.5, 2.0)
    out = C.c_double()
    assert lib.sb2_boost_from_average(C.byref(p), label, weight, 3, C.byref(out)) == 0
    assert abs(out.value - (1.0 + 1.0 + 8.0) / 3.5) < 1e-12
    p.objective = _abi.BINARY
    assert lib.sb2_boost_from_average(C.byref(p), label, None, 3, C.byref(out)) == 0
    k = float(C.c_float(1e-15).value)
    rate = 1.0 - k
    import math

    assert out.value == math.log(rate / (1.0 - rate))


def test_create_without_gpu_fails_cleanly():
    lib = _abi.load_library(build.build())
    import torch

    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    assert lib.sb2_create(0, C.byref(h)) == _abi.EDEVICE
    assert "device" in _abi.global_error().lower()
