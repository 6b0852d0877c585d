"""silvic_b200 — silvic's quantized-histogram training path on NVIDIA B200 (sm_100a).

The package is a drop-in backend for silvic's `trait Backend` (crates/silvic-core/src/backend/mod.rs:115-179):
`B200Backend` mirrors the trait method for method over the C ABI of include/silvic_b200.h, and `train()` runs
silvic's boosting loop with every split on the device. The compiled library lives in silvic_b200/_lib; without it
(or without a B200) every entry point raises instead of computing on the CPU.
"""

from ._abi import SilvicError, load_library
from .backend import B200Backend, Model, Tree, init_score, params_from_dict, train
from .dataset import BinnedDataset, FeatureGroup, FeatureMeta, numerical_mapper

__all__ = [
    "B200Backend",
    "BinnedDataset",
    "FeatureGroup",
    "FeatureMeta",
    "Model",
    "SilvicError",
    "Tree",
    "init_score",
    "load_library",
    "numerical_mapper",
    "params_from_dict",
    "train",
]
