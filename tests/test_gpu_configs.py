"""Device training against the CPU oracle at BASELINE sizes, through the C ABI.

The reference pins device == CPU model text byte for byte (crates/silvic-gpu/tests/metal_backend.rs:718-748); here
config c1 of BASELINE.json runs at full size (1,000,000 rows x 28 features, L2, 255 bins, 63 leaves, 100 trees),
its rows generated and binned as the bench does (sb2_bin_dense over counter-hash features), and the emitted model
must equal the oracle's: every tree field bit for bit, the LightGBM model text byte for byte, and f64 predictions
of the emitted file on raw features within 1e-9 relative of the oracle's Model::predict_raw_row. A second case
drives the leaf-sum kernel to its rows-per-CTA limit (20M rows)."""

from __future__ import annotations

import pytest

from silvic_b200 import _abi
from silvic_b200.backend import B200Backend, Model, init_score
import oracle_lib as orc
from synth import random_binned

pytestmark = pytest.mark.gpu

PREDICTION_RTOL = 1e-9  # f64 predictions of the emitted model vs the oracle's, relative


@pytest.fixture
def bench_config():
    """bench.py's synthetic configurations, restored to the default afterwards."""
    import bench

    yield bench
    bench.set_config("c4")


def test_c1_full_size_matches_oracle(device, bench_config):
    import torch

    from silvic_b200.model_text import TextModel

    bench = bench_config
    bench.set_config("c1")
    dev = torch.device("cuda", 0)
    data = bench.build_dataset(0, bench.ROWS, dev)
    assert data.num_rows == 1_000_000 and len(data.features) == 28
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=63, num_iterations=100, learning_rate=0.1,
                           num_grad_quant_bins=4)
    ref = orc.OracleTrainer([data], p)
    try:
        b = B200Backend(0)
        b.load(data, p.objective, p.sigmoid)
        model = b.train(p, init_score(p, data.label))
        b.close()
        assert model.init_score == ref.init_score
        assert len(model.trees) == len(ref.trees) == 100
        for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
            assert orc.trees_equal(t, r) == [], f"tree {k}"
        assert max(t.num_leaves for t in model.trees) == 63
        text = model.to_lightgbm_string(data, p)
        assert text == Model(ref.trees, ref.init_score, []).to_lightgbm_string(data, p)
        # Predictions of the emitted file (parsed back) on raw features of rows spread over the set.
        emitted = TextModel.from_string(text)
        rows = torch.arange(0, bench.ROWS, bench.ROWS // 500, dtype=torch.int64, device=dev)
        raw = bench.features_of(rows, dev).double().cpu().numpy()
        for row in raw:
            want = ref.predict_raw(row)
            got = emitted.predict_raw_row(row)
            assert abs(got - want) <= PREDICTION_RTOL * max(abs(want), 1e-300), (got, want)
    finally:
        ref.close()


def test_leaf_sums_at_the_rows_per_cta_limit(device):
    """The leaf sums add each fixed-point value as two 32-bit halves in shared memory, exact for at most 60,000
    rows a CTA; 20M rows make every CTA take close to that limit (about 59,000). Trees (their leaf values come from
    those sums) equal the oracle's."""
    data = random_binned(20_000_000, [255, 63], seed=21)
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=7, num_iterations=2)
    ref = orc.train([data], p)
    b = B200Backend(0)
    b.load(data, p.objective, p.sigmoid)
    model = b.train(p, init_score(p, data.label))
    b.close()
    assert len(model.trees) == len(ref.trees) == 2
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
