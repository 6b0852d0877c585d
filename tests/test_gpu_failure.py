"""Failure detection in the tree kernel's rank exchange, on one GPU and without a GPU fault.

The reference tests that a rank which never answers makes the others time out with an error instead of hanging
(crates/silvic-net/tests/ring.rs:338, `hung_rank_times_out`). Here the handle trains as rank 0 of two ranks whose
other rank's exchange buffer is local memory that nothing writes (sb2_test_unanswered_peer): the first wait for that
rank's histogram bins runs out of polls, the kernel records error 4 and every CTA returns, and sb2_train reports a
collective error promptly. The handle then trains as one rank again and matches the oracle."""

from __future__ import annotations

import time

import pytest

from silvic_b200 import SilvicError, _abi
from silvic_b200.backend import B200Backend, init_score
import oracle_lib as orc
from synth import random_binned

pytestmark = pytest.mark.gpu


def test_unanswered_rank_times_out_and_the_handle_recovers(device):
    data = random_binned(50_000, [255] * 8 + [31] * 4, seed=4)
    p = orc.default_params(objective=_abi.REGRESSION, num_leaves=15, num_iterations=2)
    s0 = init_score(p, data.label)
    b = B200Backend(0)
    try:
        b.load(data, p.objective, p.sigmoid)
        b.test_unanswered_peer(1 << 12)  # a few milliseconds of polls
        t0 = time.perf_counter()
        with pytest.raises(SilvicError) as err:
            b.train(p, s0)
        elapsed = time.perf_counter() - t0
        assert err.value.code == _abi.ECOLLECTIVE, str(err.value)
        assert "did not reach" in str(err.value)
        assert elapsed < 20.0, elapsed
        # The context is intact: the same handle, one rank again, grows the oracle's trees.
        b.test_unanswered_peer(0)
        model = b.train(p, s0)
    finally:
        b.close()
    ref = orc.train([data], p)
    assert len(model.trees) == len(ref.trees) == 2
    for k, (t, r) in enumerate(zip(model.trees, ref.trees)):
        assert orc.trees_equal(t, r) == [], f"tree {k}"
