"""The oracle at the full Qwen1.5-MoE-A2.7B block shapes against the
reference's own outputs on the same seeded workloads (tests/golden/moe_qwen.npz).
Also pins the synthetic generators: the regenerated weights must hash to
what the reference was given."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
from conftest import golden
from helpers import oracle_weights

from expertrelay_b200 import synth
from oracle import moe_oracle as O


def _sha(a) -> bytes:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest().encode()


@pytest.fixture(scope="module")
def g():
    return golden("moe_qwen")


def test_decode8_block(g):
    blk, x = synth.make_workload("decode8_int8", seed=0)
    assert _sha(blk.records()) == g["decode8_records_sha"].tobytes()
    assert _sha(blk.shared_record()) == g["decode8_shared_sha"].tobytes()
    assert _sha(blk.router) == g["decode8_router_sha"].tobytes()
    np.testing.assert_array_equal(x, g["decode8_x"])
    out = O.moe_block(x, oracle_weights(blk))
    np.testing.assert_array_equal(out.selected, g["decode8_sel"])
    assert O.rel_l2(out.y, g["decode8_y_blocked"]) < 1e-6
    assert O.rel_l2(out.y, g["decode8_y_fused"]) < 1e-5  # the reference's numba decode kernel
    assert 20 <= len(out.unique_experts) <= 32


def test_prefill4096_zipf_block(g):
    blk, x = synth.make_workload("prefill4096_int8_zipf", seed=0)
    assert _sha(blk.router) == g["prefill_router_sha"].tobytes()
    counts = np.array(blk.meta["zipf"]["realised"])
    np.testing.assert_array_equal(counts, g["prefill_zipf_realised"])
    # imbalanced: the busiest expert gets many times the median's tokens
    assert counts.max() > 8 * np.median(counts) and counts.sum() == 4096 * 4
    out = O.moe_block(x, oracle_weights(blk))
    np.testing.assert_array_equal(out.selected.astype(np.int8), g["prefill_sel"])
    assert O.rel_l2(out.y[:32], g["prefill_y_head"]) < 1e-6
    np.testing.assert_allclose(np.linalg.norm(out.y.astype(np.float64), axis=1), g["prefill_y_rownorm"], rtol=1e-5)
