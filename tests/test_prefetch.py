"""CPU: the prefetch policy and calibration maps against the reference's.

tests/golden/prefetch.npz holds, for seeded router logits (one token and
several, 16 and 60 experts, and an exact tie), the experts that the
reference's PrefetchPolicy (predictor/prefetch_policy.py:41-54) picks and
the guesses it skips, with no calibration, a single isotonic map and a
per-rank map fitted by the reference's own fit (predictor/offline.py), at
three top-k sizes; and each map's predictions. tests/golden/prefetch_maps.json
is the maps' JSON form as the reference writes it. Everything must agree
exactly.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import GOLDEN, golden

from expertrelay_b200.prefetch import (
    IsotonicCalibrator,
    PrefetchPolicy,
    RankedIsotonicCalibrator,
    expert_scores,
    load_calibrator,
    rank_positions,
)


@pytest.fixture(scope="module")
def fx():
    maps = json.loads((GOLDEN / "prefetch_maps.json").read_text())
    return golden("prefetch"), maps


def _policies(maps):
    single = IsotonicCalibrator.from_dict(maps["calibrator"])
    ranked = RankedIsotonicCalibrator.from_dict(maps["rank_calibrator"])
    return single, ranked, (("plain", None, 0.0), ("single", single, 0.3), ("ranked", ranked, 0.3),
                            ("ranked_hi", ranked, 0.7))


def test_choices_match_the_reference(fx):
    g, maps = fx
    _, _, policies = _policies(maps)
    for c in range(maps["cases"]):
        logits = g[f"logits{c}"]
        for name, cal, pmin in policies:
            for k in (1, 4, 8):
                choice = PrefetchPolicy(top_k=k, min_probability=pmin, calibrator=cal).choose(logits)
                assert choice.experts == g[f"experts{c}_{name}_k{k}"].tolist(), (c, name, k)
                assert choice.skipped_low_confidence == int(g[f"skipped{c}_{name}_k{k}"][0]), (c, name, k)


def test_map_predictions_match_the_reference(fx):
    g, maps = fx
    single, ranked, _ = _policies(maps)
    for c in range(maps["cases"]):
        logits = g[f"logits{c}"]
        np.testing.assert_array_equal(single.predict(logits.ravel()), g[f"single_pred{c}"])
        p = np.exp(logits) / np.exp(logits).sum(axis=-1, keepdims=True)
        np.testing.assert_array_equal(ranked.predict(p), g[f"ranked_pred{c}"])


def test_maps_round_trip_to_the_same_json(fx):
    _, maps = fx
    single, ranked, _ = _policies(maps)
    assert single.to_dict() == maps["calibrator"]
    assert ranked.to_dict() == maps["rank_calibrator"]


def test_scores_and_ranks():
    logits = np.log(np.array([[0.7, 0.1, 0.1, 0.1], [0.1, 0.1, 0.1, 0.7]], dtype=np.float32))
    np.testing.assert_allclose(expert_scores(logits), [0.7, 0.1, 0.1, 0.7], rtol=1e-6)
    np.testing.assert_array_equal(rank_positions(np.array([0.3, 0.4, 0.3, 0.1])), [1, 0, 2, 3])
    with pytest.raises(ValueError):
        expert_scores(np.zeros((2, 0), dtype=np.float32))


def test_load_calibrator_takes_the_last_record(tmp_path, fx):
    _, maps = fx
    rec = {"calibrator": maps["calibrator"], "rank_calibrator": maps["rank_calibrator"], "git_commit": "abc",
           "timestamp": "t", "model": {"store": "s"}}
    path = tmp_path / "cal.json"
    path.write_text(json.dumps([{"calibrator": maps["calibrator"]}, rec]))
    cal, prov = load_calibrator(path)
    assert isinstance(cal, RankedIsotonicCalibrator)
    assert prov == {"file": "cal.json", "git_commit": "abc", "timestamp": "t", "store": "s", "kind": "rank_isotonic"}
    cal, prov = load_calibrator(path, kind="single")
    assert isinstance(cal, IsotonicCalibrator) and prov["kind"] == "isotonic"
    path.write_text(json.dumps({"calibrator": maps["calibrator"]}))
    cal, prov = load_calibrator(path)
    assert isinstance(cal, IsotonicCalibrator) and prov["kind"] == "isotonic" and prov["store"] is None
    with pytest.raises(ValueError):
        RankedIsotonicCalibrator.from_dict({**maps["rank_calibrator"], "max_rank": 99})
