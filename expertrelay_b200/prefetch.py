"""Prefetch choice for the next MoE layer from the cross-layer router guess.

The paged MoE driver runs layer L+1's router on layer L's input on the GPU
(the Fate guess of predictor/prefetch_policy.py, used at
runtime/qwen_moe.py:314-320) and hands the resulting logits to
`PrefetchPolicy.choose`. The rule it applies is the reference's
(predictor/prefetch_policy.py:41-54):

  * every expert is scored by its best softmax probability over the call's
    tokens;
  * the `top_k` best-scored experts are the guess, best first, equal scores
    in ascending expert id;
  * with a calibration map and `min_probability` > 0, guesses whose
    calibrated chance of being picked is below `min_probability` are
    dropped and counted.

Calibration maps are monotone step functions fitted offline (isotonic
regression, predictor/offline.py:87-200); only their evaluation and their
JSON form live here, so maps fitted by the reference's tools load
unchanged:
  single map : {"num_bins": B, "edges": [...], "values": [...]}
  per rank   : {"kind": "rank_isotonic", "max_rank": R, "per_rank": [map, ...]}
A results file (a JSON list of records, or one record) holds them under
"calibrator" and "rank_calibrator"; `load_calibrator` reads the last record.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

__all__ = [
    "IsotonicCalibrator",
    "RankedIsotonicCalibrator",
    "PrefetchChoice",
    "PrefetchPolicy",
    "expert_scores",
    "guess_order",
    "rank_positions",
    "load_calibrator",
]


def expert_scores(router_logits: np.ndarray) -> np.ndarray:
    """Each expert's highest softmax probability over the tokens.

    router_logits: [E] or [tokens, E]. Probabilities are formed in float32
    from the log-sum-exp of each token's row, as the runtime's softmax does
    (runtime/qwen_moe.py:157-159)."""
    z = np.asarray(router_logits, dtype=np.float32)
    if z.ndim == 1:
        z = z[None, :]
    if z.ndim != 2 or z.shape[1] == 0:
        raise ValueError(f"router logits must be [E] or [tokens, E], got shape {np.shape(router_logits)}")
    shifted = z - z.max(axis=1, keepdims=True)
    p = np.exp(shifted)
    p /= p.sum(axis=1, keepdims=True)
    return p.max(axis=0)


def guess_order(scores: np.ndarray) -> np.ndarray:
    """Expert ids by descending score; equal scores keep ascending id."""
    s = np.asarray(scores)
    ids = np.arange(s.shape[-1])
    return np.lexsort((ids, -s))


def rank_positions(scores: np.ndarray) -> np.ndarray:
    """0-based position of every entry in its row's descending order (equal
    scores ordered by index), along the last axis."""
    s = np.asarray(scores)
    order = np.argsort(-s, axis=-1, kind="stable")
    return np.argsort(order, axis=-1, kind="stable")


class IsotonicCalibrator:
    """Evaluates a fitted monotone step map.

    `edges` ([B-1], ascending) split the score axis into B intervals and
    `values` ([B], nondecreasing) is the calibrated probability on each; a
    score equal to an edge falls in the interval above it."""

    def __init__(self, num_bins: int = 1000) -> None:
        self.num_bins = num_bins
        self.edges: np.ndarray | None = None
        self.values: np.ndarray | None = None

    def _require_fitted(self) -> tuple[np.ndarray, np.ndarray]:
        if self.edges is None or self.values is None:
            raise RuntimeError("calibration map has no fitted steps")
        return self.edges, self.values

    def predict(self, scores: np.ndarray) -> np.ndarray:
        edges, values = self._require_fitted()
        interval = np.digitize(np.asarray(scores, dtype=np.float64), edges, right=False)
        return values[interval].astype(np.float32)

    def to_dict(self) -> dict:
        edges, values = self._require_fitted()
        return {"num_bins": int(self.num_bins), "edges": [float(e) for e in edges], "values": [float(v) for v in values]}

    @classmethod
    def from_dict(cls, d: dict) -> "IsotonicCalibrator":
        edges = np.asarray(d["edges"], dtype=np.float64).reshape(-1)
        values = np.asarray(d["values"], dtype=np.float64).reshape(-1)
        if values.size != edges.size + 1:
            raise ValueError(f"calibration map: {values.size} values for {edges.size} edges (need one more value)")
        if values.size > 1 and np.any(values[1:] < values[:-1]):
            raise ValueError("calibration map: values must be nondecreasing")
        cal = cls(int(d["num_bins"]))
        cal.edges, cal.values = edges, values
        return cal


class RankedIsotonicCalibrator:
    """A separate step map for each guess rank (0 = the best-scored
    candidate); ranks at or beyond `max_rank` use the last map."""

    def __init__(self, max_rank: int = 12, num_bins: int = 200) -> None:
        self.max_rank = max_rank
        self.num_bins = num_bins
        self.per_rank: list[IsotonicCalibrator] = []

    def predict(self, probs: np.ndarray) -> np.ndarray:
        """probs: [..., candidates]; each row's candidates are ranked among
        themselves."""
        if not self.per_rank:
            raise RuntimeError("calibration map has no fitted steps")
        p = np.asarray(probs)
        bucket = np.minimum(rank_positions(p), len(self.per_rank) - 1)
        by_map = np.stack([m.predict(p) for m in self.per_rank])  # [maps, ...]
        return np.take_along_axis(by_map, bucket[None, ...], axis=0)[0]

    def to_dict(self) -> dict:
        return {"kind": "rank_isotonic", "max_rank": int(self.max_rank), "per_rank": [m.to_dict() for m in self.per_rank]}

    @classmethod
    def from_dict(cls, d: dict) -> "RankedIsotonicCalibrator":
        maps = [IsotonicCalibrator.from_dict(x) for x in d["per_rank"]]
        if len(maps) != int(d["max_rank"]):
            raise ValueError(f"rank calibration: {len(maps)} maps for max_rank {d['max_rank']}")
        cal = cls(int(d["max_rank"]))
        cal.per_rank = maps
        return cal


@dataclass(frozen=True)
class PrefetchChoice:
    """Experts to prefetch (best first) and how many guesses the calibrated
    cut dropped."""

    experts: list[int]
    skipped_low_confidence: int


@dataclass
class PrefetchPolicy:
    """top_k guesses per call, cut at `min_probability` of the calibration
    map when both are given."""

    top_k: int
    min_probability: float = 0.0
    calibrator: IsotonicCalibrator | RankedIsotonicCalibrator | None = field(default=None)

    def choose(self, router_logits: np.ndarray) -> PrefetchChoice:
        """router_logits: the predicted layer's router logits for this call's
        tokens, [tokens, E] or [E]."""
        scores = expert_scores(router_logits)
        guess = guess_order(scores)[: max(int(self.top_k), 0)]
        if self.calibrator is None or not self.min_probability > 0.0:
            return PrefetchChoice(guess.tolist(), 0)
        passed = self.calibrator.predict(scores[guess]) >= self.min_probability
        return PrefetchChoice(guess[passed].tolist(), int(passed.size - np.count_nonzero(passed)))


def load_calibrator(path: Path, kind: str = "rank") -> tuple[IsotonicCalibrator | RankedIsotonicCalibrator, dict]:
    """The calibration map of the last record in a fitted-calibration results
    file, and a provenance dict (file, git_commit, timestamp, store, kind).

    kind "rank" takes the per-rank map when the record has one and the
    single map otherwise; "single" always takes the single map."""
    if kind not in ("rank", "single"):
        raise ValueError(f"unknown calibration kind {kind!r} (expected 'rank' or 'single')")
    data = json.loads(Path(path).read_text(encoding="utf-8"))
    record = data[-1] if isinstance(data, list) else data
    ranked = kind == "rank" and "rank_calibrator" in record
    cal = RankedIsotonicCalibrator.from_dict(record["rank_calibrator"]) if ranked else IsotonicCalibrator.from_dict(
        record["calibrator"]
    )
    model = record.get("model") or {}
    provenance = {
        "file": Path(path).name,
        "git_commit": record.get("git_commit"),
        "timestamp": record.get("timestamp"),
        "store": model.get("store"),
        "kind": "rank_isotonic" if ranked else "isotonic",
    }
    return cal, provenance
