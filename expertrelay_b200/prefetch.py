"""Which experts to prefetch for the next layer, from a Fate-style guess.

Host-side policy, as predictor/prefetch_policy.py:41-54: layer L+1's router
applied to layer L's input (computed on the GPU by the paged MoE driver)
gives per-expert probabilities; the guess is the top-k experts by
probability (for several tokens, each expert's best probability over them),
and guesses whose calibrated probability of being picked falls below
`min_probability` are dropped. The calibration maps are the reference's
fitted isotonic step functions (predictor/offline.py:87-137 and 150-200),
loaded from their JSON form; fitting them stays offline.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np


def softmax(x: np.ndarray) -> np.ndarray:
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def ranks_desc(probs: np.ndarray) -> np.ndarray:
    """0-based rank along the last axis, highest first, ties in index order."""
    order = np.argsort(-probs, axis=-1, kind="stable")
    ranks = np.empty_like(order)
    np.put_along_axis(ranks, order, np.arange(probs.shape[-1]), axis=-1)
    return ranks


class IsotonicCalibrator:
    """A fitted monotone step map: edges [B-1] ascending, values [B]
    nondecreasing; a score maps to values[number of edges <= score]."""

    def __init__(self, num_bins: int = 1000) -> None:
        self.num_bins = num_bins
        self.edges: np.ndarray | None = None
        self.values: np.ndarray | None = None

    def predict(self, scores: np.ndarray) -> np.ndarray:
        if self.edges is None or self.values is None:
            raise RuntimeError("not fitted")
        return self.values[np.searchsorted(self.edges, scores, side="right")].astype(np.float32)

    def to_dict(self) -> dict:
        if self.edges is None or self.values is None:
            raise RuntimeError("not fitted")
        return {"num_bins": self.num_bins, "edges": self.edges.tolist(), "values": self.values.tolist()}

    @classmethod
    def from_dict(cls, d: dict) -> IsotonicCalibrator:
        cal = cls(d["num_bins"])
        cal.edges = np.asarray(d["edges"], dtype=np.float64)
        cal.values = np.asarray(d["values"], dtype=np.float64)
        if len(cal.values) != len(cal.edges) + 1 or (np.diff(cal.values) < 0).any():
            raise ValueError("not a fitted isotonic map (values one longer than edges, nondecreasing)")
        return cal


class RankedIsotonicCalibrator:
    """One isotonic map per guess rank, ranks >= max_rank sharing the last."""

    def __init__(self, max_rank: int = 12) -> None:
        self.max_rank = max_rank
        self.per_rank: list[IsotonicCalibrator] = []

    def predict(self, probs: np.ndarray) -> np.ndarray:
        if not self.per_rank:
            raise RuntimeError("not fitted")
        probs = np.asarray(probs)
        bucket = np.minimum(ranks_desc(probs), self.max_rank - 1)
        out = np.empty(probs.shape, dtype=np.float32)
        for r, cal in enumerate(self.per_rank):
            m = bucket == r
            if m.any():
                out[m] = cal.predict(probs[m])
        return out

    def to_dict(self) -> dict:
        return {"kind": "rank_isotonic", "max_rank": self.max_rank, "per_rank": [c.to_dict() for c in self.per_rank]}

    @classmethod
    def from_dict(cls, d: dict) -> RankedIsotonicCalibrator:
        cal = cls(d["max_rank"])
        cal.per_rank = [IsotonicCalibrator.from_dict(x) for x in d["per_rank"]]
        if len(cal.per_rank) != cal.max_rank:
            raise ValueError("one isotonic map per rank expected")
        return cal


@dataclass(frozen=True)
class PrefetchChoice:
    experts: list[int]
    skipped_low_confidence: int


@dataclass
class PrefetchPolicy:
    top_k: int
    min_probability: float = 0.0
    calibrator: IsotonicCalibrator | RankedIsotonicCalibrator | None = None

    def choose(self, router_logits: np.ndarray) -> PrefetchChoice:
        """router_logits: [n_tokens, E] (or [E]) for the layer being predicted."""
        probs = softmax(np.atleast_2d(np.asarray(router_logits, dtype=np.float32))).max(axis=0)
        order = np.argsort(-probs, kind="stable")[: self.top_k]
        if self.calibrator is None or self.min_probability <= 0.0:
            return PrefetchChoice([int(e) for e in order], 0)
        keep = self.calibrator.predict(probs[order]) >= self.min_probability
        return PrefetchChoice([int(e) for e in order[keep]], int((~keep).sum()))


def load_calibrator(path: Path, kind: str = "rank") -> tuple[IsotonicCalibrator | RankedIsotonicCalibrator, dict]:
    """From the last record of a calibration results file
    (predictor/prefetch_policy.py:57-78): the rank-aware map when asked for
    and present, else the single map; plus where it came from."""
    if kind not in ("rank", "single"):
        raise ValueError(f"unknown calibration kind {kind!r}")
    records = json.loads(Path(path).read_text(encoding="utf-8"))
    d = records[-1] if isinstance(records, list) else records
    provenance = {
        "file": Path(path).name,
        "git_commit": d.get("git_commit"),
        "timestamp": d.get("timestamp"),
        "store": (d.get("model") or {}).get("store"),
        "kind": "rank_isotonic" if kind == "rank" and "rank_calibrator" in d else "isotonic",
    }
    if kind == "rank" and "rank_calibrator" in d:
        return RankedIsotonicCalibrator.from_dict(d["rank_calibrator"]), provenance
    return IsotonicCalibrator.from_dict(d["calibrator"]), provenance
