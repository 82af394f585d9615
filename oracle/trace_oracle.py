"""CPU oracle for the expert-usage trace. TEST INFRASTRUCTURE ONLY.

Restates in numpy what ExpertRelay's trace writer puts in a trace file
(src/expertrelay/runtime/expert_trace.py): the header (:92-103), one packed
little-endian record per (token, layer) (record_dtype, :34-65), and the
per-layer fill (ExpertTraceWriter.layer, :114-135): router logits and the
Fate prediction stored as float16, the predicted top-k of the previous
layer's Fate logits (largest first), and each token's previous-token
experts at the same layer, carried across calls. The CUDA packer is
compared with this; this is compared with the files the reference itself
wrote (tests/golden/trace.npz, made by tests/golden/make_golden.py).
"""

from __future__ import annotations

import json
import struct

import numpy as np

MAGIC = b"ERTRACE1"
FORMAT_VERSION = 1
NO_EXPERT = 255


def record_dtype(num_experts: int, top_k: int) -> np.dtype:
    """expert_trace.py:34-65, field for field."""
    return np.dtype(
        [
            ("position", "<u4"),
            ("token", "<u4"),
            ("layer", "u1"),
            ("phase", "u1"),
            ("experts", "u1", (top_k,)),
            ("weights", "<f4", (top_k,)),
            ("logits", "<f2", (num_experts,)),
            ("fate_experts", "u1", (top_k,)),
            ("fate_logits", "<f2", (num_experts,)),
            ("prev_token_experts", "u1", (top_k,)),
        ]
    )


def header_bytes(num_layers: int, num_experts: int, top_k: int, metadata: dict) -> bytes:
    """expert_trace.py:92-103: magic, u32 length, UTF-8 JSON."""
    header = {
        "format_version": FORMAT_VERSION,
        "num_layers": num_layers,
        "num_experts": num_experts,
        "top_k": top_k,
        "record_itemsize": record_dtype(num_experts, top_k).itemsize,
        **metadata,
    }
    blob = json.dumps(header, ensure_ascii=False).encode("utf-8")
    return MAGIC + struct.pack("<I", len(blob)) + blob


def top_k_desc(values: np.ndarray, k: int) -> np.ndarray:
    """Largest first; exact ties to the lower index (the reference's
    argpartition order agrees whenever the k largest values are distinct)."""
    order = np.argsort(-values.astype(np.float64), axis=-1, kind="stable")
    return order[:, :k]


class TraceOracle:
    """Writer state and records, as bytes (expert_trace.py:88-135)."""

    def __init__(self, num_layers: int, num_experts: int, top_k: int, metadata: dict):
        self.L, self.E, self.k = num_layers, num_experts, top_k
        self.dtype = record_dtype(num_experts, top_k)
        self.data = bytearray(header_bytes(num_layers, num_experts, top_k, metadata))
        self.prev = np.full((num_layers, top_k), NO_EXPERT, dtype=np.uint8)
        self.pending = None
        self.call = None

    def begin(self, positions, tokens, phase: int) -> None:
        n = len(positions)
        self.call = np.zeros(n * self.L, dtype=self.dtype)
        self.call["position"] = np.repeat(np.asarray(positions), self.L)
        self.call["token"] = np.repeat(np.asarray(tokens), self.L)
        self.call["layer"] = np.tile(np.arange(self.L), n)
        self.call["phase"] = phase
        self.pending = None

    def layer(self, layer: int, logits, selected, weights, fate) -> None:
        rows = self.call[layer :: self.L]
        selected = np.asarray(selected)
        rows["experts"] = selected.astype(np.uint8)
        rows["weights"] = np.asarray(weights, dtype=np.float32)
        with np.errstate(over="ignore"):
            rows["logits"] = np.asarray(logits, dtype=np.float32).astype(np.float16)
            if self.pending is None:
                rows["fate_experts"] = NO_EXPERT
            else:
                rows["fate_logits"] = self.pending.astype(np.float16)
                rows["fate_experts"] = top_k_desc(self.pending, self.k).astype(np.uint8)
        rows["prev_token_experts"] = np.concatenate([self.prev[layer][None], selected[:-1]]).astype(np.uint8)
        self.prev[layer] = selected[-1].astype(np.uint8)
        self.pending = None if fate is None else np.asarray(fate, dtype=np.float32)

    def end(self) -> None:
        self.data += self.call.tobytes()
        self.call = None
