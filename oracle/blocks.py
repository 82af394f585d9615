"""Oracle views of synthetic blocks. TEST INFRASTRUCTURE ONLY (used by tests/
and by bench.py's CPU-baseline legs).

Turns an expertrelay_b200.synth.HostBlock (duck-typed: router, shared_gate,
shared, experts, fmt, group, top_k, gptq) into the oracle's BlockWeights
over the same arrays.
"""

from __future__ import annotations

import numpy as np

from . import moe_oracle as O


def oracle_weights(block) -> O.BlockWeights:
    """Experts in their record encodings (int8 / int4 / int4 with zero points)."""
    experts = []
    for mats in block.experts:
        if block.fmt == "int8":
            experts.append({m: O.Int8Mat(*t) for m, t in mats.items()})
        elif block.fmt == "int4":
            experts.append({m: O.Int4Mat(t[0], t[1], block.group) for m, t in mats.items()})
        else:
            experts.append({m: O.Int4Mat(t[0], t[1], block.group, t[2]) for m, t in mats.items()})
    shared = {m: O.Int8Mat(*t) for m, t in block.shared.items()}
    return O.BlockWeights(block.router, block.shared_gate, shared, experts, top_k=block.top_k)


class _F32Mat(O.Int8Mat):
    """A float32 weight matrix held as an int8-shaped matrix with unit scales (exact)."""

    def __init__(self, w: np.ndarray):
        super().__init__(w.astype(np.float32), np.ones(w.shape[0], dtype=np.float32))


def gptq_oracle_weights(block) -> O.BlockWeights:
    """For GPTQ blocks: experts dequantized straight from the GPTQ v1 tensors
    (qweight / qzeros / scales / g_idx) by the reference formula
    (bench/gptq_conversion_check.py:42-55), never from the record encoding."""
    experts = []
    for gt in block.gptq:
        experts.append(
            {m: _F32Mat(O.gptq_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"])) for m, t in gt.items()}
        )
    shared = {m: O.Int8Mat(*t) for m, t in block.shared.items()}
    return O.BlockWeights(block.router, block.shared_gate, shared, experts, top_k=block.top_k)
