"""Expert-usage traces written from the device (runtime/expert_trace.py).

ExpertTraceWriter has the reference writer's interface and file format
(expert_trace.py:88-135): begin(positions, tokens, phase) per forward call,
layer(layer, logits, selected, weights, next_layer_fate_logits) per layer,
end() appends the call's records to the file. Here the per-layer arguments
are the device tensors the block already produced (router logits, top-k ids
and weights, the next layer's router on this layer's input); er_trace_pack_
layer packs each layer's records on the GPU into one buffer per call, which
end() copies to the host once. read_trace() reads the same files as the
reference's reader, with the same errors for foreign and truncated files.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from . import _lib

MAGIC = b"ERTRACE1"
FORMAT_VERSION = 1
NO_EXPERT = 255  # "no value" for u8 expert-id fields
PHASE_PREFILL, PHASE_DECODE = 0, 1


def record_dtype(num_experts: int, top_k: int) -> np.dtype:
    """One record per (token, layer), packed little-endian (expert_trace.py:34-65)."""
    if num_experts >= NO_EXPERT:
        raise ValueError(f"u8 expert ids hold at most {NO_EXPERT - 1} experts, got {num_experts}")
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


class ExpertTraceWriter:
    """Collects one sequence's records on the device and appends them to the
    trace file after every forward call (begin ... end)."""

    def __init__(self, path, *, num_layers: int, num_experts: int, top_k: int, metadata: dict, device=None):
        self.path = Path(path)
        self.num_layers, self.num_experts, self.top_k = num_layers, num_experts, top_k
        self.dtype = record_dtype(num_experts, top_k)
        itemsize = int(_lib.lib().er_trace_record_bytes(num_experts, top_k))
        if itemsize != self.dtype.itemsize:
            raise ValueError(f"trace records of {num_experts} experts, top-{top_k}: not supported")
        if num_layers > 255:
            raise ValueError(f"u8 layer ids hold at most 255 layers, got {num_layers}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        header = {
            "format_version": FORMAT_VERSION,
            "num_layers": num_layers,
            "num_experts": num_experts,
            "top_k": top_k,
            "record_itemsize": itemsize,
            **metadata,
        }
        blob = json.dumps(header, ensure_ascii=False).encode("utf-8")
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with open(self.path, "wb") as f:
            f.write(MAGIC + struct.pack("<I", len(blob)) + blob)
        # previous-token experts, [side][layer][k] on the device: a layer's
        # packer reads its side and writes the other (its first token reads
        # the old state while its last writes the new one)
        self._prev = torch.full((2, num_layers, top_k), NO_EXPERT, dtype=torch.uint8, device=self.device)
        self._prev_side = [0] * num_layers
        self._pending_fate: torch.Tensor | None = None
        self._records: torch.Tensor | None = None
        self._n = 0

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def begin(self, positions, tokens, phase: int) -> None:
        positions = np.asarray(positions).astype(np.int64)
        tokens = np.asarray(tokens).astype(np.int64)
        self._n = n = len(positions)
        if len(tokens) != n:
            raise ValueError(f"{n} positions but {len(tokens)} tokens")
        # the reference stores both as little-endian u32 (numpy's wrapping cast)
        self._positions = torch.from_numpy(positions.astype(np.uint32).view(np.int32)).to(self.device)
        self._tokens = torch.from_numpy(tokens.astype(np.uint32).view(np.int32)).to(self.device)
        self._phase = int(phase)
        self._records = torch.zeros(n * self.num_layers * self.dtype.itemsize, dtype=torch.uint8, device=self.device)
        self._pending_fate = None

    def layer(self, layer: int, logits, selected, weights, next_layer_fate_logits) -> None:
        """Device tensors over this call's tokens: logits [n, E] f32, selected
        [n, k] int64 or int32, weights [n, k] f32; next_layer_fate_logits
        [n, E] f32 (layer + 1's router on this layer's input) or None."""
        if self._records is None:
            raise RuntimeError("ExpertTraceWriter.layer() outside begin() ... end()")
        n, E, k = self._n, self.num_experts, self.top_k
        logits = _dev(logits, torch.float32, (n, E), self.device)
        weights = _dev(weights, torch.float32, (n, k), self.device)
        sel = selected if isinstance(selected, torch.Tensor) else torch.from_numpy(np.asarray(selected))
        if sel.dtype not in (torch.int64, torch.int32):
            sel = sel.to(torch.int64)
        sel = _dev(sel, sel.dtype, (n, k), self.device)
        fate = self._pending_fate
        side = self._prev_side[layer]
        prev_in = self._prev[side]  # [num_layers, k], rows of other layers untouched
        prev_out = self._prev[side ^ 1]
        if n == 0:
            return
        rc = _lib.lib().er_trace_pack_layer(
            self._records.data_ptr(), n, self.num_layers, layer, self._positions.data_ptr(),
            self._tokens.data_ptr(), self._phase, logits.data_ptr(), sel.data_ptr(),
            1 if sel.dtype == torch.int64 else 0, weights.data_ptr(), fate.data_ptr() if fate is not None else None,
            prev_in.data_ptr(), prev_out.data_ptr(), E, k, self._stream())
        _lib.check(rc, "er_trace_pack_layer")
        self._prev_side[layer] = side ^ 1  # this layer's state now lives in the other buffer
        self._keep = (logits, weights, sel)  # alive until the packer has read them
        self._pending_fate = (None if next_layer_fate_logits is None
                              else _dev(next_layer_fate_logits, torch.float32, (n, E), self.device))

    def end(self) -> None:
        if self._records is None:
            raise RuntimeError("ExpertTraceWriter.end() without begin()")
        data = self._records.cpu().numpy().tobytes()
        with open(self.path, "ab") as f:
            f.write(data)
        self._records = None
        self._keep = None
        self._pending_fate = None


def _dev(x, dtype, shape, device) -> torch.Tensor:
    t = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x))
    t = t.to(device=device, dtype=dtype).contiguous()
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"expected shape {tuple(shape)}, got {tuple(t.shape)}")
    return t


def read_trace(path) -> tuple[dict, np.ndarray]:
    """(header, records). Raises ValueError for a file that is not a trace
    or is truncated mid-record (expert_trace.py:138-152)."""
    data = Path(path).read_bytes()
    if data[:8] != MAGIC:
        raise ValueError(f"{path}: not an expert trace (bad magic)")
    (hlen,) = struct.unpack("<I", data[8:12])
    header = json.loads(data[12 : 12 + hlen].decode("utf-8"))
    if header["format_version"] != FORMAT_VERSION:
        raise ValueError(f"{path}: unsupported trace format_version {header['format_version']}")
    dtype = record_dtype(header["num_experts"], header["top_k"])
    body = data[12 + hlen :]
    if len(body) % dtype.itemsize:
        raise ValueError(f"{path}: truncated ({len(body)} bytes is not a whole number of records)")
    return header, np.frombuffer(body, dtype=dtype)
