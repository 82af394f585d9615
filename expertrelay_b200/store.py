"""Expert record layouts of the expert store (host side).

One routed expert = one fixed-size record, padded to a multiple of 4096
bytes, matrices in the order gate [I, H], up [I, H], down [H, I]:

  int8 (store/layout.py:13-26, 53-115)
      [gate q int8][up q][down q][gate s f32 [I]][up s][down s][zero pad]
  int4 (store/int4.py:65-67, 165-244)
      [gate packed u8 [I, H/2]][up][down][gate s f16 [I, H/G]][up s][down s][zero pad]
  int4 with zero points (this package's extension for asymmetric GPTQ)
      the int4 record followed, before the padding, by
      [gate z u8 [I, H/G]][up z][down z], value = nibble - z

The HBM expert cache holds exactly these bytes, one record per slot, and the
CUDA kernels read weights, scales and zero points straight from them; the
offsets here are the ones the kernels compute (er_record_offset). Records of
layer L, expert e sit at (L * E + e) * record_size in experts.bin
(store/layout.py:148-153).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

ALIGNMENT = 4096  # store/unbuffered_io.py ALIGNMENT
MATRICES = ("gate_proj", "up_proj", "down_proj")
INT4_FORMAT = "int4_groupwise_symmetric_rtn"  # the reference's layout["format"] id for int4 stores
INT4_ZP_FORMAT = "int4_groupwise_asymmetric_zp"

FMT_INT8, FMT_INT4, FMT_INT4_ZP = 0, 1, 2


def align_up(n: int, a: int = ALIGNMENT) -> int:
    return (n + a - 1) // a * a


@dataclass(frozen=True)
class RecordLayout:
    """Byte layout of one expert record (fmt: FMT_INT8 / FMT_INT4 / FMT_INT4_ZP)."""

    fmt: int
    hidden: int
    inter: int
    group: int = 0
    quantizer: str = "rtn_absmax7"

    def __post_init__(self):
        if self.fmt not in (FMT_INT8, FMT_INT4, FMT_INT4_ZP):
            raise ValueError(f"unknown record format {self.fmt}")
        if self.fmt != FMT_INT8 and (
            self.group <= 0 or self.group % 2 or self.hidden % self.group or self.inter % self.group
        ):
            raise ValueError(f"group size {self.group} doesn't split {self.hidden} and {self.inter} into even groups")

    @classmethod
    def from_config(cls, config: dict, fmt: int = FMT_INT8, group: int = 0, quantizer: str = "rtn_absmax7"):
        return cls(fmt, config["hidden_size"], config["moe_intermediate_size"], group, quantizer)

    def shape(self, name: str) -> tuple[int, int]:
        return (self.hidden, self.inter) if name == "down_proj" else (self.inter, self.hidden)

    @property
    def matrices(self) -> tuple[tuple[str, tuple[int, int]], ...]:
        return tuple((m, self.shape(m)) for m in MATRICES)

    def _weight_bytes(self, name: str) -> int:
        r, c = self.shape(name)
        return r * c if self.fmt == FMT_INT8 else r * c // 2

    def _scale_bytes(self, name: str) -> int:
        r, c = self.shape(name)
        return r * 4 if self.fmt == FMT_INT8 else r * (c // self.group) * 2

    def _zero_bytes(self, name: str) -> int:
        r, c = self.shape(name)
        return r * (c // self.group) if self.fmt == FMT_INT4_ZP else 0

    def weight_offset(self, name: str) -> int:
        return sum(self._weight_bytes(m) for m in MATRICES[: MATRICES.index(name)])

    def scale_offset(self, name: str) -> int:
        return self.weights_bytes + sum(self._scale_bytes(m) for m in MATRICES[: MATRICES.index(name)])

    def zero_offset(self, name: str) -> int:
        if self.fmt != FMT_INT4_ZP:
            raise KeyError(f"{name}: this layout has no zero points")
        return self.weights_bytes + self.scales_bytes + sum(self._zero_bytes(m) for m in MATRICES[: MATRICES.index(name)])

    @property
    def weights_bytes(self) -> int:
        return sum(self._weight_bytes(m) for m in MATRICES)

    @property
    def scales_bytes(self) -> int:
        return sum(self._scale_bytes(m) for m in MATRICES)

    @property
    def zeros_bytes(self) -> int:
        return sum(self._zero_bytes(m) for m in MATRICES)

    @property
    def record_size(self) -> int:
        return align_up(self.weights_bytes + self.scales_bytes + self.zeros_bytes)

    def to_dict(self) -> dict:
        """The manifest entry, with the reference's keys for the int8 and int4 layouts."""
        d = {
            "matrices": [{"name": m, "shape": list(s)} for m, s in self.matrices],
            "weights_bytes": self.weights_bytes,
            "scales_bytes": self.scales_bytes,
            "scales_dtype": "float32" if self.fmt == FMT_INT8 else "float16",
            "record_size": self.record_size,
            "alignment": ALIGNMENT,
        }
        if self.fmt != FMT_INT8:
            d = {
                "format": INT4_FORMAT if self.fmt == FMT_INT4 else INT4_ZP_FORMAT,
                "quantizer": self.quantizer,
                "group_size": self.group,
                **d,
            }
        if self.fmt == FMT_INT4_ZP:
            d["zeros_bytes"] = self.zeros_bytes
        return d

    @classmethod
    def from_dict(cls, d: dict) -> RecordLayout:
        shapes = {m["name"]: tuple(m["shape"]) for m in d["matrices"]}
        inter, hidden = shapes["gate_proj"]
        if shapes.get("down_proj") != (hidden, inter) or shapes.get("up_proj") != (inter, hidden):
            raise ValueError(f"unexpected matrix shapes {shapes}")
        fmt_id = d.get("format")
        if fmt_id is None:
            return cls(FMT_INT8, hidden, inter)
        if fmt_id == INT4_FORMAT:
            return cls(FMT_INT4, hidden, inter, d["group_size"], d.get("quantizer", "rtn_absmax7"))
        if fmt_id == INT4_ZP_FORMAT:
            return cls(FMT_INT4_ZP, hidden, inter, d["group_size"], d.get("quantizer", "gptq_asym_rtn"))
        raise ValueError(f"not an expert layout: {fmt_id!r}")


def serialize_record(layout: RecordLayout, mats: dict[str, tuple]) -> np.ndarray:
    """{matrix: (weights, scales[, zeros])} -> one padded record (uint8 array).
    int8: (int8 [r, c], float32 [r]); int4: (uint8 [r, c/2], float16 [r, c/G])
    plus uint8 zeros [r, c/G] for FMT_INT4_ZP."""
    rec = np.zeros(layout.record_size, dtype=np.uint8)
    for name, (r, c) in layout.matrices:
        parts = mats[name]
        w, s = np.asarray(parts[0]), np.asarray(parts[1])
        if layout.fmt == FMT_INT8:
            if w.shape != (r, c) or w.dtype != np.int8 or s.shape != (r,):
                raise ValueError(f"{name}: got {w.dtype}{w.shape} / scales{s.shape}, expected int8{(r, c)}")
            s = s.astype("<f4")
        else:
            if w.shape != (r, c // 2) or w.dtype != np.uint8:
                raise ValueError(f"{name}: packed {w.dtype}{w.shape}, expected uint8{(r, c // 2)}")
            if s.shape != (r, c // layout.group):
                raise ValueError(f"{name}: scales {s.shape}, expected {(r, c // layout.group)}")
            s = s.astype("<f2")
        off = layout.weight_offset(name)
        rec[off : off + w.nbytes] = np.ascontiguousarray(w).view(np.uint8).reshape(-1)
        off = layout.scale_offset(name)
        rec[off : off + s.nbytes] = np.ascontiguousarray(s).view(np.uint8).reshape(-1)
        if layout.fmt == FMT_INT4_ZP:
            z = np.asarray(parts[2])
            if z.shape != (r, c // layout.group) or z.dtype != np.uint8:
                raise ValueError(f"{name}: zeros {z.dtype}{z.shape}, expected uint8{(r, c // layout.group)}")
            off = layout.zero_offset(name)
            rec[off : off + z.nbytes] = z.reshape(-1)
    return rec


def parse_record(layout: RecordLayout, buf) -> dict[str, tuple]:
    """Inverse of serialize_record, as views into `buf`."""
    b = np.frombuffer(buf, dtype=np.uint8) if not isinstance(buf, np.ndarray) else buf.view(np.uint8).reshape(-1)
    out = {}
    for name, (r, c) in layout.matrices:
        wo, so = layout.weight_offset(name), layout.scale_offset(name)
        if layout.fmt == FMT_INT8:
            w = b[wo : wo + r * c].view(np.int8).reshape(r, c)
            s = b[so : so + 4 * r].view("<f4")
            out[name] = (w, s)
        else:
            g = c // layout.group
            w = b[wo : wo + r * c // 2].reshape(r, c // 2)
            s = b[so : so + 2 * r * g].view("<f2").reshape(r, g)
            if layout.fmt == FMT_INT4_ZP:
                zo = layout.zero_offset(name)
                out[name] = (w, s, b[zo : zo + r * g].reshape(r, g))
            else:
                out[name] = (w, s)
    return out


def expert_offset(layer: int, expert: int, num_experts: int, record_size: int) -> int:
    """Byte offset of (layer, expert) in experts.bin (store/layout.py:148-153)."""
    return (layer * num_experts + expert) * record_size
