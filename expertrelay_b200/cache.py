"""HbmExpertCache: routed-expert records of many layers served from HBM slots.

The B200 counterpart of CachedExpertSource (cache/expert_cache.py:92-402),
over the library's er_cache_* functions (include/expertrelay_b200.h). The
budget buys whole slots of one store record each; a (layer, expert) record
comes from pinned host memory (HostRecords, standing in for the SSD store)
by an asynchronous copy on the cache's copy stream; eviction is LRU over the
ready slots no layer holds; pinned experts stay; prefetches are skipped when
nothing is evictable or over the read budget; the counters are SourceStats'
(runtime/weights.py:170-193).

What differs from the reference, because the copies run on the GPU's copy
engines instead of I/O threads:
  * nothing blocks the host: acquire() makes the caller's stream wait for the
    records' copies (an in-flight prefetch is waited for, not repeated);
  * a forward pass holds every expert it acquired for a layer until
    end_layer(layer) (the reference holds one at a time), and end_layer
    records when the stream is done with them, which a later refill of the
    slot waits for;
  * a copy once issued is not withdrawn: prefetches_cancelled stays 0, and
    read_seconds stays 0.0 (the host never waits for a record).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields

import numpy as np
import torch

from . import _lib
from .store import FMT_INT4_ZP, FMT_INT8, RecordLayout

Key = tuple[int, int]  # (layer, expert)


class CacheTooSmall(RuntimeError):
    """No slot could be freed (cache/expert_cache.py:60-61)."""


@dataclass
class SourceStats:
    """Cumulative counters, named as runtime/weights.py:170-193."""

    loads: int = 0
    bytes_read: int = 0
    read_seconds: float = 0.0
    demand_reads: int = 0
    cache_hits: int = 0
    prefetch_hits: int = 0
    prefetch_waits: int = 0
    prefetches_issued: int = 0
    prefetch_reads: int = 0
    prefetch_bytes: int = 0
    prefetches_wasted: int = 0
    prefetches_cancelled: int = 0
    prefetches_skipped_full: int = 0
    prefetches_skipped_budget: int = 0


@dataclass
class DeviceInt8Matrix:
    """An int8 expert matrix as device views into its cache slot (the fields of
    runtime/weights.py Int8Matrix)."""

    q: torch.Tensor  # [out, in] int8
    scales: torch.Tensor  # [out] float32


@dataclass
class DeviceInt4Matrix:
    """An int4 expert matrix as device views into its cache slot (the fields
    of runtime/weights.py Int4Matrix: two codes per byte, the even column in
    the low nibble, float16 scales per group of `group_size` inputs), plus
    the 4-bit zero points of an asymmetric GPTQ record (None for the
    store's symmetric records, whose zero point is 8)."""

    packed: torch.Tensor  # [out, in / 2] uint8
    scales: torch.Tensor  # [out, in / group_size] float16
    group_size: int
    zeros: torch.Tensor | None = None  # [out, in / group_size] uint8


def record_views(layout: RecordLayout, rec: torch.Tensor) -> dict:
    """The matrices of one store record held in the uint8 tensor `rec` (on
    any device), as views: DeviceInt8Matrix or DeviceInt4Matrix per matrix
    name, at the record layout's offsets (store/layout.py:53-115,
    store/int4.py:165-244)."""
    out = {}
    for name, (rows, cols) in layout.matrices:
        w0, s0 = layout.weight_offset(name), layout.scale_offset(name)
        if layout.fmt == FMT_INT8:
            q = rec[w0 : w0 + rows * cols].view(torch.int8).view(rows, cols)
            s = rec[s0 : s0 + rows * 4].view(torch.float32)
            out[name] = DeviceInt8Matrix(q, s)
            continue
        groups = cols // layout.group
        packed = rec[w0 : w0 + rows * cols // 2].view(rows, cols // 2)
        scales = rec[s0 : s0 + rows * groups * 2].view(torch.float16).view(rows, groups)
        zeros = None
        if layout.fmt == FMT_INT4_ZP:
            z0 = layout.zero_offset(name)
            zeros = rec[z0 : z0 + rows * groups].view(rows, groups)
        out[name] = DeviceInt4Matrix(packed, scales, layout.group, zeros)
    return out


def slots_for(capacity_bytes: int, record_size: int) -> int:
    """Whole slots a budget buys (cache/expert_cache.py:86-87)."""
    return int(capacity_bytes) // int(record_size)


class HostRecords:
    """Every (layer, expert) record of a model in host memory, page-locked so
    that copies to the GPU run asynchronously: records[layer, expert] is one
    store record (store/layout.py:53-145)."""

    def __init__(self, records: np.ndarray | torch.Tensor, layout: RecordLayout, *, pin: bool = True):
        t = torch.as_tensor(records)
        if t.dtype != torch.uint8 or t.dim() != 3 or t.shape[2] != layout.record_size:
            raise ValueError(f"records: expected [layers, experts, {layout.record_size}] uint8, got "
                             f"{tuple(t.shape)} {t.dtype}")
        t = t.contiguous()
        if pin and torch.cuda.is_available() and not t.is_pinned():
            t = t.pin_memory()
        self.tensor = t
        self.layout = layout
        self.layers, self.experts = int(t.shape[0]), int(t.shape[1])

    @classmethod
    def from_blocks(cls, blocks, *, pin: bool = True) -> HostRecords:
        """From expertrelay_b200.synth.HostBlock objects, one per layer."""
        return cls(np.stack([b.records() for b in blocks]), blocks[0].layout, pin=pin)

    def addresses(self) -> list[int]:
        base, rs = self.tensor.data_ptr(), self.layout.record_size
        return [base + i * rs for i in range(self.layers * self.experts)]

    def record(self, layer: int, expert: int) -> torch.Tensor:
        return self.tensor[layer, expert]


class HbmExpertCache:
    """Routed-expert records in HBM slots (see the module docstring).

    capacity_bytes buys slots_for(capacity_bytes, record_size) slots; fewer
    than len(pinned) + min_free_slots raises CacheTooSmall, like the reference
    (expert_cache.py:104-113). dry=True keeps only the bookkeeping (no device
    memory or copies, fills complete at once), for host-side use and tests.
    """

    def __init__(
        self,
        source: HostRecords,
        *,
        capacity_bytes: int,
        pinned: list[Key] | tuple = (),
        min_free_slots: int = 1,
        device: str | torch.device | None = None,
        dry: bool = False,
    ):
        self.source = source
        self.layout = source.layout
        rs = self.layout.record_size
        n = slots_for(capacity_bytes, rs)
        if n < len(pinned) + min_free_slots:
            raise CacheTooSmall(
                f"{capacity_bytes / 1e9:.2f} GB holds {n} experts; need {len(pinned)} pinned + {min_free_slots} free"
            )
        self.dry = dry
        self.min_free_slots = int(min_free_slots)
        self.device = None
        if not dry:
            self.device = torch.device(device if device is not None else "cuda")
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
        self.arena = None if dry else torch.empty(n * rs, dtype=torch.uint8, device=self.device)
        handle = C.c_void_p()
        flags = _lib.CACHE_DRY if dry else 0
        arena_ptr = None if dry else self.arena.data_ptr()
        self._check(_lib.lib().er_cache_create(n, rs, self.min_free_slots, arena_ptr, flags, C.byref(handle)),
                    "er_cache_create")
        self._h = handle
        addrs = source.addresses()
        arr = (C.c_void_p * len(addrs))(*addrs)
        self._check(_lib.lib().er_cache_set_source(self._h, source.layers, source.experts, arr), "er_cache_set_source")
        for layer, expert in pinned:
            self._check(_lib.lib().er_cache_pin(self._h, int(layer), int(expert)), "er_cache_pin")

    # ------------------------------------------------------------- internals

    @staticmethod
    def _check(rc: int, what: str) -> None:
        if rc == _lib.ER_ENOSPACE:
            raise CacheTooSmall(f"{what}: {_lib.last_error()}")
        _lib.check(rc, what)

    def _stream(self, stream) -> int | None:
        if self.dry:
            return None
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return s.cuda_stream

    # ---------------------------------------------------------------- queries

    @property
    def num_slots(self) -> int:
        slots = C.c_int()
        self._check(_lib.lib().er_cache_info(self._h, None, C.byref(slots), None, None), "er_cache_info")
        return slots.value

    @property
    def capacity_bytes(self) -> int:
        return self.num_slots * self.layout.record_size

    @property
    def supports_prefetch(self) -> bool:
        return True

    @property
    def arena_base(self) -> int:
        return 0 if self.arena is None else self.arena.data_ptr()

    @property
    def copy_stream(self) -> torch.cuda.ExternalStream | None:
        """The stream the record copies run on."""
        if self.dry:
            return None
        s = C.c_void_p()
        self._check(_lib.lib().er_cache_info(self._h, None, None, None, C.byref(s)), "er_cache_info")
        return torch.cuda.ExternalStream(s.value, device=self.device)

    @property
    def stats(self) -> SourceStats:
        cs = _lib.CacheStats()
        self._check(_lib.lib().er_cache_stats_get(self._h, C.byref(cs)), "er_cache_stats_get")
        out = SourceStats()
        for f in fields(SourceStats):
            if f.name != "read_seconds":
                setattr(out, f.name, int(getattr(cs, f.name)))
        return out

    def lookup(self, layer: int, expert: int) -> tuple[int, int]:
        """(slot, state) of a key; slot -1 when absent. States: _lib.SLOT_*."""
        slot, state = C.c_int(), C.c_int()
        self._check(_lib.lib().er_cache_lookup(self._h, int(layer), int(expert), C.byref(slot), C.byref(state)),
                    "er_cache_lookup")
        return slot.value, state.value

    def cached_keys(self) -> set[Key]:
        """Keys whose record is resident or on its way."""
        return {
            (layer, e)
            for layer in range(self.source.layers)
            for e in range(self.source.experts)
            if self.lookup(layer, e)[0] >= 0
        }

    # ----------------------------------------------------------- the forward

    def acquire(self, layer: int, experts, stream=None) -> np.ndarray:
        """Make `experts` of `layer` resident for the forward pass: returns
        each record's device address (uint64). `stream` (default: the current
        one) waits for their copies; the slots stay held until end_layer."""
        ex = np.ascontiguousarray(experts, dtype=np.int32).reshape(-1)
        out = np.zeros(ex.size, dtype=np.uint64)
        self._check(
            _lib.lib().er_cache_acquire(self._h, int(layer), ex.ctypes.data_as(C.POINTER(C.c_int)), ex.size,
                                        self._stream(stream), out.ctypes.data_as(C.POINTER(C.c_uint64))),
            "er_cache_acquire",
        )
        return out

    def load(self, layer: int, expert: int, stream=None) -> dict:
        """ExpertSource.load (runtime/weights.py:199-207): the expert's
        matrices as device views into its slot (DeviceInt8Matrix, or
        DeviceInt4Matrix for int4 records), held until end_layer."""
        if self.dry:
            raise RuntimeError("a dry cache holds no records")
        addr = int(self.acquire(layer, [expert], stream)[0])
        off = addr - self.arena.data_ptr()
        return record_views(self.layout, self.arena[off : off + self.layout.record_size])

    def prefetch(self, layer: int, experts, keep=(), max_new_reads: int | None = None) -> None:
        """Start copying `experts` of `layer` (cache/expert_cache.py:264-294)."""
        ex = np.ascontiguousarray(experts, dtype=np.int32).reshape(-1)
        kp = np.ascontiguousarray(list(keep), dtype=np.int32).reshape(-1)
        self._check(
            _lib.lib().er_cache_prefetch(
                self._h, int(layer), ex.ctypes.data_as(C.POINTER(C.c_int)), ex.size,
                kp.ctypes.data_as(C.POINTER(C.c_int)), kp.size // 2,
                -1 if max_new_reads is None else int(max_new_reads),
            ),
            "er_cache_prefetch",
        )

    def end_layer(self, layer: int, stream=None) -> None:
        """The forward pass is done with `layer` (cache/expert_cache.py:296-305)."""
        self._check(_lib.lib().er_cache_end_layer(self._h, int(layer), self._stream(stream)), "er_cache_end_layer")

    def resize(self, capacity_bytes: int) -> int:
        """New budget, whole slots (cache/expert_cache.py:307-354); returns the
        slot count. Records move to a new arena (arena_base changes)."""
        rs = self.layout.record_size
        n = slots_for(capacity_bytes, rs)
        new = None if self.dry else torch.empty(max(n, 1) * rs, dtype=torch.uint8, device=self.device)
        out = C.c_int()
        self._check(_lib.lib().er_cache_resize(self._h, n, None if new is None else new.data_ptr(), C.byref(out)),
                    "er_cache_resize")
        if new is not None:
            self.arena = new  # the old arena's records were copied before the call returned
        return out.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().er_cache_destroy(self._h)
            self._h = None

    def __enter__(self) -> HbmExpertCache:
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
