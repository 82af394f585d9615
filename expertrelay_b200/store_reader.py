"""The expert store on disk -> host memory (store/expert_reader.py, store/
layout.py:148-211, store/unbuffered_io.py).

A store directory holds experts.bin (one record per routed expert, layer L
expert e at (L * E + e) * record_size) and experts_index.json (the record
layout and one entry per expert: offset, size, shapes, sha256). Reading an
expert is one read of the whole record, bypassing the page cache, into a
4096-aligned buffer (er_store_read; O_DIRECT on Linux, where the reference
has Win32 unbuffered reads), normally pinned host memory that the HBM
expert cache copies from.

read_expert_index validates the index as strictly as the reference
(format version, every offset 4096-aligned, every size the record size, no
duplicate expert). ExpertStoreReader mirrors the reference's reader
(read_raw, read_into, read, verify, entry, entries); load_host_records reads
every expert of the store into one pinned [layers, experts, record_size]
buffer with several reads in flight, as the cache's HostRecords source.
write_expert_store writes a store in the same format (tests, converters).
"""

from __future__ import annotations

import ctypes as C
import hashlib
import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np

from . import _lib
from .store import ALIGNMENT, RecordLayout, expert_offset, parse_record

EXPERTS_BIN = "experts.bin"
EXPERTS_INDEX = "experts_index.json"
INDEX_FORMAT_VERSION = 1


@dataclass(frozen=True)
class ExpertIndexEntry:
    layer: int
    expert: int
    offset: int
    size: int
    shapes: dict[str, list[int]]
    sha256: str
    quant_error: dict = field(default_factory=dict)


def read_expert_index(path) -> tuple[RecordLayout, list[ExpertIndexEntry]]:
    """Load and validate an expert index (store/layout.py:194-211): an
    unaligned or wrong-sized entry would break the one-read-per-expert rule."""
    doc = json.loads(Path(path).read_text())
    if doc.get("format_version") != INDEX_FORMAT_VERSION:
        raise ValueError(f"unsupported expert index format_version {doc.get('format_version')}")
    layout = RecordLayout.from_dict(doc["layout"])
    entries = [ExpertIndexEntry(**e) for e in doc["entries"]]
    seen: set[tuple[int, int]] = set()
    for e in entries:
        if e.offset % ALIGNMENT or e.size != layout.record_size:
            raise ValueError(f"expert ({e.layer},{e.expert}): offset {e.offset} / size {e.size} breaks the layout")
        if (e.layer, e.expert) in seen:
            raise ValueError(f"duplicate expert ({e.layer},{e.expert}) in index")
        seen.add((e.layer, e.expert))
    return layout, entries


def write_expert_store(store_dir, layout: RecordLayout, records: dict[tuple[int, int], bytes], num_experts: int) -> None:
    """experts.bin + experts_index.json for {(layer, expert): record bytes},
    each record at the reference builder's offset."""
    store_dir = Path(store_dir)
    store_dir.mkdir(parents=True, exist_ok=True)
    rs = layout.record_size
    entries = []
    end = max(expert_offset(lay, e, num_experts, rs) + rs for lay, e in records) if records else 0
    with open(store_dir / EXPERTS_BIN, "wb") as f:
        f.truncate(end)
        for (layer, expert), rec in sorted(records.items()):
            rec = bytes(rec)
            if len(rec) != rs:
                raise ValueError(f"expert ({layer},{expert}): {len(rec)} bytes, the layout's record is {rs}")
            off = expert_offset(layer, expert, num_experts, rs)
            f.seek(off)
            f.write(rec)
            entries.append(ExpertIndexEntry(layer, expert, off, rs, {m: list(s) for m, s in layout.matrices},
                                            hashlib.sha256(rec).hexdigest(), {}))
    doc = {"format_version": INDEX_FORMAT_VERSION, "layout": layout.to_dict(),
           "entries": [asdict(e) for e in sorted(entries, key=lambda e: e.offset)]}
    (store_dir / EXPERTS_INDEX).write_text(json.dumps(doc, indent=1))


def aligned_host_buffer(nbytes: int, *, pinned: bool):
    """A uint8 torch tensor of nbytes starting on a 4096-byte boundary:
    pinned (page-locked, for copies to the GPU) when asked, else ordinary
    host memory. It is a view that keeps the larger allocation alive."""
    import torch

    base = torch.empty(nbytes + ALIGNMENT, dtype=torch.uint8, pin_memory=pinned)
    skip = (-base.data_ptr()) % ALIGNMENT
    return base[skip : skip + nbytes]


class _Store:
    """An open experts.bin (er_store_open)."""

    def __init__(self, path: Path, direct: bool):
        h = C.c_void_p()
        _lib.check(_lib.lib().er_store_open(str(path).encode(), 0 if direct else 1, C.byref(h)), "er_store_open")
        self.handle = h
        size, d = C.c_uint64(), C.c_int()
        _lib.check(_lib.lib().er_store_info(h, C.byref(size), C.byref(d)), "er_store_info")
        self.file_bytes, self.direct = int(size.value), bool(d.value)

    def close(self) -> None:
        if self.handle:
            _lib.lib().er_store_close(self.handle)
            self.handle = None


class ExpertStoreReader:
    """Use as a context manager: holds experts.bin open. read_raw() reads
    into a record-sized aligned buffer of its own, reused (the view is valid
    until the next read); read_into() reads into a caller's 4096-aligned host
    buffer (store/expert_reader.py:43-117)."""

    def __init__(self, store_dir, *, direct: bool = True):
        self.store_dir = Path(store_dir)
        self.layout, entries = read_expert_index(self.store_dir / EXPERTS_INDEX)
        self._entries = {(e.layer, e.expert): e for e in entries}
        self._direct = direct
        self._store: _Store | None = None
        self._buf = None  # torch uint8, 4096-aligned

    def __enter__(self) -> ExpertStoreReader:
        self._store = _Store(self.store_dir / EXPERTS_BIN, self._direct)
        return self

    def __exit__(self, *exc) -> None:
        if self._store is not None:
            self._store.close()
        self._store = self._buf = None

    @property
    def unbuffered(self) -> bool:
        """Whether reads bypass the page cache (O_DIRECT was accepted)."""
        return self._open().direct

    def _open(self) -> _Store:
        if self._store is None:
            raise RuntimeError("ExpertStoreReader must be used as a context manager")
        return self._store

    def entry(self, layer: int, expert: int) -> ExpertIndexEntry:
        return self._entries[(layer, expert)]

    def entries(self) -> list[ExpertIndexEntry]:
        return list(self._entries.values())

    def read_into(self, layer: int, expert: int, address: int) -> int:
        """One read of the record into the host buffer at `address` (4096-
        aligned, at least record_size bytes). Returns the bytes read."""
        st = self._open()
        e = self.entry(layer, expert)
        _lib.check(_lib.lib().er_store_read(st.handle, e.offset, e.size, C.c_void_p(address)), "er_store_read")
        return e.size

    def read_raw(self, layer: int, expert: int) -> memoryview:
        self._open()
        if self._buf is None:
            self._buf = aligned_host_buffer(self.layout.record_size, pinned=False)
        n = self.read_into(layer, expert, self._buf.data_ptr())
        return memoryview(self._buf.numpy())[:n]

    def read(self, layer: int, expert: int) -> dict[str, tuple]:
        """{matrix: (weights, scales[, zeros])}, copies (store/expert_reader.py:103-112)."""
        parsed = parse_record(self.layout, self.read_raw(layer, expert))
        return {m: tuple(np.array(a) for a in v) for m, v in parsed.items()}

    def verify(self, layer: int, expert: int) -> bool:
        """Does the record on disk hash to what the index recorded?"""
        return hashlib.sha256(self.read_raw(layer, expert)).hexdigest() == self.entry(layer, expert).sha256


def load_host_records(store_dir, *, layers: int | None = None, pinned: bool = True, direct: bool = True,
                      threads: int = 8):
    """Every expert of the store in one [layers, experts, record_size] uint8
    host buffer (pinned for the HBM cache), read with `threads` reads in
    flight, one read per record. Returns a HostRecords (the cache's source)."""
    from .cache import HostRecords

    store_dir = Path(store_dir)
    layout, entries = read_expert_index(store_dir / EXPERTS_INDEX)
    nl = layers if layers is not None else max(e.layer for e in entries) + 1
    ne = max(e.expert for e in entries) + 1
    want = {(lay, x) for lay in range(nl) for x in range(ne)}
    have = {(e.layer, e.expert): e for e in entries}
    if want - set(have):
        missing = sorted(want - set(have))[:4]
        raise ValueError(f"the store's index lacks experts {missing} of {nl} layers x {ne} experts")
    rs = layout.record_size
    buf = aligned_host_buffer(nl * ne * rs, pinned=pinned)
    keys = sorted(want)
    offsets = (C.c_uint64 * len(keys))(*[have[k].offset for k in keys])
    dsts = (C.c_void_p * len(keys))(*[buf.data_ptr() + (lay * ne + x) * rs for lay, x in keys])
    st = _Store(store_dir / EXPERTS_BIN, direct)
    failed = C.c_int(-1)
    try:
        rc = _lib.lib().er_store_read_many(st.handle, len(keys), offsets, rs, dsts, threads, C.byref(failed))
        try:
            _lib.check(rc, "er_store_read_many")
        except (OSError, ValueError) as e:
            if 0 <= failed.value < len(keys):  # name the expert, as the reference's cache does
                raise RuntimeError(f"background read of expert {keys[failed.value]} failed") from e
            raise
    finally:
        st.close()
    return HostRecords(buf.view(nl, ne, rs), layout, pin=False)
