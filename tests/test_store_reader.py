"""The expert store on disk (store/expert_reader.py, store/layout.py:148-211,
store/unbuffered_io.py), on the CPU: a store written by the reference's own
record and index writers is read back record for record (one aligned read
each, er_store_read), its sha256s verify, the index is validated as strictly
as the reference validates it, misaligned and short reads fail like the
reference's, and our store writer reproduces the reference's files."""

from __future__ import annotations

import hashlib
import json
import shutil

import numpy as np
import pytest
from conftest import GOLDEN

from expertrelay_b200.store import expert_offset
from expertrelay_b200.store_reader import (
    EXPERTS_BIN,
    EXPERTS_INDEX,
    ExpertStoreReader,
    aligned_host_buffer,
    load_host_records,
    read_expert_index,
    write_expert_store,
)

STORE = GOLDEN / "store_small"
LAYERS, EXPERTS = 2, 3


def test_reads_the_reference_store():
    blob = (STORE / EXPERTS_BIN).read_bytes()
    with ExpertStoreReader(STORE) as r:
        assert len(r.entries()) == LAYERS * EXPERTS
        rs = r.layout.record_size
        assert rs == 8192 and r.layout.hidden == 64 and r.layout.inter == 32
        for layer in range(LAYERS):
            for expert in range(EXPERTS):
                off = expert_offset(layer, expert, EXPERTS, rs)
                assert r.entry(layer, expert).offset == off
                assert bytes(r.read_raw(layer, expert)) == blob[off : off + rs]
                assert r.verify(layer, expert)
                mats = r.read(layer, expert)
                q, s = mats["down_proj"][:2]
                assert q.shape == (64, 32) and q.dtype == np.int8 and s.shape == (64,)
                assert np.abs(q).max() == 127  # row-wise absmax quantization reaches +-127


def test_read_into_a_caller_buffer_and_misaligned_reads():
    with ExpertStoreReader(STORE) as r:
        rs = r.layout.record_size
        buf = aligned_host_buffer(2 * rs, pinned=False)
        assert r.read_into(1, 2, buf.data_ptr() + rs) == rs
        assert bytes(buf[rs:].numpy()) == bytes(r.read_raw(1, 2))
        with pytest.raises(ValueError, match="unaligned unbuffered read"):
            r.read_into(0, 0, buf.data_ptr() + 512)
    with pytest.raises(RuntimeError, match="context manager"):
        ExpertStoreReader(STORE).read_raw(0, 0)


def _index(tmp_path, edit):
    d = tmp_path / "s"
    shutil.copytree(STORE, d)
    doc = json.loads((d / EXPERTS_INDEX).read_text())
    edit(doc)
    (d / EXPERTS_INDEX).write_text(json.dumps(doc))
    return d


def test_index_validation(tmp_path):
    def version(doc):
        doc["format_version"] = 2

    def unaligned(doc):
        doc["entries"][1]["offset"] += 512

    def size(doc):
        doc["entries"][2]["size"] = 4096

    def duplicate(doc):
        doc["entries"][3]["expert"] = doc["entries"][4]["expert"]
        doc["entries"][3]["layer"] = doc["entries"][4]["layer"]

    for edit, match in ((version, "format_version"), (unaligned, "breaks the layout"), (size, "breaks the layout"),
                        (duplicate, "duplicate expert")):
        d = _index(tmp_path / edit.__name__, edit)
        with pytest.raises(ValueError, match=match):
            read_expert_index(d / EXPERTS_INDEX)


def test_short_read_is_an_error(tmp_path):
    def beyond(doc):
        doc["entries"][0]["offset"] = 100 * 8192  # past the end of experts.bin

    d = _index(tmp_path, beyond)
    with ExpertStoreReader(d) as r:
        with pytest.raises(OSError, match="short read"):
            r.read_raw(0, 0)


@pytest.mark.parametrize("threads", [1, 4])
def test_failed_bulk_read_names_the_expert(tmp_path, threads):
    """A record whose read comes up short fails the whole load with the
    reference cache's error for a failed read (cache/expert_cache.py:
    281-282): RuntimeError naming the (layer, expert) key, chained from the
    read's OSError."""

    def beyond(doc):
        e = next(e for e in doc["entries"] if (e["layer"], e["expert"]) == (1, 2))
        e["offset"] = 100 * 8192  # past the end of experts.bin

    d = _index(tmp_path, beyond)
    with pytest.raises(RuntimeError, match=r"background read of expert \(1, 2\) failed") as info:
        load_host_records(d, pinned=False, threads=threads)
    assert isinstance(info.value.__cause__, OSError) and "short read" in str(info.value.__cause__)


@pytest.mark.parametrize("threads", [1, 4])
def test_load_host_records(threads):
    blob = np.frombuffer((STORE / EXPERTS_BIN).read_bytes(), dtype=np.uint8)
    recs = load_host_records(STORE, pinned=False, threads=threads)
    assert (recs.layers, recs.experts) == (LAYERS, EXPERTS)
    np.testing.assert_array_equal(recs.tensor.numpy().reshape(-1), blob)


def test_writer_reproduces_the_reference_store(tmp_path):
    layout, entries = read_expert_index(STORE / EXPERTS_INDEX)
    blob = (STORE / EXPERTS_BIN).read_bytes()
    rs = layout.record_size
    records = {(e.layer, e.expert): blob[e.offset : e.offset + rs] for e in entries}
    write_expert_store(tmp_path, layout, records, EXPERTS)
    assert (tmp_path / EXPERTS_BIN).read_bytes() == blob
    ours, ref = json.loads((tmp_path / EXPERTS_INDEX).read_text()), json.loads((STORE / EXPERTS_INDEX).read_text())
    assert ours == ref
    assert all(e["sha256"] == hashlib.sha256(records[(e["layer"], e["expert"])]).hexdigest() for e in ours["entries"])
