"""GPU: experts read from an on-disk store into pinned host memory
(load_host_records, er_store_read_many) serve the HBM expert cache: a
paged MoE stack over a store written from synthetic layers gives exactly
the output of the same stack over the in-memory records."""

from __future__ import annotations

import pytest
import torch

from expertrelay_b200 import _lib, synth
from expertrelay_b200.cache import HbmExpertCache, HostRecords
from expertrelay_b200.paged import PagedMoeStack
from expertrelay_b200.store_reader import ExpertStoreReader, load_host_records, write_expert_store

pytestmark = pytest.mark.gpu

SHAPE = {"hidden": 256, "inter": 128, "shared_inter": 384, "num_experts": 16, "top_k": 4}


def test_store_loaded_records_serve_the_paged_stack(cuda, tmp_path):
    blocks = [synth.make_block(60 + layer, **SHAPE) for layer in range(3)]
    mem = HostRecords.from_blocks(blocks)
    layout, rs = mem.layout, mem.layout.record_size
    records = {(l, e): mem.record(l, e).numpy().tobytes() for l in range(3) for e in range(SHAPE["num_experts"])}
    write_expert_store(tmp_path, layout, records, SHAPE["num_experts"])
    loaded = load_host_records(tmp_path, pinned=True, threads=4)
    assert loaded.tensor.is_pinned()
    assert torch.equal(loaded.tensor, mem.tensor)
    with ExpertStoreReader(tmp_path) as r:
        assert all(r.verify(l, e) for l in range(3) for e in range(SHAPE["num_experts"]))
    outs = []
    for src in (mem, loaded):
        cache = HbmExpertCache(src, capacity_bytes=20 * rs)
        stack = PagedMoeStack(blocks, cache)
        x = torch.from_numpy(synth.make_tokens(5, 9, SHAPE["hidden"])).to(cuda)
        outs.append(stack.forward(x, path=_lib.PATH_TC))
        torch.cuda.synchronize()
        cache.close()
    assert torch.equal(outs[0], outs[1])
