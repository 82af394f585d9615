"""GPU: the HBM expert cache (er_cache_*) and the paged MoE stack on it.

Records copied into slots must equal the host records, through evictions,
refills and resizes; a load whose prefetch copy is still in flight must wait
for that copy instead of copying again; and a stack of MoE layers served
from a cache much smaller than its experts must give exactly the output of
the same layers with every record resident.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from expertrelay_b200 import _lib, synth
from expertrelay_b200.cache import CacheTooSmall, HbmExpertCache, HostRecords
from expertrelay_b200.moe import MoeBlock
from expertrelay_b200.paged import PagedMoeStack
from expertrelay_b200.prefetch import PrefetchPolicy

pytestmark = pytest.mark.gpu

SHAPE = {"hidden": 256, "inter": 128, "shared_inter": 384, "num_experts": 16, "top_k": 4}
LAYERS = 3


@pytest.fixture(scope="module")
def blocks():
    return [synth.make_block(50 + layer, **SHAPE) for layer in range(LAYERS)]


@pytest.fixture(scope="module")
def source(blocks, cuda):
    return HostRecords.from_blocks(blocks)


def _slot_bytes(c: HbmExpertCache, addr: int) -> torch.Tensor:
    off = int(addr) - c.arena_base
    return c.arena[off : off + c.layout.record_size]


def test_slots_hold_the_host_records_through_evictions(source):
    rs = source.layout.record_size
    c = HbmExpertCache(source, capacity_bytes=5 * rs)
    rng = np.random.default_rng(0)
    for step in range(12):
        layer = step % LAYERS
        experts = rng.choice(SHAPE["num_experts"], size=4, replace=False)
        addrs = c.acquire(layer, experts)
        got = [_slot_bytes(c, a).clone() for a in addrs]  # ordered after the copies on this stream
        c.end_layer(layer)
        torch.cuda.synchronize()
        for e, g in zip(experts, got):
            assert torch.equal(g.cpu(), source.record(layer, int(e))), f"layer {layer} expert {e}"
    s = c.stats
    assert s.loads == 48 and s.demand_reads + s.cache_hits == 48 and s.demand_reads > 5
    c.close()


def test_a_load_waits_for_its_prefetch_in_flight(source):
    rs = source.layout.record_size
    c = HbmExpertCache(source, capacity_bytes=4 * rs)
    with torch.cuda.stream(c.copy_stream):
        torch.cuda._sleep(200_000_000)  # holds the copy engine queue: the prefetch below stays in flight
    c.prefetch(1, [3], keep=[])
    assert c.lookup(1, 3)[1] == _lib.SLOT_LOADING
    addr = c.acquire(1, [3])[0]
    got = _slot_bytes(c, addr).clone()  # this stream waited for the copy
    c.end_layer(1)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), source.record(1, 3))
    s = c.stats
    assert (s.prefetch_waits, s.demand_reads, s.prefetches_issued, s.prefetch_reads) == (1, 0, 1, 1)
    c.close()


def test_load_views_match_the_record(source, blocks):
    rs = source.layout.record_size
    c = HbmExpertCache(source, capacity_bytes=3 * rs)
    w = c.load(2, 7)
    torch.cuda.synchronize()
    for name, (q, sc) in blocks[2].experts[7].items():
        assert np.array_equal(w[name].q.cpu().numpy(), q)
        assert np.array_equal(w[name].scales.cpu().numpy(), sc)
    c.end_layer(2)
    with pytest.raises(CacheTooSmall):
        c.acquire(0, [0, 1, 2, 3])
    c.close()


@pytest.mark.parametrize("fmt", ["int4", "gptq_asym"])
def test_load_views_of_int4_records(cuda, fmt):
    from expertrelay_b200.store import parse_record

    blk = synth.make_block(61, fmt=fmt, **SHAPE)
    src = HostRecords.from_blocks([blk])
    c = HbmExpertCache(src, capacity_bytes=2 * src.layout.record_size)
    w = c.load(0, 5)
    torch.cuda.synchronize()
    want = parse_record(src.layout, blk.records()[5])
    for name, m in w.items():
        assert m.packed.is_cuda and m.group_size == src.layout.group
        assert np.array_equal(m.packed.cpu().numpy(), want[name][0])
        assert np.array_equal(m.scales.cpu().numpy(), want[name][1])
        if fmt == "gptq_asym":
            assert np.array_equal(m.zeros.cpu().numpy(), want[name][2])
        else:
            assert m.zeros is None
    c.end_layer(0)
    c.close()


def test_resize_moves_the_kept_records(source):
    rs = source.layout.record_size
    c = HbmExpertCache(source, capacity_bytes=6 * rs)
    c.acquire(0, [0, 1, 2, 3, 4])
    c.end_layer(0)
    old = c.arena_base
    assert c.resize(3 * rs) == 3 and c.arena_base != old
    assert c.cached_keys() == {(0, 2), (0, 3), (0, 4)}
    addrs = c.acquire(0, [2, 3, 4])
    got = [_slot_bytes(c, a).clone() for a in addrs]
    c.end_layer(0)
    torch.cuda.synchronize()
    for e, g in zip((2, 3, 4), got):
        assert torch.equal(g.cpu(), source.record(0, e))
    assert c.stats.cache_hits == 3
    c.close()


@pytest.mark.parametrize("path", ["gemv", "tc"])
@pytest.mark.parametrize("prefetch", [False, True])
def test_paged_stack_equals_resident_layers(blocks, source, cuda, path, prefetch):
    """Twenty slots for 48 records: a layer's experts (up to all 16) fit at
    once, and the layers evict each other's. Both sides route from the same
    router logits, so the outputs must be bit-identical."""
    p = {"gemv": _lib.PATH_GEMV, "tc": _lib.PATH_TC}[path]
    rs = source.layout.record_size
    cache = HbmExpertCache(source, capacity_bytes=20 * rs)
    policy = PrefetchPolicy(top_k=SHAPE["top_k"]) if prefetch else None
    stack = PagedMoeStack(blocks, cache, prefetcher=policy)
    resident = [MoeBlock.from_host_block(b, device=cuda) for b in blocks]
    for n in (1, 8, 40):
        x = torch.from_numpy(synth.make_tokens(7 + n, n, SHAPE["hidden"])).to(cuda)
        ref = x
        for blk in resident:  # routed from the same logits as the stack (er_linear_f32)
            ref = ref + blk.forward(ref, logits=blk.router_logits(ref), path=p)
        for _ in range(2):
            got = stack.forward(x, path=p)
            torch.cuda.synchronize()
            assert torch.equal(got, ref), f"n={n}"
    s = cache.stats
    assert s.demand_reads + s.cache_hits + s.prefetch_hits + s.prefetch_waits == s.loads
    assert s.demand_reads + s.prefetches_issued > 20  # records were evicted and copied again
    if prefetch:
        assert s.prefetches_issued > 0
    cache.close()
