"""HBM expert cache bookkeeping (er_cache_* in dry mode, no device) and the
prefetch policy.

The cases follow the reference's own tests of CachedExpertSource
(tests/test_expert_cache.py) and PrefetchPolicy (tests/test_prefetch_policy.py),
with one difference of contract: the B200 forward pass holds every expert it
acquired for a layer until end_layer(layer), so a case where the reference
loads experts one after another acquires each and ends the layer in between.
Cases about threads and queued reads have no counterpart (copies are handed
to the GPU's copy engine and never withdrawn); the GPU tests cover waiting for
a copy in flight.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from expertrelay_b200.cache import CacheTooSmall, HbmExpertCache, HostRecords, record_views, slots_for
from expertrelay_b200.prefetch import IsotonicCalibrator, PrefetchPolicy, RankedIsotonicCalibrator, load_calibrator
from expertrelay_b200.store import FMT_INT8, RecordLayout

LAYOUT = RecordLayout(FMT_INT8, 32, 16)  # a 4096-byte record
LAYERS, EXPERTS = 3, 8


@pytest.fixture(scope="module")
def source() -> HostRecords:
    recs = np.zeros((LAYERS, EXPERTS, LAYOUT.record_size), dtype=np.uint8)
    return HostRecords(recs, LAYOUT, pin=False)


def cache(source, slots: float, **kw) -> HbmExpertCache:
    kw.setdefault("min_free_slots", 1)
    return HbmExpertCache(source, capacity_bytes=int(slots * LAYOUT.record_size), dry=True, **kw)


def use(c: HbmExpertCache, layer: int, expert: int) -> None:
    """One expert used and released, like one reference load()."""
    c.acquire(layer, [expert])
    c.end_layer(layer)


def test_budget_buys_whole_slots_and_nothing_more(source):
    c = cache(source, 5.9)
    assert c.num_slots == 5 == slots_for(5.9 * LAYOUT.record_size, LAYOUT.record_size)
    assert c.capacity_bytes == 5 * LAYOUT.record_size
    for layer in range(3):
        c.acquire(layer, list(range(4)))
        c.end_layer(layer)
        c.acquire(layer, list(range(4, 8)))
        c.end_layer(layer)
    assert len(c.cached_keys()) == 5


def test_lru_eviction(source):
    c = cache(source, 3)
    for key in [(0, 0), (0, 1), (0, 2), (0, 0), (0, 3)]:  # (0, 1) is least recently used when (0, 3) arrives
        use(c, *key)
    assert c.cached_keys() == {(0, 0), (0, 2), (0, 3)}
    s = c.stats
    assert (s.demand_reads, s.cache_hits, s.loads) == (4, 1, 5)


def test_held_experts_are_not_evicted(source):
    c = cache(source, 2)
    c.acquire(0, [0])  # held by layer 0 until end_layer(0)
    c.prefetch(1, [0, 1, 2], keep=[])  # one free slot: (1, 0); nothing else may go
    assert (0, 0) in c.cached_keys() and (1, 0) in c.cached_keys()
    assert c.stats.prefetches_skipped_full == 2
    c.end_layer(0)


def test_a_layer_needing_more_slots_than_exist_is_refused(source):
    c = cache(source, 3)
    with pytest.raises(CacheTooSmall):
        c.acquire(0, [0, 1, 2, 3])


def test_repeats_within_one_acquire_are_one_load(source):
    c = cache(source, 4)
    addrs = c.acquire(1, [5, 5, 2])
    c.end_layer(1)
    assert addrs[0] == addrs[1] and c.stats.loads == 2 and c.stats.demand_reads == 2


def test_pinned_experts_stay(source):
    pinned = [(0, e) for e in range(8)]
    c = cache(source, 11, pinned=pinned)
    reads_after_pinning = c.stats.demand_reads
    for layer in (1, 2):
        for e in range(8):
            use(c, layer, e)
    for e in range(8):
        use(c, 0, e)
    assert set(pinned) <= c.cached_keys()
    assert c.stats.demand_reads - reads_after_pinning == 16  # layers 1-2 only; layer 0 all hits
    assert c.stats.cache_hits == 8


def test_too_small_budget_is_rejected(source):
    with pytest.raises(CacheTooSmall):
        cache(source, 9, pinned=[(0, e) for e in range(8)], min_free_slots=2)
    with pytest.raises(CacheTooSmall):
        cache(source, 0.5)


def test_prefetch_then_use_is_a_prefetch_hit(source):
    c = cache(source, 6)
    c.prefetch(1, [3, 5], keep=[])
    c.acquire(1, [5, 3])
    c.end_layer(1)
    s = c.stats
    assert (s.prefetch_hits, s.demand_reads, s.prefetch_reads, s.prefetches_issued) == (2, 0, 2, 2)


def test_unused_prefetch_evicted_counts_as_wasted(source):
    c = cache(source, 3)
    c.prefetch(2, [7], keep=[])
    for e in range(3):
        use(c, 0, e)
    assert c.stats.prefetches_wasted == 1
    assert (2, 7) not in c.cached_keys()


def test_prefetch_keeps_the_listed_experts(source):
    c = cache(source, 3)
    for e in range(3):
        use(c, 0, e)
    c.prefetch(1, [4], keep=[(0, 0)])  # (0, 0) was least recently used, but is about to be needed
    assert (0, 0) in c.cached_keys()
    assert (0, 1) not in c.cached_keys()


def test_prefetch_read_budget_counts_only_new_reads(source):
    c = cache(source, 8)
    use(c, 1, 0)
    c.prefetch(1, [0, 2, 3, 4], keep=[], max_new_reads=2)  # (1, 0) is cached: costs nothing
    assert c.stats.prefetches_issued == 2
    assert c.stats.prefetches_skipped_budget == 1
    assert {(1, 0), (1, 2), (1, 3)} <= c.cached_keys()
    assert (1, 4) not in c.cached_keys()


def test_resize_shrinks_keeping_the_most_recent_experts(source):
    c = cache(source, 6)
    for e in range(5):
        use(c, 0, e)
    assert c.resize(3 * LAYOUT.record_size) == 3 and c.capacity_bytes == 3 * LAYOUT.record_size
    assert c.cached_keys() == {(0, 2), (0, 3), (0, 4)}  # the least recently used went first
    hits = c.stats.cache_hits
    use(c, 0, 4)
    assert c.stats.cache_hits == hits + 1


def test_resize_grows_and_new_slots_are_used(source):
    c = cache(source, 2)
    assert c.resize(5 * LAYOUT.record_size) == 5
    c.acquire(1, list(range(5)))
    c.end_layer(1)
    assert len(c.cached_keys()) == 5 and c.stats.demand_reads == 5


def test_resize_keeps_pinned_and_refuses_too_small(source):
    c = cache(source, 6, pinned=[(0, 0), (0, 1)], min_free_slots=2)
    for e in range(2, 6):
        use(c, 1, e)
    with pytest.raises(CacheTooSmall):
        c.resize(3 * LAYOUT.record_size)
    assert c.num_slots == 6  # unchanged after a refusal
    assert c.resize(4 * LAYOUT.record_size) == 4
    assert {(0, 0), (0, 1)} <= c.cached_keys()


def test_resize_refused_while_a_layer_holds_slots(source):
    c = cache(source, 4)
    c.acquire(0, [1])
    with pytest.raises(ValueError):
        c.resize(2 * LAYOUT.record_size)
    c.end_layer(0)
    assert c.resize(2 * LAYOUT.record_size) == 2


def test_keys_outside_the_source_are_rejected(source):
    c = cache(source, 4)
    with pytest.raises(ValueError):
        c.acquire(LAYERS, [0])
    with pytest.raises(ValueError):
        c.acquire(0, [EXPERTS])
    assert c.cached_keys() == set()


# ---------------------------------------------------------------- prefetch policy


def calibrator() -> IsotonicCalibrator:
    """P(picked) = 0 below probability 0.12, 0.5 up to 0.25, 0.9 above."""
    cal = IsotonicCalibrator(num_bins=3)
    cal.edges = np.array([0.12, 0.25])
    cal.values = np.array([0.0, 0.5, 0.9])
    return cal


def test_top_k_by_router_probability():
    logits = np.log(np.array([0.05, 0.4, 0.1, 0.3, 0.15]))
    choice = PrefetchPolicy(top_k=3).choose(logits)
    assert choice.experts == [1, 3, 4] and choice.skipped_low_confidence == 0


def test_low_confidence_guesses_are_skipped():
    logits = np.log(np.array([0.05, 0.4, 0.1, 0.3, 0.15]))
    choice = PrefetchPolicy(top_k=4, min_probability=0.4, calibrator=calibrator()).choose(logits)
    assert choice.experts == [1, 3, 4] and choice.skipped_low_confidence == 1
    choice = PrefetchPolicy(top_k=4, min_probability=0.6, calibrator=calibrator()).choose(logits)
    assert choice.experts == [1, 3] and choice.skipped_low_confidence == 2


def test_several_tokens_use_each_experts_best_probability():
    logits = np.log(np.array([[0.7, 0.1, 0.1, 0.1], [0.1, 0.1, 0.1, 0.7]]))
    assert PrefetchPolicy(top_k=2).choose(logits).experts == [0, 3]


def test_calibrator_round_trip_and_validation():
    cal = calibrator()
    back = IsotonicCalibrator.from_dict(cal.to_dict())
    x = np.linspace(0, 1, 11)
    np.testing.assert_array_equal(back.predict(x), cal.predict(x))
    with pytest.raises(ValueError):
        IsotonicCalibrator.from_dict({"num_bins": 2, "edges": [0.5], "values": [0.9, 0.1]})


def test_ranked_calibrator_maps_each_rank(tmp_path):
    top = calibrator()
    rest = IsotonicCalibrator(1)
    rest.edges, rest.values = np.array([]), np.array([0.2])
    ranked = RankedIsotonicCalibrator(max_rank=2)
    ranked.per_rank = [top, rest]
    out = ranked.predict(np.array([0.3, 0.4, 0.1]))  # ranks 1, 0, 2 (2 shares the last map)
    np.testing.assert_allclose(out, [0.2, 0.9, 0.2])
    path = tmp_path / "cal.json"
    path.write_text(json.dumps([{"calibrator": top.to_dict(), "rank_calibrator": ranked.to_dict()}]))
    cal, prov = load_calibrator(path)
    assert isinstance(cal, RankedIsotonicCalibrator) and prov["kind"] == "rank_isotonic"
    cal, prov = load_calibrator(path, kind="single")
    assert isinstance(cal, IsotonicCalibrator) and prov["kind"] == "isotonic"
    with pytest.raises(ValueError):
        load_calibrator(path, kind="other")


@pytest.mark.parametrize("fmt", ["int8", "int4", "gptq_asym"])
def test_record_views_match_the_store_parser(fmt):
    """What load() hands out for a cached record: views at the record
    layout's offsets, the fields of the reference's Int8Matrix / Int4Matrix
    (runtime/weights.py:51-80), equal to the store's own parse of the same
    bytes; zero points only for asymmetric GPTQ records."""
    import torch

    from expertrelay_b200 import synth
    from expertrelay_b200.store import parse_record

    blk = synth.make_block(61, fmt=fmt, hidden=256, inter=128, shared_inter=384, num_experts=8, top_k=2)
    rec = blk.records()[5]
    views = record_views(blk.layout, torch.from_numpy(rec.copy()))
    want = parse_record(blk.layout, rec)
    assert set(views) == set(want)
    for name, m in views.items():
        if fmt == "int8":
            assert np.array_equal(m.q.numpy(), want[name][0]) and np.array_equal(m.scales.numpy(), want[name][1])
            continue
        assert m.group_size == blk.layout.group and m.scales.dtype == torch.float16
        assert np.array_equal(m.packed.numpy(), want[name][0])
        assert np.array_equal(m.scales.numpy(), want[name][1])
        if fmt == "gptq_asym":
            assert np.array_equal(m.zeros.numpy(), want[name][2])
        else:
            assert m.zeros is None
