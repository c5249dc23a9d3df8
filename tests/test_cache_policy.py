"""Residency policy of the HBM expert cache, on the CPU (no slab: the policy
alone).  Restates tests/vulkan_resident_expert_cache_test.cpp:314-382 of the
reference (E0, E1, E0, E2 with room for two: E1 is evicted) and compares random
access streams with a Python model of
src/backend/vulkan_resident_expert_cache.cpp:40-200 (victim = smallest
(use count, last use, key); use counts survive evictions)."""
import random

import pytest

ACCOUNTED = 17152  # the reference fixture's accounted bytes per expert


@pytest.fixture(scope="module")
def osm():
    from osm_b200 import build

    build.build()
    import osm_b200

    return osm_b200


class Model:
    def __init__(self, budget, accounted):
        self.budget, self.acc = budget, accounted
        self.entries = {}          # key -> [freq, last_use]
        self.hist = {}
        self.tick = 0
        self.hits = self.misses = self.loads = self.evictions = 0
        self.protect = set()

    def acquire(self, layer, experts, failing=()):
        """get() of each pick of one call; entries used by this call are not
        evicted by it (they must stay resident until the call runs).  A pick
        whose source fails ends the call; the picks before it stay loaded."""
        self.protect = set()
        try:
            for e in experts:
                self.get(layer, e, source_fails=e in failing)
                self.protect.add((layer << 32) | e)
        finally:
            self.protect = set()

    def get(self, layer, expert, source_fails=False):
        self.tick += 1
        key = (layer << 32) | expert
        f = self.hist.get(key, 0) + 1
        self.hist[key] = f
        if key in self.entries:
            self.hits += 1
            self.entries[key] = [f, self.tick]
            return
        self.misses += 1
        if source_fails:
            # the reference fetches and uploads before it evicts
            # (vulkan_resident_expert_cache.cpp:101-140): nothing else changes
            raise RuntimeError("source failed")
        while self.entries and (len(self.entries) + 1) * self.acc > self.budget:
            cand = [k for k in self.entries if k not in self.protect]
            victim = min(cand, key=lambda k: (self.entries[k][0], self.entries[k][1], k))
            del self.entries[victim]
            self.evictions += 1
        self.entries[key] = [f, self.tick]
        self.loads += 1

    def stats(self):
        return {"hits": self.hits, "misses": self.misses, "loads": self.loads,
                "evictions": self.evictions, "resident_entries": len(self.entries),
                "resident_bytes": len(self.entries) * self.acc, "budget_bytes": self.budget}


def test_reference_eviction_kat(osm):
    c = osm.ExpertCache(None, 2 * ACCOUNTED, ACCOUNTED)
    c.get(0, 0)
    c.get(0, 1)
    s = c.stats()
    assert (s["hits"], s["misses"], s["loads"], s["evictions"]) == (0, 2, 2, 0)
    assert s["resident_entries"] == 2 and s["resident_bytes"] == 2 * ACCOUNTED
    c.get(0, 0)
    c.get(0, 2)
    s = c.stats()
    assert (s["hits"], s["misses"], s["loads"], s["evictions"]) == (1, 3, 3, 1)
    assert s["resident_entries"] == 2 and s["resident_bytes"] <= s["budget_bytes"]
    assert c.contains(0, 0) and not c.contains(0, 1) and c.contains(0, 2)
    c.get(0, 0)
    c.get(0, 2)
    s = c.stats()
    assert (s["hits"], s["misses"], s["loads"], s["evictions"]) == (3, 3, 3, 1)
    c.close()


@pytest.mark.parametrize("seed", range(4))
def test_random_streams_match_the_policy_model(osm, seed):
    rng = random.Random(seed)
    slots = rng.choice([3, 5, 8])
    c = osm.ExpertCache(None, slots * ACCOUNTED, ACCOUNTED)
    m = Model(slots * ACCOUNTED, ACCOUNTED)
    # Zipf-skewed experts over two layers
    weights = [1.0 / (r + 1) ** 1.1 for r in range(24)]
    for _ in range(600):
        layer = rng.randrange(2)
        expert = rng.choices(range(24), weights)[0]
        c.get(layer, expert)
        m.get(layer, expert)
    assert c.stats() == m.stats()
    for layer in range(2):
        for e in range(24):
            assert c.contains(layer, e) == (((layer << 32) | e) in m.entries)
    c.close()


def test_one_call_larger_than_the_budget_is_refused(osm):
    from osm_b200 import OsmError

    c = osm.ExpertCache(None, 3 * ACCOUNTED, ACCOUNTED)
    c.acquire(0, [1, 2, 3])
    with pytest.raises(OsmError) as e:
        c.acquire(0, [4, 5, 6, 7])  # four experts of one call, room for three
    assert e.value.code == -4  # OSM_ENOMEM
    # refused before anything changed (ExpertCache::fetch rejects an
    # oversized request before mutation, tests/expert_cache_test.cpp:180-195)
    s = c.stats()
    assert (s["hits"], s["misses"], s["loads"], s["evictions"]) == (0, 3, 3, 0)
    assert all(c.contains(0, e) for e in (1, 2, 3))
    c.close()
    with pytest.raises(OsmError):
        osm.ExpertCache(None, ACCOUNTED - 1, ACCOUNTED).get(0, 0)


def test_failing_source_leaves_residency_unchanged(osm):
    """A host source that fails in the middle of an acquire (the analogue of
    tests/expert_cache_test.cpp:150-176): the failing expert is not made
    resident and evicts nothing; the picks before it stay loaded; a pick
    resident before the call is not lost; the failed get counts one miss and
    one use, as in the reference's get().  The same experts then load once
    the source works again."""
    from osm_b200 import OsmError

    broken = {7}

    def source(layer, expert):
        if expert in broken:
            raise RuntimeError("storage read failed")
        return 1

    c = osm.ExpertCache(None, 3 * ACCOUNTED, ACCOUNTED, source=source)
    m = Model(3 * ACCOUNTED, ACCOUNTED)
    c.acquire(0, [0, 1, 2])
    m.acquire(0, [0, 1, 2])
    c.get(0, 0)
    m.get(0, 0)
    with pytest.raises(OsmError) as e:
        c.acquire(0, [0, 5, 7])      # 5 loads (evicting 1), then 7 fails
    assert e.value.code == -2        # OSM_ERUNTIME
    with pytest.raises(RuntimeError):
        m.acquire(0, [0, 5, 7], failing=broken)
    assert c.stats() == m.stats()
    assert c.contains(0, 0) and c.contains(0, 5) and c.contains(0, 2)
    assert not c.contains(0, 7) and not c.contains(0, 1)
    s = c.stats()
    assert (s["misses"], s["loads"], s["evictions"]) == (5, 4, 1)
    broken.clear()
    c.acquire(0, [7])
    m.acquire(0, [7])
    assert c.contains(0, 7) and c.stats() == m.stats()
    c.close()
