"""The LRU replay restatement (oracle/cache_oracle.py) on the reference's own
scenarios: a 1-slot cache switching between two experts 102 times fills 102
times with 101 evictions (tests/gpu/test_gpu_expert_cache.py:28-69 restated
on the CPU replay), empty slots are filled before any eviction, ties go to
the lower slot, and the sweep's expected misses behave as LRU must."""
from oracle.cache_oracle import LruLayer, pass_accesses, replay_passes
from specfit_b200 import synthetic


def test_alternating_single_slot():
    lay = LruLayer(1)
    for i in range(102):
        lay.access(i % 2)
    assert (lay.h2d_submissions, lay.evictions, lay.resident_hits) == (102, 101, 0)
    assert lay.resident() == (1,)


def test_empty_slots_first_then_lru_then_lower_slot():
    lay = LruLayer(3)
    for e in (5, 6, 7):
        assert lay.access(e)
    assert lay.evictions == 0 and lay.resident() == (5, 6, 7)
    assert not lay.access(5)            # hit refreshes 5
    assert lay.access(8)                # evicts 6, the least recently used
    assert lay.resident() == (5, 8, 7) and lay.evictions == 1
    lay2 = LruLayer(2)
    assert lay2.access(1) and lay2.access(2)
    lay2.last_used = [4, 4]             # equal stamps: the lower slot goes
    lay2.access(3)
    assert lay2.resident() == (3, 2)


def test_execution_orders():
    assert pass_accesses([7, 3, 3, 9]) == [3, 7, 9]
    assert pass_accesses([7, 3, 9], "resident_first", resident=(9,)) == [9, 3, 7]


def test_sweep_expectations_are_lru_shaped():
    """Zipf routes of configuration 3 (129 tokens, top-8, 4 layers): a cache
    as large as the layer misses only on the cold pass; smaller caches miss
    more, and a warm pass never misses more than a cold one."""
    routes = [synthetic.zipf_routes(129, l, seed=3).reshape(-1) for l in range(4)]
    distinct = sum(len(set(r.tolist())) for r in routes)
    full = replay_passes(128, routes, 2)
    assert full == [distinct, 0]
    prev = None
    for slots in (48, 24, 12):
        cold, warm = replay_passes(slots, routes, 2)
        assert warm <= cold == distinct
        if prev is not None:
            assert warm >= prev
        prev = warm
