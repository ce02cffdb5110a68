"""Prefetch session bookkeeping (simulate mode: no GPU) against the
reference's cache-manager semantics restated in oracle/cache.py
(ControlledExpertCacheManager, runtime/cache_manager.py:208-279), one LRU of
slots_per_layer entries per layer, demand misses inserted."""
import numpy as np
import pytest

from oracle import cache as ocache


def _compare(seed, layers=3, experts=32, slots=6, steps=400):
    from mtp_b200 import PrefetchSession
    rng = np.random.default_rng(seed)
    sess = PrefetchSession(layers, experts, slots, 4096, simulate=True)
    ref = [ocache.LruExpertCache(slots) for _ in range(layers)]
    for _ in range(steps):
        l = int(rng.integers(layers))
        if rng.random() < 0.5:
            ids = rng.choice(experts, size=int(rng.integers(1, 5)), replace=False)
            sess.issue(l, ids)
            for e in ids:
                ref[l].issue_prefetch(l, int(e))
        else:
            ids = rng.choice(experts, size=int(rng.integers(1, 4)), replace=False)
            sess.demand(l, ids)
            for e in ids:
                ref[l].demand(l, int(e))
    got = sess.poll()
    snaps = [r.snapshot() for r in ref]
    for name in ("issued_fetch_count", "used_fetch_count", "unused_fetch_count", "demand_count",
                 "demand_hit_count", "demand_miss_count", "evicted_before_use_count"):
        assert got[name] == sum(getattr(s_, name) for s_ in snaps), name
    assert got["resident_count"] == sum(s_.resident_count for s_ in snaps)
    assert got["ready_late_miss_count"] == 0 and got["inflight_count"] == 0
    sess.close()


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_session_counters_match_cache_manager(built_lib, seed):
    _compare(seed)


def test_session_capacity_one_and_full(built_lib):
    _compare(7, layers=1, experts=8, slots=1, steps=200)
    _compare(8, layers=2, experts=8, slots=8, steps=200)


def test_session_rejects_bad_arguments(built_lib):
    import ctypes as C
    from mtp_b200 import PrefetchSession, _lib
    sess = PrefetchSession(2, 16, 4, 4096, simulate=True)
    with pytest.raises(_lib.MtpError):
        sess.issue(2, [0])          # layer out of range
    with pytest.raises(_lib.MtpError):
        sess.demand(0, [16])        # expert out of range
    sess.close()
    lib = _lib.load()
    assert lib.mtp_prefetch_poll(C.c_uint64(12345), None) == 7  # bad handle
    cfg = _lib.MtpPrefetchConfig(0, 1, 8, 9, 4096, None, None, None, 1)  # more slots than experts
    h = _lib.u64()
    assert lib.mtp_prefetch_session_create(C.byref(cfg), C.byref(h)) == 2
