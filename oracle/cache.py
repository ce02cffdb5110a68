"""Expert-cache managers restated in plain Python (hit / miss accounting).

Test infrastructure (see ``oracle/__init__.py``).

Reference: src/mtp_expert_prefetch/runtime/cache_manager.py
  * ``CacheManagerSnapshot`` :193-205 - counter names kept verbatim;
  * ``ControlledExpertCacheManager`` :208-279 - bounded LRU keyed by
    (layer, expert); ``issue_prefetch`` inserts a prefetched entry unless
    resident; ``demand`` counts a hit (and a used fetch the first time a
    prefetched entry is used) or a miss that inserts a demand entry; an entry
    evicted while prefetched and unused counts as evicted-before-use;
  * ``ReadyTimeExpertCacheManager`` :298-578 - the same with a virtual transfer
    queue: an issued fetch becomes resident only when its batch completes; a
    demand that finds its key still in flight is a ready-late miss.
"""
from __future__ import annotations

import math
from collections import OrderedDict, deque
from dataclasses import asdict, dataclass


@dataclass
class _Entry:
    prefetched: bool
    used: bool = False


@dataclass(frozen=True)
class Snapshot:
    capacity: int
    resident_count: int
    issued_fetch_count: int
    used_fetch_count: int
    unused_fetch_count: int
    demand_count: int
    demand_hit_count: int
    demand_miss_count: int
    evicted_before_use_count: int

    def as_dict(self):
        return asdict(self)


class LruExpertCache:
    """cache_manager.py:208-279."""

    def __init__(self, capacity: int):
        self.capacity = int(capacity)
        self.cache: OrderedDict = OrderedDict()
        self.issued = self.used = self.demands = self.hits = self.misses = self.evicted_unused = 0

    def _insert(self, key, entry):
        if self.capacity <= 0:
            if entry.prefetched and not entry.used:
                self.evicted_unused += 1
            return
        self.cache[key] = entry
        self.cache.move_to_end(key)
        while len(self.cache) > self.capacity:
            _, old = self.cache.popitem(last=False)
            if old.prefetched and not old.used:
                self.evicted_unused += 1

    def issue_prefetch(self, layer: int, expert: int) -> bool:
        key = (int(layer), int(expert))
        if key in self.cache:
            self.cache.move_to_end(key)
            return False
        self.issued += 1
        self._insert(key, _Entry(prefetched=True))
        return True

    def demand(self, layer: int, expert: int) -> bool:
        self.demands += 1
        key = (int(layer), int(expert))
        entry = self.cache.get(key)
        if entry is None:
            self.misses += 1
            self._insert(key, _Entry(prefetched=False, used=True))
            return False
        self.hits += 1
        if entry.prefetched and not entry.used:
            self.used += 1
        entry.used = True
        self.cache.move_to_end(key)
        return True

    def snapshot(self) -> Snapshot:
        unused = sum(1 for e in self.cache.values() if e.prefetched and not e.used)
        return Snapshot(self.capacity, len(self.cache), self.issued, self.used, unused,
                        self.demands, self.hits, self.misses, self.evicted_unused)


class ReadyTimeExpertCache(LruExpertCache):
    """cache_manager.py:298-578 (virtual-time transfer queue)."""

    def __init__(self, capacity: int, *, service_us_per_issue: float = 0.0,
                 service_us_per_batch: float = 0.0, queue_batch_size: int = 1,
                 queue_deadline_us: float = 0.0):
        super().__init__(capacity)
        for name, v in (("service_us_per_issue", service_us_per_issue),
                        ("service_us_per_batch", service_us_per_batch),
                        ("queue_deadline_us", queue_deadline_us)):
            if not math.isfinite(float(v)):
                raise ValueError(f"{name} must be finite")
        self.per_issue = max(0.0, float(service_us_per_issue))
        self.per_batch = max(0.0, float(service_us_per_batch))
        self.batch = max(1, int(queue_batch_size) or 1)
        self.deadline = max(0.0, float(queue_deadline_us))
        self.pending: list = []
        self.pending_first = None
        self.completions: deque = deque()
        self.inflight: set = set()
        self.server_free = 0.0
        self.last_completion = 0.0
        self.last_arrival = 0.0
        self.ready_late = 0
        self.late_unused = 0
        self.batches = 0
        self.service_total = 0.0
        self.wait_total = 0.0
        self.max_delay = 0.0

    def issue_prefetch(self, layer: int, expert: int, *, arrival_us: float) -> bool:
        key = (int(layer), int(expert))
        self.advance_to(arrival_us)
        if key in self.cache:
            self.cache.move_to_end(key)
            return False
        if key in self.inflight:
            return False
        self.issued += 1
        self.inflight.add(key)
        if not self.pending:
            self.pending_first = float(arrival_us)
        self.pending.append(key)
        self._flush_full(float(arrival_us))
        return True

    def demand(self, layer: int, expert: int, *, arrival_us: float) -> bool:
        due = float(arrival_us) + self.deadline
        self._flush_due(due)
        self._drain(due)
        self.demands += 1
        key = (int(layer), int(expert))
        entry = self.cache.get(key)
        if entry is not None:
            self.hits += 1
            if entry.prefetched and not entry.used:
                self.used += 1
            entry.used = True
            self.cache.move_to_end(key)
            return True
        if key in self.inflight:
            self.ready_late += 1
        self.misses += 1
        self._insert(key, _Entry(prefetched=False, used=True))
        return False

    def advance_to(self, arrival_us: float) -> None:
        a = max(0.0, float(arrival_us))
        self.last_arrival = max(self.last_arrival, a)
        self._flush_due(a)
        self._drain(a)

    def finish(self) -> None:
        if self.pending and self.pending_first is not None:
            first = self.pending_first
            ready = first + self.deadline if self.deadline > 0.0 else self.last_arrival
            keys = list(self.pending)
            self.pending.clear()
            self.pending_first = None
            self._flush(keys, ready, first)
        self._drain(float("inf"))

    def snapshot_ready(self) -> dict:
        base = self.snapshot().as_dict()
        base["unused_fetch_count"] += self.late_unused
        base.update(ready_late_miss_count=self.ready_late, late_completion_unused_count=self.late_unused,
                    queue_batch_count=self.batches)
        return base

    def _flush(self, keys, ready, first):
        if not keys:
            return
        service = self.per_batch + self.per_issue * float(len(keys))
        start = max(self.server_free, float(ready))
        self.batches += 1
        self.service_total += service
        self.wait_total += max(0.0, start - float(ready))
        done = start + service
        self.max_delay = max(self.max_delay, done - float(first))
        self.server_free = done
        self.last_completion = done
        self.completions.append((done, list(keys)))

    def _flush_full(self, ready):
        while len(self.pending) >= self.batch:
            first = ready if self.pending_first is None else self.pending_first
            keys = self.pending[: self.batch]
            del self.pending[: self.batch]
            self._flush(keys, ready, first)
            self.pending_first = ready if self.pending else None

    def _flush_due(self, t):
        if (self.pending and self.pending_first is not None and self.deadline > 0.0
                and float(t) >= self.pending_first + self.deadline):
            first = self.pending_first
            keys = list(self.pending)
            self.pending.clear()
            self.pending_first = None
            self._flush(keys, first + self.deadline, first)

    def _drain(self, t):
        while self.completions and self.completions[0][0] <= t:
            _, keys = self.completions.popleft()
            for key in keys:
                self.inflight.discard(key)
                entry = self.cache.get(key)
                if entry is not None:
                    if not entry.prefetched:
                        self.late_unused += 1
                    self.cache.move_to_end(key)
                    continue
                self._insert(key, _Entry(prefetched=True))
