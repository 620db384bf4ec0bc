"""The adapter pool: every adapter the router knows, where its weights live,
and which ones hold the engine's LoRA GPU slots.

Placement tiers, coldest first: ``disk`` (only the PEFT directory), ``cpu``
(a host copy) and ``gpu`` (in a LoRA slot, servable now). Weights change tier
one step at a time through a *backend* with four verbs -- ``load`` (disk to
cpu), ``activate`` (cpu to gpu), ``deactivate`` (gpu to cpu) and ``unload``
(cpu to disk) -- which is the engine's slot table in a server and a fake in
tests.

Levels: an ``active`` adapter is routable (its centroid is in the pool's
index); a ``retired`` one holds no memory and is never chosen by the router
but stays servable by name, and keeps its centroid and reference samples so
that coming back needs no encoding.

Policies (the reference's behaviour, ``adapter_routing/pool.py:107-545``;
the structure here is this package's own):

* usage: each adapter carries a meter that every hit raises by one and that
  decays with half-life ``half_life_s``;
* GPU slots: the ``protected`` hottest slot holders are never evicted; a slot
  is freed from the coldest other holder that no running request uses;
* admission: a candidate is measured against the active set on reference
  samples (its self-recall, the share it would take from others); a full
  active set retires its least used, then most redundant, member past its
  grace period (``retire_least_used``), lets the newcomer in retired
  (``admit_retired``), or refuses (``reject``).

Persistence: after each change the routable index is written to a new
numbered file when it changed, then the registry (``pool.json``) is replaced
in one rename, so a reader sees the old pool or the new one; a restart
restores levels, pins and ids.
"""

from __future__ import annotations

import json
import os
import re
import threading
import time
from dataclasses import dataclass, field

from ... import dprint
from .decision import admission_report
from .index import CentroidIndex

GPU, CPU, DISK = "gpu", "cpu", "disk"
ACTIVE, RETIRED = "active", "retired"
RETIRE_LEAST_USED, ADMIT_RETIRED, REJECT = "retire_least_used", "admit_retired", "reject"
REGISTRY_FILE = "pool.json"
REGISTRY_LAYOUT = "dsv-adapter-pool/2"
_INDEX_FILE = re.compile(r"index-(\d+)\.npz")

_RANK = {DISK: 0, CPU: 1, GPU: 2}
_BY_RANK = (DISK, CPU, GPU)
_VERB = {(0, 1): "load", (1, 2): "activate", (2, 1): "deactivate", (1, 0): "unload"}


class PoolFull(Exception):
    """The active set has no room for another adapter."""


class _Meter:
    """Exponentially decaying hit count."""

    __slots__ = ("level", "stamp")

    def __init__(self, now: float):
        self.level, self.stamp = 0.0, now

    def read(self, now: float, half_life: float) -> float:
        dt = now - self.stamp
        if half_life <= 0 or dt <= 0:
            return self.level
        return self.level * 2.0 ** (-dt / half_life)

    def bump(self, now: float, half_life: float) -> None:
        self.level, self.stamp = self.read(now, half_life) + 1.0, now


@dataclass
class PoolEntry:
    """One adapter: identity, placement, level and usage."""
    name: str
    path: str
    job: str | None
    uid: int
    meter: _Meter
    level: str = ACTIVE
    tier: str = DISK
    pinned: bool = False
    since: float = 0.0            # when it (re-)entered the active set
    centroid: object = None
    refs: object = None
    hits: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def enabled(self) -> bool:
        return self.level == ACTIVE


class AdapterPool:
    def __init__(self, backend, index: CentroidIndex | None = None, *, capacity: int = 32,
                 gpu_slots: int = 1, protected: int = 0, half_life_s: float = 300.0,
                 clock=time.monotonic, directory: str | None = None, when_full: str = RETIRE_LEAST_USED,
                 grace_s: float = 600.0, min_pool: int = 4, min_self_recall: float = 0.0,
                 max_stolen: float = 1.0):
        if when_full not in (RETIRE_LEAST_USED, ADMIT_RETIRED, REJECT):
            raise ValueError(f"when_full must be one of {RETIRE_LEAST_USED}, {ADMIT_RETIRED}, {REJECT}")
        self.backend = backend
        self.index = index if index is not None else CentroidIndex()
        self.capacity, self.gpu_slots = int(capacity), int(gpu_slots)
        self.protected = min(max(int(protected), 0), self.gpu_slots)
        self.half_life_s, self.grace_s = float(half_life_s), float(grace_s)
        self.clock, self.directory, self.when_full = clock, directory, when_full
        self.min_pool = int(min_pool)
        self.min_self_recall, self.max_stolen = float(min_self_recall), float(max_stolen)
        self.entries: dict[str, PoolEntry] = {}
        self.listeners: list = []          # fn(pool), called when the routable set changed
        self.version = 0                   # registry revision
        self.evictions = 0
        self.cold_loads = 0
        self._uid_next = 1
        self._index_stale = True
        self._batch = 0                    # > 0: inside a compound change, publish once at its end
        self._lock = threading.RLock()

    # ------------------------------------------------------------ queries
    def __len__(self) -> int:
        return len(self.entries)

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def get(self, name: str) -> PoolEntry:
        try:
            return self.entries[name]
        except KeyError:
            raise KeyError(f"adapter '{name}' is not in the pool") from None

    def names(self) -> list[str]:
        return list(self.entries)

    def _with_level(self, level: str) -> list[str]:
        return [e.name for e in self.entries.values() if e.level == level]

    def active_names(self) -> list[str]:
        return self._with_level(ACTIVE)

    def retired_names(self) -> list[str]:
        return self._with_level(RETIRED)

    def routable_names(self) -> list[str]:
        return self.index.names

    def count(self, tier: str) -> int:
        return sum(e.tier == tier for e in self.entries.values())

    def score_of(self, e: PoolEntry, now: float | None = None) -> float:
        """``e``'s decayed usage at ``now``."""
        return e.meter.read(self.clock() if now is None else now, self.half_life_s)

    # ------------------------------------------------------------ internals
    def _set_tier(self, e: PoolEntry, tier: str) -> None:
        """Walk ``e``'s weights to ``tier`` one step at a time; the entry
        records every step the backend completed."""
        goal = _RANK[tier]
        while _RANK[e.tier] != goal:
            here = _RANK[e.tier]
            nxt = here + (1 if goal > here else -1)
            getattr(self.backend, _VERB[(here, nxt)])(e)
            e.tier = _BY_RANK[nxt]

    def _route_set_changed(self) -> None:
        self._index_stale = True
        for fn in self.listeners:
            fn(self)

    def _index_put(self, e: PoolEntry) -> None:
        self.index.add(e.name, e.centroid, refs=e.refs)
        self._route_set_changed()

    def _index_drop(self, name: str) -> None:
        if self.index.remove(name):
            self._route_set_changed()

    def _changed(self) -> None:
        if self.directory and self._batch == 0:
            self.save(self.directory)

    def _slot_holders(self, now: float) -> list[PoolEntry]:
        """GPU slot holders, hottest first (ties by name)."""
        return sorted((e for e in self.entries.values() if e.tier == GPU),
                      key=lambda e: (-e.meter.read(now, self.half_life_s), e.name))

    def protected_names(self, now: float | None = None) -> set[str]:
        now = self.clock() if now is None else now
        return {e.name for e in self._slot_holders(now)[:self.protected]}

    def choose_victim(self, in_use=(), exclude: str | None = None) -> str | None:
        """The slot holder to evict: the coldest one outside the protected
        set, not used by a running request and not ``exclude``."""
        holders = self._slot_holders(self.clock())
        spare = set(in_use) | {e.name for e in holders[:self.protected]} | {exclude}
        for e in reversed(holders):
            if e.name not in spare:
                return e.name
        return None

    def _full(self) -> str:
        return f"no room in the active set: {len(self.active_names())} of {self.capacity} adapters are active"

    # ------------------------------------------------------------ membership
    def register(self, name: str, path: str, centroid=None, refs=None, job: str | None = None,
                 load: bool = True, prewarm: bool = True, level: str = ACTIVE, pinned: bool = False,
                 uid: int | None = None) -> PoolEntry:
        """Add an adapter as it is (no admission check). ``load`` brings its
        weights to the host; ``prewarm`` also gives it a GPU slot if one is
        free (it never evicts for that)."""
        with self._lock:
            if name in self.entries:
                raise ValueError(f"adapter '{name}' is already in the pool")
            if level == ACTIVE and len(self.active_names()) >= self.capacity:
                raise PoolFull(self._full())
            uid = self._uid_next if uid is None else int(uid)
            self._uid_next = max(self._uid_next, uid + 1)
            now = self.clock()
            e = PoolEntry(name, path, job, uid, _Meter(now), level=level, pinned=pinned, since=now,
                          centroid=centroid, refs=refs)
            self.entries[name] = e
            try:
                if level == ACTIVE:
                    if load:
                        self._set_tier(e, CPU)
                    if centroid is not None:
                        self._index_put(e)
                    if load and prewarm and self.count(GPU) < self.gpu_slots:
                        self._set_tier(e, GPU)
            except Exception:
                del self.entries[name]
                self._index_drop(name)
                raise
            dprint(f"[adapter-pool] + {name} ({e.level}, {e.tier}); {len(self.active_names())}/"
                   f"{self.capacity} active, {len(self.retired_names())} retired")
            self._changed()
            return e

    def remove(self, name: str) -> None:
        with self._lock:
            e = self.get(name)
            self._set_tier(e, DISK)
            self._index_drop(name)
            del self.entries[name]
            self._changed()

    # ------------------------------------------------------------ serving
    def ensure_gpu(self, name: str, in_use=()) -> bool:
        """Give ``name`` a GPU slot, evicting the coldest unprotected holder
        when every slot is taken. False when nothing can be evicted; the
        adapter then at least reaches the host tier."""
        with self._lock:
            e = self.get(name)
            if e.tier == GPU:
                return True
            if self.count(GPU) >= self.gpu_slots:
                victim = self.choose_victim(in_use, exclude=name)
                if victim is None:
                    if e.tier == DISK:
                        self._set_tier(e, CPU)
                    return False
                self._set_tier(self.entries[victim], CPU)
                self.evictions += 1
            self._set_tier(e, GPU)
            return True

    def note_hit(self, name: str, in_use=(), place: bool = True) -> PoolEntry:
        """A request uses ``name`` (routed or by name): its meter goes up by
        one; with ``place`` it is also given a GPU slot now if possible."""
        with self._lock:
            e = self.get(name)
            e.meter.bump(self.clock(), self.half_life_s)
            e.hits += 1
            if e.tier == DISK:
                self.cold_loads += 1
            if place:
                self.ensure_gpu(name, in_use)
            return e

    # ------------------------------------------------------------ admission
    def _redundancy(self, e: PoolEntry) -> float:
        """Cosine of ``e``'s centroid to the nearest other routable centroid."""
        if e.centroid is None or e.name not in self.index or len(self.index) < 2:
            return 0.0
        cos = self.index.scores(e.centroid)
        return max(float(c) for n, c in zip(self.index.names, cos) if n != e.name)

    def _retire_candidate(self, exclude: str | None) -> str | None:
        """Least used active adapter that is unpinned and past its grace
        period; among equally used ones the most redundant (then by name)."""
        now = self.clock()
        pool = [e for e in self.entries.values()
                if e.level == ACTIVE and not e.pinned and e.name != exclude and now - e.since >= self.grace_s]
        if not pool:
            return None
        best = min(pool, key=lambda e: (round(self.score_of(e, now), 6), -self._redundancy(e), e.name))
        return best.name

    def _verdict(self, name: str, centroid, refs) -> dict:
        """The admission report of a candidate: the level it may reach on its
        own merits (before the capacity check) and the measurements."""
        rep = {"name": name, "level": ACTIVE, "reason": "", "retired": None}
        if centroid is None:
            rep.update(level=RETIRED, reason="no centroid: servable by name only")
            return rep
        rep.update(admission_report(self.index, name, centroid, refs, self.min_pool))
        recall, stolen = rep.get("self_recall"), rep.get("stolen_max", 0.0)
        if recall is not None and recall < self.min_self_recall:
            rep.update(level=RETIRED, reason=f"self-recall {recall} < {self.min_self_recall}")
        elif stolen > self.max_stolen:
            rep.update(level=RETIRED, reason=f"takes {stolen} of {rep['stolen_from']}")
        return rep

    def admit(self, name: str, path: str, centroid=None, refs=None, job: str | None = None,
              load: bool = False, prewarm: bool = False, pinned: bool = False) -> dict:
        """The way into the active set for a new adapter, a retired one coming
        back or a new version of a known one. Returns the admission report
        with the ``level`` reached, the ``reason`` when it is ``retired``, and
        the adapter ``retired`` to make room, if any."""
        with self._lock:
            known = self.entries.get(name)
            if centroid is None and known is not None:
                centroid, refs = known.centroid, known.refs
            rep = self._verdict(name, centroid, refs)
            needs_room = (rep["level"] == ACTIVE and not (known is not None and known.level == ACTIVE)
                          and len(self.active_names()) >= self.capacity)
            victim = None
            if needs_room:
                if self.when_full == REJECT:
                    raise PoolFull(self._full())
                victim = self._retire_candidate(name) if self.when_full == RETIRE_LEAST_USED else None
                if victim is None:
                    rep.update(level=RETIRED, reason="active set is full" if self.when_full == ADMIT_RETIRED
                               else "active set is full and nobody can be retired")
            self._batch += 1
            try:
                if victim is not None:
                    self.retire(victim)
                    rep["retired"] = victim
                if known is None:
                    self.register(name, path, centroid, refs, job, load=load, prewarm=prewarm,
                                  level=rep["level"], pinned=pinned)
                else:
                    self._update(known, path, centroid, refs, job, pinned, rep["level"])
            finally:
                self._batch -= 1
            self._changed()
            note = (f" ({rep['reason']})" if rep["reason"] else "") + (f", retired {victim}" if victim else "")
            dprint(f"[adapter-pool] admission of {name}: {rep['level']}{note}")
            return rep

    def _update(self, e: PoolEntry, path: str, centroid, refs, job, pinned: bool, level: str) -> None:
        """A known adapter re-admitted: new weights get a new id (and leave
        every tier), then the level the report allows."""
        if path != e.path:
            self._set_tier(e, DISK)
            e.path, e.uid = path, self._uid_next
            self._uid_next += 1
        e.centroid, e.refs = centroid, refs
        e.job = job or e.job
        e.pinned = e.pinned or pinned
        if level == ACTIVE:
            e.level, e.since = ACTIVE, self.clock()
            self._index_put(e)
        elif e.level == ACTIVE:
            self.retire(e.name)

    # ------------------------------------------------------------ operator
    def offload(self, name: str) -> PoolEntry:
        with self._lock:
            e = self.get(name)
            self._set_tier(e, DISK)
            self._changed()
            return e

    def retire(self, name: str) -> PoolEntry:
        with self._lock:
            e = self.get(name)
            e.level = RETIRED
            self._index_drop(name)
            self._set_tier(e, DISK)
            self._changed()
            return e

    def reactivate(self, name: str) -> dict:
        with self._lock:
            return self.admit(name, self.get(name).path)

    def pin(self, name: str, pinned: bool = True) -> PoolEntry:
        with self._lock:
            e = self.get(name)
            e.pinned = bool(pinned)
            self._changed()
            return e

    def op(self, name: str, op: str):
        """The verbs of ``POST /adapters/{name}/{op}``."""
        verbs = {
            "load": lambda: {"on_gpu": self.ensure_gpu(name)},
            "offload": lambda: self.describe(self.offload(name)),
            "retire": lambda: self.describe(self.retire(name)),
            "reactivate": lambda: self.reactivate(name),
            "pin": lambda: self.describe(self.pin(name, True)),
            "unpin": lambda: self.describe(self.pin(name, False)),
            "remove": lambda: (self.remove(name), {"removed": name})[1],
        }
        aliases = {"prewarm": "load", "unload": "offload", "disable": "retire", "enable": "reactivate"}
        fn = verbs.get(aliases.get(op, op))
        if fn is None:
            raise ValueError(f"unknown adapter op '{op}' (one of {', '.join([*verbs, *aliases])})")
        with self._lock:
            return fn()

    # ------------------------------------------------------------ reporting
    def describe(self, e: PoolEntry, now: float | None = None) -> dict:
        return {"name": e.name, "path": e.path, "job": e.job, "uid": e.uid, "level": e.level,
                "enabled": e.enabled, "pinned": e.pinned, "tier": e.tier, "hits": e.hits,
                "score": round(self.score_of(e, now), 4), "indexed": e.centroid is not None}

    def status(self) -> dict:
        with self._lock:
            now = self.clock()
            return {"capacity": self.capacity, "gpu_slots": self.gpu_slots,
                    "active": len(self.active_names()), "retired": len(self.retired_names()),
                    "version": self.version, "protected": sorted(self.protected_names(now)),
                    "evictions": self.evictions, "cold_loads": self.cold_loads,
                    "adapters": [self.describe(self.entries[n], now) for n in sorted(self.entries)]}

    # ------------------------------------------------------------ persistence
    def save(self, directory: str) -> None:
        """Write the routable index to a new numbered file if it changed, then
        replace the registry in one rename; index files older than the
        previous revision are deleted."""
        with self._lock:
            os.makedirs(directory, exist_ok=True)
            if self._index_stale or self.version == 0:
                self.version += 1
                self.index.save(os.path.join(directory, f"index-{self.version}.npz"))
                self._index_stale = False
            now = self.clock()
            doc = {"layout": REGISTRY_LAYOUT, "version": self.version, "uid_next": self._uid_next,
                   "index_file": f"index-{self.version}.npz",
                   "adapters": [{"name": e.name, "path": e.path, "job": e.job, "uid": e.uid, "level": e.level,
                                 "pinned": e.pinned, "tier": e.tier, "hits": e.hits,
                                 "score": round(self.score_of(e, now), 4)} for e in self.entries.values()]}
            target = os.path.join(directory, REGISTRY_FILE)
            part = f"{target}.{os.getpid()}.part"
            with open(part, "w") as f:
                json.dump(doc, f, indent=1)
            os.replace(part, target)
            for fn in os.listdir(directory):
                m = _INDEX_FILE.fullmatch(fn)
                if m and int(m.group(1)) < self.version - 1:
                    try:
                        os.unlink(os.path.join(directory, fn))
                    except OSError:
                        pass

    def restore(self, directory: str, centroids: CentroidIndex | None = None) -> int:
        """Bring a saved pool back: every adapter with its level, pin and id,
        its weights on the host (and a free GPU slot) unless it was on disk;
        centroids from ``centroids`` or the registry's index file. Returns the
        number of adapters."""
        reg = read_registry(directory)
        if reg is None:
            return 0
        with self._lock:
            if centroids is None and reg.get("index_file"):
                centroids = CentroidIndex.load_or_none(os.path.join(directory, reg["index_file"]))
            self._batch += 1
            try:
                self.version = max(self.version, int(reg.get("version", 0)))
                for rec in reg["adapters"]:
                    have = centroids is not None and rec["name"] in centroids
                    warm = rec.get("tier", CPU) != DISK
                    self.register(rec["name"], rec["path"],
                                  centroids.centroid_of(rec["name"]) if have else None,
                                  centroids.refs.get(rec["name"]) if have else None,
                                  rec.get("job"), load=warm, prewarm=warm, level=rec.get("level", ACTIVE),
                                  pinned=bool(rec.get("pinned")), uid=rec.get("uid"))
                self._uid_next = max(self._uid_next, int(reg.get("uid_next", 0)))
            finally:
                self._batch -= 1
            self._index_stale = True
            self._changed()
            return len(reg["adapters"])


def read_registry(directory: str) -> dict | None:
    """The registry of a pool directory, or None when it is absent, unreadable
    or of another layout."""
    try:
        with open(os.path.join(directory, REGISTRY_FILE)) as f:
            doc = json.load(f)
    except (OSError, ValueError):
        return None
    if not isinstance(doc, dict) or doc.get("layout") != REGISTRY_LAYOUT or not isinstance(doc.get("adapters"), list):
        return None
    return doc
