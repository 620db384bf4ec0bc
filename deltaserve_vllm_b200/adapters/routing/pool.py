"""The adapter pool: every routable adapter, where its weights are, and the
policy deciding which ones hold the engine's LoRA GPU slots.

Tiers: ``gpu`` (in a LoRA slot, usable now), ``cpu`` (host copy), ``disk``
(only the PEFT directory). Levels: ``active`` adapters compete in routing;
``retired`` ones are never auto-selected and hold no memory but stay servable
by name (their centroid and reference samples are kept, so re-activation
needs no encoding).

Weights move through a *backend* with four calls — ``load`` (disk -> cpu),
``activate`` (cpu -> gpu), ``deactivate`` (gpu -> cpu), ``unload`` (-> disk) —
the engine's LoRA slots in a server, a fake in tests.

GPU slots are kept by decayed hit frequency (half-life ``half_life_s``): the
eviction victim is the lowest-scoring slot holder not used by running
requests and not among the ``protected`` best. Admission compares a candidate
with the active set on reference samples (self-recall, share stolen from
others); a full active set retires its least-used, most redundant member
(``retire_least_used``), admits the newcomer retired (``admit_retired``), or
refuses (``reject``). Behaviour follows
``deltaserve-plugin/deltaserve/adapter_routing/pool.py:107-545``.

The registry (``pool.json``) and the routable index it points at are written
after each change (new index file first, registry swapped by one rename), so
a restart restores levels, pins and ids.
"""

from __future__ import annotations

import functools
import json
import os
import re
import threading
import time
from dataclasses import dataclass

from ... import dprint
from .decision import admission_report
from .index import CentroidIndex

GPU, CPU, DISK = "gpu", "cpu", "disk"
ACTIVE, RETIRED = "active", "retired"
RETIRE_LEAST_USED, ADMIT_RETIRED, REJECT = "retire_least_used", "admit_retired", "reject"
REGISTRY_FILE = "pool.json"
_ROUTABLE = re.compile(r"routable-(\d+)\.npz")


def decayed(score: float, dt: float, half_life: float) -> float:
    return score if half_life <= 0 or dt <= 0 else score * 0.5 ** (dt / half_life)


class PoolFull(Exception):
    """The active set has no room for another adapter."""


# Where an adapter's weights can be, coldest first; a move walks this order
# one hop at a time, calling the backend verb of each hop.
_TIERS = (DISK, CPU, GPU)
_HOP_UP = {DISK: "load", CPU: "activate"}          # tier -> verb to the next warmer tier
_HOP_DOWN = {GPU: "deactivate", CPU: "unload"}     # tier -> verb to the next colder tier


@dataclass
class PoolEntry:
    """One adapter of the pool: identity, placement and usage.

    ``usage`` is a frequency with exponential decay: every hit adds 1 to the
    value decayed to the hit's time (``usage_at``)."""
    name: str
    path: str
    job: str | None = None
    uid: int = 0                  # stable id (never reused, survives restarts)
    tier: str = DISK
    level: str = ACTIVE
    pinned: bool = False
    admitted_at: float = 0.0
    centroid: object = None
    refs: object = None
    hits: int = 0
    usage: float = 0.0
    usage_at: float = 0.0

    @property
    def enabled(self) -> bool:
        return self.level == ACTIVE


def _locked(fn):
    @functools.wraps(fn)
    def wrap(self, *a, **kw):
        with self._lock:
            return fn(self, *a, **kw)
    return wrap


class AdapterPool:
    def __init__(self, backend, index: CentroidIndex | None = None, capacity: int = 32,
                 gpu_slots: int = 1, protected: int = 0, half_life_s: float = 300.0,
                 clock=time.monotonic, directory: str | None = None,
                 when_full: str = RETIRE_LEAST_USED, grace_s: float = 600.0, min_pool: int = 4,
                 min_self_recall: float = 0.0, max_stolen: float = 1.0):
        self.backend = backend
        self.index = index if index is not None else CentroidIndex()
        self.capacity, self.gpu_slots = int(capacity), int(gpu_slots)
        self.protected = max(0, min(int(protected), self.gpu_slots))
        self.half_life_s = float(half_life_s)
        self.clock = clock
        self.directory = directory
        self.when_full, self.grace_s = when_full, float(grace_s)
        self.min_pool = int(min_pool)
        self.min_self_recall, self.max_stolen = float(min_self_recall), float(max_stolen)
        self.entries: dict[str, PoolEntry] = {}
        self.version = 0
        self.evictions = 0
        self.cold_loads = 0
        self._next_uid = 1
        self._dirty = True
        self._hold_save = 0
        self._lock = threading.RLock()
        self.listeners: list = []          # fn(pool) after the routable set changed

    # ------------------------------------------------------------ membership
    def __len__(self) -> int:
        return len(self.entries)

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def get(self, name: str) -> PoolEntry:
        if name not in self.entries:
            raise KeyError(f"adapter '{name}' is not in the pool")
        return self.entries[name]

    def names(self) -> list[str]:
        return list(self.entries)

    def active_names(self) -> list[str]:
        return [n for n, e in self.entries.items() if e.level == ACTIVE]

    def retired_names(self) -> list[str]:
        return [n for n, e in self.entries.items() if e.level == RETIRED]

    def routable_names(self) -> list[str]:
        return list(self.index.names)

    def _index_changed(self) -> None:
        self._dirty = True
        for fn in self.listeners:
            fn(self)

    def _full_message(self) -> str:
        return f"no room in the active set: {len(self.active_names())} of {self.capacity} adapters are active"

    def _publish(self) -> None:
        if self.directory and not self._hold_save:
            self.save(self.directory)

    @_locked
    def register(self, name: str, path: str, centroid=None, refs=None, job: str | None = None,
                 load: bool = True, prewarm: bool = True, level: str = ACTIVE, pinned: bool = False,
                 uid: int | None = None) -> PoolEntry:
        """Add an adapter. ``load`` brings it to the CPU tier; ``prewarm`` also
        gives it a free GPU slot (never by evicting)."""
        if name in self.entries:
            raise ValueError(f"adapter '{name}' is already in the pool")
        if level == ACTIVE and len(self.active_names()) >= self.capacity:
            raise PoolFull(self._full_message())
        if uid is None:
            uid = self._next_uid
        self._next_uid = max(self._next_uid, uid + 1)
        now = self.clock()
        e = PoolEntry(name=name, path=path, job=job, uid=uid, level=level, pinned=pinned, admitted_at=now,
                      centroid=centroid, refs=refs, usage_at=now)
        self.entries[name] = e
        try:
            if level == ACTIVE:
                if load:
                    self._move(e, CPU)
                if centroid is not None:
                    self.index.add(name, centroid, refs=refs)
                    self._index_changed()
                if load and prewarm and self.count(GPU) < self.gpu_slots:
                    self._move(e, GPU)
        except Exception:
            self.entries.pop(name, None)
            if self.index.remove(name):
                self._index_changed()
            raise
        dprint(f"[adapter-pool] + {name} ({e.level}, {e.tier}); {len(self.active_names())}/"
               f"{self.capacity} active, {len(self.retired_names())} retired")
        self._publish()
        return e

    @_locked
    def remove(self, name: str) -> None:
        e = self.get(name)
        self._move(e, DISK)
        if self.index.remove(name):
            self._index_changed()
        del self.entries[name]
        self._publish()

    # ------------------------------------------------------------ tiers
    def count(self, tier: str) -> int:
        return sum(1 for e in self.entries.values() if e.tier == tier)

    def _move(self, e: PoolEntry, target: str) -> None:
        """Bring ``e``'s weights to ``target``, one tier at a time (the backend
        sees load / activate going warmer, deactivate / unload going colder).
        The entry's tier follows every hop that succeeded."""
        want = _TIERS.index(target)
        while _TIERS.index(e.tier) != want:
            here = _TIERS.index(e.tier)
            warmer = want > here
            getattr(self.backend, (_HOP_UP if warmer else _HOP_DOWN)[e.tier])(e)
            e.tier = _TIERS[here + (1 if warmer else -1)]

    def score_of(self, e: PoolEntry, now: float | None = None) -> float:
        """Decayed usage of ``e`` at ``now``."""
        now = self.clock() if now is None else now
        return decayed(e.usage, now - e.usage_at, self.half_life_s)

    def protected_names(self, now: float | None = None) -> set[str]:
        now = self.clock() if now is None else now
        gpu = sorted((e for e in self.entries.values() if e.tier == GPU),
                     key=lambda e: (-self.score_of(e, now), e.name))
        return {e.name for e in gpu[:self.protected]}

    def choose_victim(self, in_use=(), exclude: str | None = None) -> str | None:
        now = self.clock()
        keep = set(in_use) | self.protected_names(now) | ({exclude} if exclude else set())
        cands = [e for e in self.entries.values() if e.tier == GPU and e.name not in keep]
        if not cands:
            return None
        return min(cands, key=lambda e: (self.score_of(e, now), e.name)).name

    @_locked
    def ensure_gpu(self, name: str, in_use=()) -> bool:
        """Give ``name`` a GPU slot, freeing the least-used unprotected slot
        when all are taken; False when no slot can be freed (the adapter then
        at least reaches the CPU tier)."""
        e = self.get(name)
        if e.tier != GPU and self.count(GPU) >= self.gpu_slots:
            victim = self.choose_victim(in_use, exclude=name)
            if victim is None:
                self._move(e, max(e.tier, CPU, key=_TIERS.index))
                return False
            self._move(self.entries[victim], CPU)
            self.evictions += 1
        self._move(e, GPU)
        return True

    @_locked
    def note_hit(self, name: str, in_use=(), place: bool = True) -> PoolEntry:
        """A request uses ``name`` (routed or named): one more unit of decayed
        usage; with ``place``, try to give it a GPU slot now."""
        e = self.get(name)
        now = self.clock()
        e.usage, e.usage_at = self.score_of(e, now) + 1.0, now
        e.hits += 1
        self.cold_loads += e.tier == DISK
        if place:
            self.ensure_gpu(name, in_use)
        return e

    # ------------------------------------------------------------ admission
    def _retire_victim(self, exclude: str | None = None) -> str | None:
        """Least used active adapter (unpinned, past its grace period); among
        equals the most redundant (closest to another active centroid)."""
        now = self.clock()
        cands = [e for e in self.entries.values() if e.level == ACTIVE and not e.pinned
                 and e.name != exclude and now - e.admitted_at >= self.grace_s]
        if not cands:
            return None

        def redundancy(e):
            if e.centroid is None or e.name not in self.index or len(self.index) < 2:
                return 0.0
            s = self.index.scores(e.centroid)
            s[self.index.names.index(e.name)] = -1.0
            return float(s.max())
        return min(cands, key=lambda e: (round(self.score_of(e, now), 6), -redundancy(e), e.name)).name

    @_locked
    def admit(self, name: str, path: str, centroid=None, refs=None, job: str | None = None,
              load: bool = False, prewarm: bool = False, pinned: bool = False) -> dict:
        """The one way into the active set (new adapter, a retired one coming
        back, or a new version of an existing one). Returns the admission
        report with the ``level`` reached and why."""
        old = self.entries.get(name)
        if centroid is None and old is not None:
            centroid, refs = old.centroid, old.refs
        rep = {"name": name, "level": ACTIVE, "reason": "", "retired": None}
        if centroid is None:
            rep.update(level=RETIRED, reason="no centroid: servable by name only")
        else:
            rep.update(admission_report(self.index, name, centroid, refs, self.min_pool))
            sr = rep.get("self_recall")
            if sr is not None and sr < self.min_self_recall:
                rep.update(level=RETIRED, reason=f"self-recall {sr} < {self.min_self_recall}")
            elif rep.get("stolen_max", 0.0) > self.max_stolen:
                rep.update(level=RETIRED, reason=f"takes {rep['stolen_max']} of {rep['stolen_from']}")
        was_active = old is not None and old.level == ACTIVE
        victim = None
        if rep["level"] == ACTIVE and not was_active and len(self.active_names()) >= self.capacity:
            if self.when_full == REJECT:
                raise PoolFull(self._full_message())
            if self.when_full == RETIRE_LEAST_USED:
                victim = self._retire_victim(exclude=name)
            if victim is None:
                rep.update(level=RETIRED, reason="active set is full" if self.when_full == ADMIT_RETIRED
                           else "active set is full and nobody can be retired")
        self._hold_save += 1
        try:
            if victim is not None:
                self.retire(victim)
                rep["retired"] = victim
            if old is None:
                self.register(name, path, centroid, refs, job, load=load, prewarm=prewarm,
                              level=rep["level"], pinned=pinned)
            else:
                if path != old.path:          # a new version: new weights, new id
                    self._move(old, DISK)
                    old.path, old.uid = path, self._next_uid
                    self._next_uid += 1
                old.centroid, old.refs, old.job = centroid, refs, job or old.job
                old.pinned = old.pinned or pinned
                if rep["level"] == ACTIVE:
                    old.level, old.admitted_at = ACTIVE, self.clock()
                    self.index.add(name, centroid, refs=refs)
                    self._index_changed()
                elif old.level == ACTIVE:
                    self.retire(name)
        finally:
            self._hold_save -= 1
        self._publish()
        dprint(f"[adapter-pool] admission of {name}: {rep['level']}"
               + (f" ({rep['reason']})" if rep["reason"] else "")
               + (f", retired {victim}" if victim else ""))
        return rep

    # ------------------------------------------------------------ operator
    @_locked
    def offload(self, name: str) -> PoolEntry:
        e = self.get(name)
        self._move(e, DISK)
        self._publish()
        return e

    @_locked
    def retire(self, name: str) -> PoolEntry:
        e = self.get(name)
        e.level = RETIRED
        if self.index.remove(name):
            self._index_changed()
        self._move(e, DISK)
        self._publish()
        return e

    @_locked
    def reactivate(self, name: str) -> dict:
        return self.admit(name, self.get(name).path)

    @_locked
    def pin(self, name: str, pinned: bool = True) -> PoolEntry:
        e = self.get(name)
        e.pinned = bool(pinned)
        self._publish()
        return e

    @_locked
    def op(self, name: str, op: str):
        """Operator verbs of ``POST /adapters/{name}/{op}``."""
        if op in ("load", "prewarm"):
            return {"on_gpu": self.ensure_gpu(name)}
        if op in ("offload", "unload"):
            return self.describe(self.offload(name))
        if op in ("retire", "disable"):
            return self.describe(self.retire(name))
        if op in ("reactivate", "enable"):
            return self.reactivate(name)
        if op == "pin":
            return self.describe(self.pin(name, True))
        if op == "unpin":
            return self.describe(self.pin(name, False))
        if op == "remove":
            self.remove(name)
            return {"removed": name}
        raise ValueError(f"unknown adapter op '{op}' (load, prewarm, offload, retire, reactivate, "
                         f"pin, unpin, remove)")

    def describe(self, e: PoolEntry, now: float | None = None) -> dict:
        return {"name": e.name, "path": e.path, "job": e.job, "uid": e.uid, "level": e.level,
                "pinned": e.pinned, "tier": e.tier, "enabled": e.enabled, "hits": e.hits,
                "score": round(self.score_of(e, now), 4), "indexed": e.centroid is not None}

    @_locked
    def status(self) -> dict:
        now = self.clock()
        return {"capacity": self.capacity, "gpu_slots": self.gpu_slots,
                "active": len(self.active_names()), "retired": len(self.retired_names()),
                "version": self.version, "protected": sorted(self.protected_names(now)),
                "evictions": self.evictions, "cold_loads": self.cold_loads,
                "adapters": [self.describe(e, now) for e in sorted(self.entries.values(),
                                                                  key=lambda e: e.name)]}

    # ------------------------------------------------------------ persistence
    def _registry(self) -> dict:
        """The registry document: pool version, next id, the routable index
        file of this version, one record per adapter."""
        now = self.clock()
        recs = []
        for e in self.entries.values():
            rec = self.describe(e, now)
            rec["offloaded"] = e.tier == DISK
            recs.append(rec)
        return {"version": self.version, "next_uid": self._next_uid,
                "routable": f"routable-{self.version}.npz", "adapters": recs}

    @_locked
    def save(self, directory: str) -> None:
        """Write the routable index (a new versioned file whenever it changed)
        and then the registry, replaced in one rename: a reader sees either
        the previous pool or this one. Index files two versions old go."""
        os.makedirs(directory, exist_ok=True)
        if self._dirty or self.version == 0:
            self.version += 1
            self.index.save(os.path.join(directory, f"routable-{self.version}.npz"))
            self._dirty = False
        _write_json_atomic(os.path.join(directory, REGISTRY_FILE), self._registry())
        stale = [f for f in os.listdir(directory)
                 if (m := _ROUTABLE.fullmatch(f)) and int(m.group(1)) < self.version - 1]
        for f in stale:
            try:
                os.unlink(os.path.join(directory, f))
            except OSError:
                pass

    @_locked
    def restore(self, directory: str, centroids: CentroidIndex | None = None) -> int:
        """Bring back a saved pool: every adapter with its level, pin and id,
        loaded unless it was offloaded; centroids from ``centroids`` or the
        registry's routable index file. Returns the number of adapters."""
        reg = read_registry(directory)
        if reg is None:
            return 0
        if centroids is None:
            f = os.path.join(directory, reg.get("routable") or "")
            centroids = CentroidIndex.load_or_none(f) if reg.get("routable") else None
        self._hold_save += 1
        try:
            self.version = max(self.version, int(reg.get("version", 0)))
            for rec in reg["adapters"]:
                known = centroids is not None and rec["name"] in centroids
                cold = bool(rec.get("offloaded"))
                self.register(rec["name"], rec["path"],
                              centroids.centroid_of(rec["name"]) if known else None,
                              centroids.refs.get(rec["name"]) if known else None,
                              rec.get("job"), load=not cold, prewarm=not cold, level=rec.get("level", ACTIVE),
                              pinned=bool(rec.get("pinned")), uid=rec.get("uid"))
            self._next_uid = max(self._next_uid, int(reg.get("next_uid", 0)))
        finally:
            self._hold_save -= 1
        self._dirty = True
        self._publish()
        return len(reg["adapters"])


def _write_json_atomic(path: str, obj) -> None:
    """``obj`` as JSON at ``path``, replacing the old file in one rename."""
    tmp = f"{path}.tmp"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=1)
    os.replace(tmp, path)


def read_registry(directory: str) -> dict | None:
    """The registry of a pool directory (None when absent or unreadable)."""
    try:
        with open(os.path.join(directory, REGISTRY_FILE)) as f:
            reg = json.load(f)
    except (OSError, ValueError):
        return None
    ok = isinstance(reg, dict) and isinstance(reg.get("adapters"), list)
    return reg if ok else None
