"""The adapter pool's policies against a fake backend: the order of tier
moves the backend sees, protection and in-use rules of GPU slot eviction,
the three full-pool policies, re-admission of a new version, operator verbs
and aliases, and a registry round trip with ids and pins."""
import numpy as np
import pytest

from deltaserve_vllm_b200.adapters.routing.index import l2_normalize
from deltaserve_vllm_b200.adapters.routing.pool import (ACTIVE, CPU, DISK, GPU, RETIRED, AdapterPool, PoolFull,
                                                        read_registry)


class Backend:
    def __init__(self):
        self.calls = []

    def load(self, e):
        self.calls.append(("load", e.name))

    def activate(self, e):
        self.calls.append(("activate", e.name))

    def deactivate(self, e):
        self.calls.append(("deactivate", e.name))

    def unload(self, e):
        self.calls.append(("unload", e.name))


class Clock:
    t = 0.0

    def __call__(self):
        return self.t


def _cent(i, dim=16):
    v = np.zeros(dim)
    v[i] = 1.0
    return l2_normalize(v + 0.01)


def test_tier_walks_one_step_at_a_time():
    be = Backend()
    pool = AdapterPool(be, gpu_slots=1)
    pool.register("a", "/a", load=False)
    assert pool.entries["a"].tier == DISK and be.calls == []
    assert pool.ensure_gpu("a")
    assert be.calls == [("load", "a"), ("activate", "a")]
    pool.offload("a")
    assert be.calls[2:] == [("deactivate", "a"), ("unload", "a")] and pool.entries["a"].tier == DISK


def test_eviction_respects_protection_and_use():
    clk = Clock()
    pool = AdapterPool(Backend(), gpu_slots=2, protected=1, half_life_s=10.0, clock=clk)
    for n in "abc":
        pool.register(n, f"/{n}")                  # a and b get the free slots, c stays on the host
    assert [pool.entries[n].tier for n in "abc"] == [GPU, GPU, CPU]
    for _ in range(2):
        pool.note_hit("b", place=False)
    assert pool.protected_names() == {"b"}
    assert not pool.ensure_gpu("c", in_use={"a"})   # a is used, b is protected
    assert pool.entries["c"].tier == CPU and pool.evictions == 0
    assert pool.ensure_gpu("c")                     # a is free now: it goes
    assert pool.entries["a"].tier == CPU and pool.evictions == 1
    clk.t = 100.0                                   # b's hits decayed below c's fresh one
    pool.note_hit("c", place=False)
    assert pool.protected_names() == {"c"}
    assert pool.score_of(pool.entries["b"]) == pytest.approx(2 * 0.5 ** 10)


@pytest.mark.parametrize("policy", ["retire_least_used", "admit_retired", "reject"])
def test_full_pool_policies(policy):
    clk = Clock()
    pool = AdapterPool(Backend(), capacity=2, clock=clk, when_full=policy, grace_s=0.0)
    pool.admit("a", "/a", _cent(0))
    pool.admit("b", "/b", _cent(1))
    pool.note_hit("b")
    if policy == "reject":
        with pytest.raises(PoolFull):
            pool.admit("c", "/c", _cent(2))
        return
    rep = pool.admit("c", "/c", _cent(2))
    if policy == "retire_least_used":
        assert rep["level"] == ACTIVE and rep["retired"] == "a"     # a has no hits
        assert pool.entries["a"].level == RETIRED and "a" not in pool.routable_names()
    else:
        assert rep["level"] == RETIRED and rep["reason"] == "active set is full"
        assert sorted(pool.routable_names()) == ["a", "b"]


def test_pinned_and_grace_are_never_retired():
    clk = Clock()
    pool = AdapterPool(Backend(), capacity=2, clock=clk, grace_s=10.0)
    pool.admit("a", "/a", _cent(0), pinned=True)
    pool.admit("b", "/b", _cent(1))
    clk.t = 5.0
    rep = pool.admit("c", "/c", _cent(2))          # b is still in its grace period, a is pinned
    assert rep["level"] == RETIRED and rep["retired"] is None
    clk.t = 20.0
    rep = pool.admit("d", "/d", _cent(3))
    assert rep["level"] == ACTIVE and rep["retired"] == "b"


def test_new_version_gets_a_new_id_and_leaves_the_gpu():
    be = Backend()
    pool = AdapterPool(be, gpu_slots=1)
    pool.admit("a", "/a/v1", _cent(0), load=True, prewarm=True)
    uid = pool.entries["a"].uid
    assert pool.entries["a"].tier == GPU
    pool.admit("a", "/a/v2", _cent(0))
    e = pool.entries["a"]
    assert e.path == "/a/v2" and e.uid != uid and e.tier == DISK and e.level == ACTIVE
    assert pool.ensure_gpu("a") and be.calls[-2:] == [("load", "a"), ("activate", "a")]


def test_operator_verbs_and_aliases():
    pool = AdapterPool(Backend(), gpu_slots=1)
    pool.admit("a", "/a", _cent(0))
    assert pool.op("a", "prewarm") == {"on_gpu": True}
    assert pool.op("a", "disable")["level"] == RETIRED and "a" not in pool.routable_names()
    assert pool.op("a", "enable")["level"] == ACTIVE and "a" in pool.routable_names()
    assert pool.op("a", "pin")["pinned"] and not pool.op("a", "unpin")["pinned"]
    assert pool.op("a", "unload")["tier"] == DISK
    assert pool.op("a", "remove") == {"removed": "a"} and "a" not in pool
    with pytest.raises(ValueError, match="unknown adapter op"):
        pool.op("b", "explode")


def test_registry_round_trip(tmp_path):
    clk = Clock()
    d = str(tmp_path)
    pool = AdapterPool(Backend(), capacity=3, gpu_slots=1, clock=clk, directory=d)
    for i, n in enumerate("abc"):
        pool.admit(n, f"/{n}", _cent(i), load=True)
    pool.retire("b")
    pool.pin("c")
    pool.offload("a")
    reg = read_registry(d)
    assert reg["layout"] == "dsv-adapter-pool/2" and (tmp_path / reg["index_file"]).exists()
    back = AdapterPool(Backend(), capacity=3, gpu_slots=1, clock=clk, directory=d)
    assert back.restore(d) == 3
    assert {n: back.entries[n].uid for n in "abc"} == {n: pool.entries[n].uid for n in "abc"}
    assert back.entries["b"].level == RETIRED and back.entries["c"].pinned
    assert back.entries["a"].tier == DISK and back.entries["c"].tier in (CPU, GPU)
    assert sorted(back.routable_names()) == ["a", "c"]
    np.testing.assert_allclose(back.index.centroid_of("c"), pool.index.centroid_of("c"))
    # only this revision's and the previous revision's index files remain
    assert len(list(tmp_path.glob("index-*.npz"))) <= 2
    (tmp_path / "pool.json").write_text('{"adapters": []}')        # another layout: not restored
    assert AdapterPool(Backend(), directory=None).restore(d) == 0
