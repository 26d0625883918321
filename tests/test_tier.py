"""The tiered frame store's policy and slot bookkeeping, on the CPU
(bookkeeping-only stores: no device memory, no copies).

Residency decisions must equal, access for access, a serial replay of the
same id stream through KVManager's LRU (cache/kv_cache.cpp:86-148: a hit
moves the page to the front; a miss evicts lru_.back() when size >=
capacity, then inserts at the front) -- here the oracle's restatement, whose
own parity with the compiled reference is pinned by the lru golden fixture.
The store starts with frames 0..capacity-1 resident in that order, so the
replay is fed that prefix first.
"""
import numpy as np
import pytest

import kvgen

from kvx import KvxError
from kvx.tier import Tier, lib


def zipf_stream(seed, steps, per_step, universe):
    ranks = kvgen.zipf_pages(seed, steps * per_step, universe, 1.1)
    perm = kvgen.permutation(seed + 1, universe)  # hot ranks scattered over the ids
    return perm[ranks].astype(np.int32).reshape(steps, per_step)


def check_slots(t, universe):
    dev, host = {}, {}
    for f in range(universe):
        tier, slot = t.location(f)
        d = dev if tier == "device" else host
        assert slot not in d, (tier, slot)
        d[slot] = f
    return dev, host


@pytest.mark.parametrize("universe,capacity,spare,per_step", [(3000, 900, 300, 250), (1200, 1500, 10, 100),
                                                                 (5000, 400, 200, 150)])
def test_policy_matches_kvmanager_replay(oracle, universe, capacity, spare, per_step):
    t = Tier(4096, universe, capacity, spare, device=-1)
    stream = zipf_stream(7 + universe, 24, per_step, universe)
    got_ev, got_hit = [], []
    for s in range(stream.shape[0]):
        slots, ev, hit, st = t.step(stream[s])
        got_ev.append(ev)
        got_hit.append(hit)
        assert st["hits"] + st["misses"] == per_step
        assert st["frames_h2d"] + st["reloads"] == st["misses"]
        for f in set(stream[s].tolist()):  # every frame of the step ends on the device
            assert t.location(f)[0] == "device"
    ids = np.concatenate([np.arange(min(capacity, universe), dtype=np.int32), stream.ravel()])
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), capacity)
    k = min(capacity, universe)
    assert np.array_equal(np.concatenate(got_hit), want_hit[k:])
    assert np.array_equal(np.concatenate(got_ev), want_ev[k:])
    dev, host = check_slots(t, universe)
    assert len(dev) == min(capacity, universe) and len(dev) + len(host) == universe
    tot = t.totals()
    assert tot["accesses"] == stream.size and tot["evictions"] == int((np.concatenate(got_ev) >= 0).sum())


def test_slots_within_a_step_are_stable_and_distinct():
    universe, capacity = 2000, 600
    t = Tier(4096, universe, capacity, 200, device=-1)
    stream = zipf_stream(3, 10, 400, universe)
    for s in range(stream.shape[0]):
        slots, ev, hit, st = t.step(stream[s])
        seen = {}
        for f, sl in zip(stream[s].tolist(), slots.tolist()):
            assert 0 <= sl < capacity + 200
            assert seen.setdefault(f, sl) == sl  # a frame keeps one slot for the whole step
        assert len(set(seen.values())) == len(seen)  # distinct frames, distinct slots
        for f, sl in seen.items():
            assert t.location(f) == ("device", sl)


def test_reload_within_a_step_keeps_slot_and_counts_miss(oracle):
    # capacity 4: frames 0..3 resident, 0 least recent
    t = Tier(64, 10, 4, 4, device=-1)
    slot0 = t.location(0)[1]
    # 5 evicts 0, then 0 comes back in the same step (evicting 1)
    slots, ev, hit, st = t.step(np.array([5, 0], np.int32))
    assert ev.tolist() == [0, 1] and hit.tolist() == [0, 0]
    assert st["reloads"] == 1 and st["frames_h2d"] == 1 and st["frames_d2h"] == 1
    assert slots[1] == slot0  # no bytes moved for frame 0
    ids = np.array([0, 1, 2, 3, 5, 0], np.int32)
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(6, np.uint8), 4)
    assert want_ev[4:].tolist() == [0, 1] and want_hit[4:].tolist() == [0, 0]


def test_errors_leave_the_store_unchanged():
    t = Tier(64, 100, 20, 3, device=-1)
    with pytest.raises(KvxError) as e:
        t.step(np.array([1, 200], np.int32))  # id outside the universe
    assert e.value.status == -1
    with pytest.raises(KvxError) as e:
        t.step(np.arange(20, dtype=np.int32))  # a step must be shorter than the capacity
    assert e.value.status == -1
    with pytest.raises(KvxError) as e:
        t.step(np.array([50, 51, 52, 53], np.int32))  # 4 loads, 3 spare slots
    assert e.value.status == -6
    assert t.totals()["accesses"] == 0
    assert t.location(50) == ("host", 30)
    slots, ev, hit, st = t.step(np.array([50, 51, 52], np.int32))
    assert st["misses"] == 3 and ev.tolist() == [0, 1, 2]
    with pytest.raises(KvxError):
        Tier(60, 100, 20, 3, device=-1)  # frame bytes not a multiple of 16


def test_disk_tier_policy_and_placement(oracle):
    """With a RAM tier smaller than the non-resident frames, the rest live on
    disk; device decisions stay KVManager's LRU, RAM never holds more than its
    size at a step boundary, and RAM evicts in arrival order."""
    universe, capacity, spare, host = 4000, 900, 200, 800
    t = Tier(4096, universe, capacity, spare, device=-1, host_frames=host, spill_path="unused")
    assert t.location(capacity) == ("host", 0) and t.location(capacity + host) == ("disk", capacity + host)
    stream = zipf_stream(29, 20, 250, universe)
    evs = []
    for s in range(stream.shape[0]):
        slots, ev, hit, st = t.step(stream[s])
        evs.append(ev)
        tiers = [t.location(f)[0] for f in range(universe)]
        assert tiers.count("device") == capacity and tiers.count("host") <= host
        for f in set(stream[s].tolist()):
            assert t.location(f)[0] == "device"
    ids = np.concatenate([np.arange(capacity, dtype=np.int32), stream.ravel()])
    want_ev, _ = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), capacity)
    assert np.array_equal(np.concatenate(evs), want_ev[capacity:])
    tot = t.totals()
    assert tot["frames_disk_read"] > 0 and tot["frames_disk_write"] > 0
    with pytest.raises(KvxError):
        Tier(4096, universe, capacity, spare, device=-1, host_frames=3 * spare - 1, spill_path="x")


def test_device_policy_config_is_checked():
    """device_policy stores keep their bookkeeping on a device: a
    bookkeeping-only store, a disk tier, a step bound of capacity or more
    and a universe that fits the device are refused before any device is
    touched; the device-array step is refused on a host-policy store."""
    for kw in ({"device": -1, "max_step": 10}, {"device": 0, "max_step": 0}, {"device": 0, "max_step": 20},
               {"device": 0, "max_step": 10, "host_frames": 40, "spill_path": "/nonexistent/x"}):
        with pytest.raises(KvxError) as e:
            Tier(64, 100, 20, 3, device_policy=True, **kw)
        assert e.value.status == -1, kw
    with pytest.raises(KvxError) as e:
        Tier(64, 20, 20, 3, device=0, device_policy=True, max_step=10)  # everything resident
    assert e.value.status == -1
    t = Tier(64, 100, 20, 3, device=-1)
    assert lib.kvx_tier_step_device(t.h, None, 0, None, None, None, None) == -4
    import ctypes
    st = ctypes.c_void_p()
    assert lib.kvx_tier_plan_stream(t.h, ctypes.byref(st)) == -4  # host-policy store: no plan stream
    with pytest.raises(KvxError):
        Tier(64, 100, 20, 3, device=-1, lookahead=63)  # lookahead 0..62


def test_lookahead_contract_and_slot_quarantine(oracle):
    """With lookahead L a step may be planned while the reads of the last
    L+1 steps are unmarked (one more: KVX_EBUSY); a device slot freed by a
    victim is not loaded again within L+1 steps (too few older free slots:
    KVX_ENOSPC, nothing changed); decisions stay KVManager's."""
    t = Tier(64, 100, 20, 3, device=-1, lookahead=1)
    t.step(np.array([30, 31, 32], np.int32))      # step 0: 3 loads into the 3 spare slots
    with pytest.raises(KvxError) as e:             # step 1: the only free slots were freed at step 0
        t.step(np.array([33], np.int32))
    assert e.value.status == -6
    t.step(np.array([30, 31], np.int32))           # step 1: hits need no slot
    t.step(np.array([30], np.int32))               # step 2: three steps unmarked at L = 1
    with pytest.raises(KvxError) as e:             # step 3 needs step 0's reads marked
        t.step(np.array([33], np.int32))
    assert e.value.status == -2
    t.mark_read()                                  # step 0
    _, ev, _, _ = t.step(np.array([33], np.int32))  # step 3: slots freed at step 0 are old enough
    assert ev.tolist() == [3]
    for _ in range(3):
        t.mark_read()
    with pytest.raises(KvxError) as e:             # every planned step is marked
        t.mark_read()
    assert e.value.status == -1
    ids = np.concatenate([np.arange(20, dtype=np.int32), [30, 31, 32, 30, 31, 30, 33]]).astype(np.int32)
    want_ev, _ = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), 20)
    assert want_ev[20:].tolist() == [0, 1, 2, -1, -1, -1, 3]


@pytest.mark.parametrize("lookahead", [0, 2, 5])
def test_lookahead_never_loads_into_a_slot_read_since(oracle, lookahead):
    """Zipf steps planned `lookahead` steps ahead of their (marked) reads: a
    slot loaded at step s was read by none of steps s-L-1 .. s-1, and the
    decisions equal the replay."""
    U, C, S, per, steps = 3000, 600, 400, 60, 80
    t = Tier(64, U, C, S, device=-1, lookahead=lookahead)
    ranks = kvgen.zipf_pages(61, steps * per, U, 0.9)
    stream = kvgen.permutation(62, U)[ranks].astype(np.int32).reshape(steps, per)
    slots, evs, hits = [], [], []
    for s in range(steps):
        if lookahead and s - lookahead - 1 > 0:
            t.mark_read()  # the reads of step s-L-2
        sl, ev, ht, _ = t.step(stream[s])
        slots.append(sl.copy())
        evs.append(ev)
        hits.append(ht)
        # slots written by this step's loads: misses of frames not evicted
        # earlier in the step (a second miss keeps its slot, no load)
        victims = set(ev[ev >= 0].tolist())
        loaded = {int(x) for x, h, f in zip(sl, ht, stream[s]) if h == 0 and int(f) not in victims}
        for j in range(max(0, s - lookahead - 1), s):
            assert not loaded & set(slots[j].tolist()), (s, j)
    ids = np.concatenate([np.arange(C, dtype=np.int32), stream.ravel()])
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    assert np.array_equal(np.concatenate(hits), want_hit[C:])
