"""The device plan of the frame store (csrc/kvx_tier_dev.cu), restated
serially and checked against KVManager's LRU replay (cache/kv_cache.cpp:
86-148, via the oracle) on CPU.

The restatement follows the kernels step for step with the same state:
stamps and a recency log (an entry is current while its frame's stamp
equals its position), first touches, the misses of non-resident frames in
time order, the merge of misses with the log's candidates from the head
(windows of 2,048 positions holding only current entries not touched
before the pending miss; zip runs of untouched candidates cut at the
earliest pending second miss; the rest one miss at a time, second misses
of evicted frames through a min-heap), slots from a FIFO of free device
slots that a load takes only once they are L+1 steps old, write-backs onto
a stack of free host slots, and the log's compaction when it nears
W = 4 capacity + 2 max_step.  The GPU tests (test_gpu_tier_policy.py)
check the kernels against the host-policy store; this file checks the
design itself, quickly and without a GPU.
"""
import heapq

import numpy as np
import pytest

import kvgen

INT_MAX = 2**31 - 1
WIN = 2048


class DevicePlan:
    def __init__(self, U, C, S, max_n, lookahead=0):
        self.U, self.C, self.max_n, self.L = U, C, max_n, lookahead
        self.W = 4 * C + 2 * max_n
        r0 = min(U, C)
        ids = np.arange(U)
        self.stamp = np.where(ids < r0, ids, -1).astype(np.int64)
        self.dslot = np.where(ids < r0, ids, -1)
        self.hslot = np.where(ids >= r0, ids - r0, -1)
        self.first = np.full(U, INT_MAX, np.int64)
        self.evict_ev = np.full(U, -1)
        self.log = np.zeros(self.W, np.int64)
        self.log[:r0] = ids[:r0]
        self.dev_free = list(range(r0, C + S))            # FIFO
        self.freed_at = {d: -(1 << 62) for d in range(C + S)}
        self.host_free = [U - r0 + S - 1 - h for h in range(S)]  # stack, popped from the end
        self.head, self.base, self.resident, self.step_no = 0, r0, r0, 0
        self.devmem = np.full(C + S, -1)
        self.devmem[:r0] = ids[:r0]
        self.hostmem = np.full(U - r0 + S, -1)
        self.hostmem[:U - r0] = ids[r0:]
        self.zips = self.compactions = 0

    def merge(self, m0, base):
        room, heap, ev_t, ev_v = self.C - self.resident, [], [], []
        p0 = ci = tp = 0
        cand, tl = [], []  # the window's candidates (frame, first touch, offset); touched ones' indices
        fill = fill_end = self.head

        def rec(t, v):
            if v >= 0:
                self.stamp[v] = -1
                self.evict_ev[v] = len(ev_t)
            ev_t.append(t)
            ev_v.append(v)

        while True:
            act, run, tn = "done", 0, INT_MAX
            while True:
                tm = m0[p0] if p0 < len(m0) else INT_MAX
                htop = heap[0] if heap else INT_MAX
                tn = min(tm, htop)
                if tn == INT_MAX:
                    break
                if room > 0 and not heap:
                    act, run = "room", min(room, len(m0) - p0)
                    break
                if room <= 0:
                    while ci < len(cand) and cand[ci][1] < tn:
                        ci += 1
                    if ci == len(cand):
                        act = "refill"
                        break
                    if cand[ci][1] == INT_MAX and tm < htop:
                        while tp < len(tl) and tl[tp] < ci:
                            tp += 1
                        run = min((tl[tp] if tp < len(tl) else len(cand)) - ci, len(m0) - p0)
                        if heap:
                            run = min(run, 1024)
                        if run >= 8:
                            act = "zip"
                            break
                if tm < htop:
                    t, p0 = tm, p0 + 1
                else:
                    t = heapq.heappop(heap)
                v = -1
                if room > 0:
                    room -= 1
                else:
                    v, tau, _ = cand[ci]
                    ci += 1
                    if tau != INT_MAX:  # touched later: misses again then
                        heapq.heappush(heap, tau)
                rec(t, v)
            if act == "done":
                break
            if act in ("zip", "room"):
                if act == "zip" and heap:  # only the misses before the pending second miss
                    run = sum(1 for i in range(run) if m0[p0 + i] < heap[0])
                self.zips += act == "zip"
                for i in range(run):
                    rec(m0[p0 + i], cand[ci + i][0] if act == "zip" else -1)
                p0 += run
                if act == "zip":
                    ci += run
                else:
                    room -= run
                continue
            h, end = fill_end, min(fill_end + WIN, base)
            assert h < end, "no candidate left"
            cand, tl = [], []
            for pos in range(h, end):
                c = int(self.log[pos % self.W])
                if self.stamp[c] == pos and self.first[c] >= tn:
                    if self.first[c] != INT_MAX:
                        tl.append(len(cand))
                    cand.append((c, int(self.first[c]), pos - h))
            fill, fill_end, ci, tp = h, end, 0, 0
        self.head = fill + cand[ci][2] if ci < len(cand) else fill_end
        return ev_t, ev_v

    def step(self, frames):
        n = len(frames)
        for i, f in enumerate(frames):
            self.first[f] = min(self.first[f], i)
        m0 = [i for i, f in enumerate(frames) if self.first[f] == i and self.stamp[f] < 0]
        ok = len(m0) <= len(self.dev_free) and len(m0) <= len(self.host_free) and (
            not m0 or self.freed_at[self.dev_free[len(m0) - 1]] <= self.step_no - self.L - 1)
        if not ok:  # rejected: nothing changes
            for f in frames:
                self.first[f] = INT_MAX
            raise RuntimeError("ENOSPC")
        base = self.base
        ev_t, ev_v = self.merge(m0, base)
        loads, wbs = [], []
        for k, t in enumerate(ev_t):
            f, v = frames[t], ev_v[k]
            if self.evict_ev[f] < 0:  # not evicted earlier in the step
                ds = self.dev_free[len(loads)]
                loads.append((ds, self.hslot[f]))
                self.dslot[f], self.hslot[f] = ds, -1
            if v >= 0 and self.first[v] == INT_MAX:  # not touched again in the step
                hs = self.host_free[len(self.host_free) - 1 - len(wbs)]
                wbs.append((self.dslot[v], hs))
                self.hslot[v], self.dslot[v] = hs, -1
        for ds, hs in wbs:
            self.hostmem[hs] = self.devmem[ds]
        for ds, hs in loads:
            self.devmem[ds] = self.hostmem[hs]
        ev_of = {t: k for k, t in enumerate(ev_t)}
        slots = np.array([self.dslot[f] for f in frames])
        hit = np.array([0 if i in ev_of else 1 for i in range(n)], np.uint8)
        evicted = np.array([ev_v[ev_of[i]] if i in ev_of else -1 for i in range(n)])
        for i, f in enumerate(frames):
            self.stamp[f] = max(self.stamp[f], base + i)
            self.log[(base + i) % self.W] = f
        for f in frames:
            self.first[f] = INT_MAX
        for v in ev_v:
            if v >= 0:
                self.evict_ev[v] = -1
        self.dev_free = self.dev_free[len(loads):] + [d for d, _ in wbs]
        for d, _ in wbs:
            self.freed_at[d] = self.step_no
        self.host_free = self.host_free[:len(self.host_free) - len(wbs)] + [h for _, h in loads]
        self.resident += len(ev_t) - sum(v >= 0 for v in ev_v)
        self.base += n
        self.step_no += 1
        if self.base + self.max_n - self.head > self.W:
            cur = [int(self.log[p % self.W]) for p in range(self.head, self.base)
                   if self.stamp[self.log[p % self.W]] == p]
            assert len(cur) == self.resident <= self.C
            for i, c in enumerate(cur):
                self.log[i], self.stamp[c] = c, i
            self.head, self.base = 0, len(cur)
            self.compactions += 1
        return slots, evicted, hit

    def check_bytes(self):
        for f in range(self.U):
            if self.stamp[f] >= 0:
                assert self.dslot[f] >= 0 and self.devmem[self.dslot[f]] == f, f
            else:
                assert self.hslot[f] >= 0 and self.hostmem[self.hslot[f]] == f, f


def _replay_check(oracle, C, steps, evs, hits):
    ids = np.concatenate([np.arange(C, dtype=np.int32)] + [np.asarray(s, np.int32) for s in steps])
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    assert np.array_equal(np.concatenate(hits), want_hit[C:])


@pytest.mark.parametrize("U,C,S,n,steps,zipf", [(400, 64, 63, 63, 120, 0.3), (3000, 800, 640, 640, 30, 1.1),
                                                (3000, 2000, 1900, 1999, 12, 0.5), (70, 60, 59, 59, 60, 0.2)])
def test_device_plan_equals_kvmanager_replay(oracle, U, C, S, n, steps, zipf):
    rng = np.random.default_rng(U + n)
    p = DevicePlan(U, C, S, n)
    perm = kvgen.permutation(U, U)
    done, evs, hits = [], [], []
    for s in range(steps):
        ids = perm[kvgen.zipf_pages(1000 * U + s, int(rng.integers(1, n + 1)), U, zipf)].astype(np.int32)
        _, ev, ht = p.step(ids)
        done.append(ids)
        evs.append(ev)
        hits.append(ht)
    p.check_bytes()
    _replay_check(oracle, C, done, evs, hits)


def test_device_plan_zips_and_compacts(oracle):
    """Hit-only steps on part of the resident set keep the log's head on old
    frames until the log is compacted; uniform steps evict frames touched
    again later in the same step (second misses through the heap) and zip
    most other misses."""
    U, C, S, n = 600, 200, 100, 100
    p = DevicePlan(U, C, S, n)
    rng = np.random.default_rng(81)
    steps = [rng.integers(100, 200, size=n) for _ in range(40)]
    steps += [rng.integers(0, U, size=int(rng.integers(1, n + 1))) for _ in range(30)]
    steps += [rng.integers(0, U, size=n) for _ in range(20)]
    evs, hits = [], []
    for ids in steps:
        _, ev, ht = p.step(ids.astype(np.int32))
        evs.append(ev)
        hits.append(ht)
    assert p.compactions >= 3 and p.zips > 0
    p.check_bytes()
    _replay_check(oracle, C, steps, evs, hits)


def test_device_plan_lookahead_delays_slot_reuse(oracle):
    """With lookahead L a load takes only device slots freed L+1 or more
    steps earlier: no slot read in the last L+1 steps is written, a step
    that would need a younger slot is rejected whole, and the decisions stay
    KVManager's."""
    U, C, S, n, L = 2000, 400, 160, 40, 3
    p = DevicePlan(U, C, S, n, lookahead=L)
    rng = np.random.default_rng(7)
    done, evs, hits, reads = [], [], [], []
    for s in range(80):
        ids = rng.integers(0, U, size=n).astype(np.int32)
        slots, ev, ht = p.step(ids)
        victims = set(ev[ev >= 0].tolist())
        loaded = {int(x) for x, h, f in zip(slots, ht, ids) if h == 0 and int(f) not in victims}
        for j in range(max(0, s - L - 1), s):
            assert not loaded & reads[j], (s, j)
        reads.append(set(slots.tolist()))
        done.append(ids)
        evs.append(ev)
        hits.append(ht)
    _replay_check(oracle, C, done, evs, hits)
    tight = DevicePlan(U, C, 4, n, lookahead=L)  # 4 spare slots: the second miss-heavy step must wait
    tight.step(np.array([1000, 1001, 1002, 1003], np.int32))
    with pytest.raises(RuntimeError):
        tight.step(np.array([1004], np.int32))
