"""The frame store with its LRU bookkeeping on the device (device_policy):
every decision equals KVManager's serial replay (cache/kv_cache.cpp:86-148,
via the oracle) and the host-policy store's, access for access, through
steps that evict frames touched again later in the same step (second
misses), steps that only hit (the recency log's head stays on old frames
until the log is compacted), empty steps and rejected steps; frames keep
their bytes through every move.
"""
import numpy as np
import pytest

import kvgen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-2
FB_PAGE = 2 * 1 * 16 * 128 * 2  # one 16-token page of one kv head, K and V, fp16


@pytest.fixture(scope="module")
def kvx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx as k
    return k


def _phases(U, n_max, steps, seed):
    """Access steps: Zipf(1.1) steps of random length, uniform steps (many
    second misses), hot steps over the frames of the step before (hits only),
    one empty step."""
    rng = np.random.default_rng(seed)
    perm = kvgen.permutation(seed + 1, U)
    out, prev = [], np.arange(8, dtype=np.int32)
    for s in range(steps):
        kind = (s // 6) % 3
        m = int(rng.integers(1, n_max + 1))
        if s == 5:
            ids = np.zeros(0, np.int32)
        elif kind == 0:
            ids = perm[kvgen.zipf_pages(seed * 1000 + s, m, U, 1.1)].astype(np.int32)
        elif kind == 1:
            ids = rng.integers(0, U, size=m).astype(np.int32)
        else:
            ids = prev[rng.integers(0, prev.size, size=m)].astype(np.int32)
        out.append(ids)
        if ids.size:
            prev = np.unique(ids)
    return out


def test_device_policy_equals_host_policy_and_replay(kvx, oracle):
    from kvx.tier import Tier
    U, C, S, N = 4000, 800, 640, 640
    FB = 1024
    raw = kvgen.randint(71, U * FB // 4, 0, 2**31 - 1).astype(np.int32).view(np.uint8).reshape(U, FB)
    ref = Tier(FB, U, C, S, device=0)
    dev = Tier(FB, U, C, S, device=0, device_policy=True, max_step=N)
    for f in range(U):
        ref.write_frame(f, raw[f])
        dev.write_frame(f, raw[f])
    steps = _phases(U, N, 48, 72)
    evs, hits = [], []
    for k, ids in enumerate(steps):
        s_ref, e_ref, h_ref, st_ref = ref.step(ids)
        s_dev, e_dev, h_dev, st_dev = dev.step(ids)
        assert np.array_equal(e_dev, e_ref), k
        assert np.array_equal(h_dev, h_ref), k
        assert np.array_equal(s_dev, s_ref), k  # same FIFO of free slots: same placement
        assert st_dev == st_ref, (k, st_dev, st_ref)
        if ids.size:  # a frame read twice in a step sits in one slot
            assert (s_dev >= 0).all() and (s_dev < C + S).all()
            first = {}
            for f, sl in zip(ids.tolist(), s_dev.tolist()):
                assert first.setdefault(f, sl) == sl, (k, f)
            assert len(set(first.values())) == len(first), k
        evs.append(e_dev)
        hits.append(h_dev)
    ref.sync()
    dev.sync()
    assert dev.totals() == ref.totals()
    tot = dev.totals()
    assert tot["reloads"] > 20 and tot["evictions"] > 1000, tot  # second misses exercised
    ids = np.concatenate([np.arange(C, dtype=np.int32)] + steps)
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    assert np.array_equal(np.concatenate(hits), want_hit[C:])
    for f in range(U):
        assert dev.location(f)[0] == ref.location(f)[0], f
        assert np.array_equal(dev.read_frame(f), raw[f]), f
    ref.close()
    dev.close()


def test_device_policy_compacts_its_log(kvx, oracle):
    """Hits only on a resident set that excludes the oldest frames: the
    recency log fills and is compacted many times; the next misses still
    evict exactly the replay's victims."""
    from kvx.tier import Tier
    U, C, S, N = 600, 200, 100, 100
    dev = Tier(256, U, C, S, device=0, device_policy=True, max_step=N)
    rng = np.random.default_rng(81)
    steps = [rng.integers(100, 200, size=N).astype(np.int32) for _ in range(40)]  # compacted several times
    steps += [rng.integers(0, U, size=int(rng.integers(1, N + 1))).astype(np.int32) for _ in range(30)]
    steps += [rng.integers(150, 200, size=N).astype(np.int32) for _ in range(20)]
    steps += [rng.integers(0, U, size=N).astype(np.int32) for _ in range(10)]
    evs, hits = [], []
    for ids in steps:
        _, ev, ht, _ = dev.step(ids)
        evs.append(ev)
        hits.append(ht)
    dev.sync()
    ids = np.concatenate([np.arange(C, dtype=np.int32)] + steps)
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    assert np.array_equal(np.concatenate(hits), want_hit[C:])
    dev.close()


def test_step_device_feeds_decode(kvx, oracle):
    """Steps on device arrays (ids uploaded on the caller's stream, slots
    consumed there by decode after wait_resident), no host round trip per
    step; decode over each step's frames matches the oracle and the
    decisions equal the replay."""
    from kvx.tier import Tier
    U, C, S, steps, per = 6000, 1500, 600, 12, 500
    data = kvgen.normal(91, (U, 2, 1, 16, 128)).astype(np.float16)
    raw = data.reshape(U, -1).view(np.uint8)
    t = Tier(FB_PAGE, U, C, S, device=0, device_policy=True, max_step=per)
    for f in range(U):
        t.write_frame(f, raw[f])
    ranks = kvgen.zipf_pages(92, steps * per, U, 1.1)
    stream = kvgen.permutation(93, U)[ranks].astype(np.int32).reshape(steps, per)
    q = kvgen.normal(94, (steps, 2, 3, 128))
    lens = torch.full((2,), 250 * 16, dtype=torch.int32, device="cuda")
    pinned = torch.from_numpy(stream).pin_memory()
    outs, evs, hits = [], [], []
    for s in range(steps):
        # the ids land late on the caller's (default) stream: a plan that did
        # not wait for that stream would read an unwritten buffer
        ids = torch.full((per,), -1, dtype=torch.int32, device="cuda")
        torch.cuda._sleep(2_000_000)
        ids.copy_(pinned[s], non_blocking=True)
        slots = torch.empty(per, dtype=torch.int32, device="cuda")
        ev = torch.empty(per, dtype=torch.int32, device="cuda")
        hit = torch.empty(per, dtype=torch.uint8, device="cuda")
        t.step_device(ids, slots, ev, hit)
        t.wait_resident()
        outs.append(kvx.decode(t.paged(1), slots.view(2, 250), lens, torch.from_numpy(q[s]).cuda()))
        t.mark_read()
        evs.append(ev)
        hits.append(hit)
    t.sync()
    torch.cuda.synchronize()
    for s in range(steps):
        ref = oracle.paged_decode(data, stream[s].reshape(2, 250), np.full(2, 4000, np.int32), q[s])
        got = outs[s].cpu().numpy()
        assert (np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max() <= 0, s
    ids = np.concatenate([np.arange(C, dtype=np.int32), stream.ravel()])
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(torch.cat(evs).cpu().numpy(), want_ev[C:])
    assert np.array_equal(torch.cat(hits).cpu().numpy(), want_hit[C:])
    for f in range(0, U, 7):
        assert np.array_equal(t.read_frame(f), raw[f]), f
    t.close()


def test_device_policy_rejects_bad_steps_and_changes_nothing(kvx, oracle):
    """An id out of range or more first-time loads than spare slots rejects
    the step on the device: kvx_tier_step returns the error (EINVAL /
    ENOSPC), kvx_tier_step_device reports it at kvx_tier_sync, and the store
    goes on exactly as if the step had not been made."""
    from kvx import KvxError
    from kvx.tier import Tier
    U, C, S, N = 1000, 300, 40, 200
    FB = 512
    raw = kvgen.randint(101, U * FB // 4, 0, 2**31 - 1).astype(np.int32).view(np.uint8).reshape(U, FB)
    t = Tier(FB, U, C, S, device=0, device_policy=True, max_step=N)
    for f in range(U):
        t.write_frame(f, raw[f])
    rng = np.random.default_rng(102)
    good = []

    def ok_step():
        # at most S frames outside the resident set: draw from the last step's frames plus a few new ones
        base = np.unique(good[-1]) if good else np.arange(C, dtype=np.int32)  # resident
        ids = np.concatenate([base[rng.integers(0, base.size, size=150)],
                              rng.integers(0, U, size=30)]).astype(np.int32)
        rng.shuffle(ids)
        t.step(ids)
        good.append(ids)

    for _ in range(5):
        ok_step()
    before = t.totals()
    with pytest.raises(KvxError) as e:
        t.step(np.array([3, 4, U], np.int32))
    assert e.value.status == -1
    with pytest.raises(KvxError) as e:  # 100 distinct frames nobody loaded recently: more than 40 spare slots
        far = np.setdiff1d(np.arange(C, U, dtype=np.int32), np.concatenate(good))[:100]
        t.step(far)
    assert e.value.status == -6
    assert t.totals() == before
    ids = torch.tensor([1, 2, U + 5], dtype=torch.int32, device="cuda")
    t.step_device(ids, torch.empty(3, dtype=torch.int32, device="cuda"))
    with pytest.raises(KvxError):
        t.sync()
    t.sync()  # the error is reported once
    assert t.totals() == before
    for _ in range(5):
        ok_step()
    evs, hits = [], []
    t2 = Tier(FB, U, C, S, device=0)  # host policy over the good steps only
    for ids in good:
        _, ev, ht, _ = t2.step(ids)
        evs.append(ev)
        hits.append(ht)
    t2.sync()
    assert t.totals() == t2.totals()
    for f in range(U):
        assert t.location(f)[0] == t2.location(f)[0], f
        assert np.array_equal(t.read_frame(f), raw[f]), f
    t.close()
    t2.close()


@pytest.mark.parametrize("device_policy", [False, True])
def test_plans_ahead_of_the_decode(kvx, oracle, device_policy):
    """lookahead 3: every step is planned (and its copies queued) four steps
    before the decode that reads it; wait_resident / mark_read address the
    oldest unmarked step.  Decode matches the oracle, decisions the replay,
    and both policies place every frame in the same slot."""
    from kvx.tier import Tier
    U, C, S, steps, per, L = 6000, 1500, 2400, 12, 500, 3
    data = kvgen.normal(111, (U, 2, 1, 16, 128)).astype(np.float16)
    raw = data.reshape(U, -1).view(np.uint8)
    kw = {"device_policy": True, "max_step": per} if device_policy else {}
    t = Tier(FB_PAGE, U, C, S, device=0, lookahead=L, **kw)
    for f in range(U):
        t.write_frame(f, raw[f])
    ranks = kvgen.zipf_pages(112, steps * per, U, 1.1)
    stream = kvgen.permutation(113, U)[ranks].astype(np.int32).reshape(steps, per)
    q = kvgen.normal(114, (steps, 2, 3, 128))
    lens = torch.full((2,), 250 * 16, dtype=torch.int32, device="cuda")
    slots = [torch.empty(per, dtype=torch.int32, device="cuda") for _ in range(steps)]
    ids_d = [torch.from_numpy(stream[s]).cuda() for s in range(steps)]  # alive until the plans read them
    host_slots = [None] * steps
    outs = [None] * steps
    for s in range(steps + L + 1):
        if s < steps:
            if device_policy:
                t.step_device(ids_d[s], slots[s])
            else:
                host_slots[s] = t.step(stream[s])[0].copy()
                slots[s].copy_(torch.from_numpy(host_slots[s]))
        j = s - L - 1
        if j >= 0:
            t.wait_resident()
            outs[j] = kvx.decode(t.paged(1), slots[j].view(2, 250), lens, torch.from_numpy(q[j]).cuda())
            t.mark_read()
    t.sync()
    torch.cuda.synchronize()
    for j in range(steps):
        ref = oracle.paged_decode(data, stream[j].reshape(2, 250), np.full(2, 4000, np.int32), q[j])
        got = outs[j].cpu().numpy()
        assert (np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max() <= 0, j
    for f in range(0, U, 5):
        assert np.array_equal(t.read_frame(f), raw[f]), f
    # the placement equals a bookkeeping-only host store's with the same lookahead
    b = Tier(FB_PAGE, U, C, S, device=-1, lookahead=L)
    for s in range(steps):
        if s - L - 1 >= 0:
            b.mark_read()
        want = b.step(stream[s])[0]
        assert np.array_equal(slots[s].cpu().numpy(), want), s
    t.close()
