"""The tiered frame store on the GPU: frames keep their bytes through any
number of evictions and loads, decode reads them while later steps' copies
run, and the residency decisions equal KVManager's LRU replay
(cache/kv_cache.cpp:86-148, via the oracle).

Frames here are pages of one kv head ([2][1][16][128] fp16, 8 KiB); each
step is one decode of 2 sequences x 250 pages whose page ids are the step's
Zipf(1.1) accesses, checked against the oracle's paged decode over the
frames laid out by id.
"""
import numpy as np
import pytest

import kvgen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-2
FB = 2 * 1 * 16 * 128 * 2


@pytest.fixture(scope="module")
def kvx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx as k
    return k


def test_tier_moves_bytes_exactly_and_decode_sees_them(kvx, oracle):
    from kvx.tier import Tier
    U, C, S, steps, per = 6000, 1500, 600, 12, 500
    data = kvgen.normal(41, (U, 2, 1, 16, 128)).astype(np.float16)
    t = Tier(FB, U, C, S, device=0)
    dev = t.device_tensor()
    dev[:C * FB] = torch.from_numpy(data[:C].reshape(-1).view(np.uint8)).cuda()
    t.host_array()[:(U - C) * FB] = data[C:].reshape(-1).view(np.uint8)
    torch.cuda.synchronize()
    ranks = kvgen.zipf_pages(42, steps * per, U, 1.1)
    stream = kvgen.permutation(43, U)[ranks].astype(np.int32).reshape(steps, per)
    q = kvgen.normal(44, (steps, 2, 3, 128))
    lens = torch.full((2,), 250 * 16, dtype=torch.int32, device="cuda")
    outs, evs, hits = [], [], []
    for s in range(steps):
        slots, ev, hit, st = t.step(stream[s])
        evs.append(ev)
        hits.append(hit)
        t.wait_resident()
        bt = torch.from_numpy(slots.reshape(2, 250)).cuda()
        outs.append(kvx.decode(t.paged(1), bt, lens, torch.from_numpy(q[s]).cuda()))
        t.mark_read()
    t.sync()
    torch.cuda.synchronize()
    for s in range(steps):
        ref = oracle.paged_decode(data, stream[s].reshape(2, 250), np.full(2, 4000, np.int32), q[s])
        got = outs[s].cpu().numpy()
        assert (np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max() <= 0, s
    # every frame's bytes where the store says it is
    devb = dev.cpu().numpy()
    hostb = t.host_array()
    raw = data.reshape(U, -1).view(np.uint8)
    for f in range(U):
        tier, slot = t.location(f)
        src = devb if tier == "device" else hostb
        assert np.array_equal(src[slot * FB:(slot + 1) * FB], raw[f]), (f, tier, slot)
    ids = np.concatenate([np.arange(C, dtype=np.int32), stream.ravel()])
    want_ev, want_hit = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    assert np.array_equal(np.concatenate(hits), want_hit[C:])
    tot = t.totals()
    assert tot["frames_h2d"] > 0 and tot["frames_d2h"] > 0
    t.close()


def test_tier_with_disk_keeps_bytes_through_three_tiers(kvx, oracle, tmp_path):
    """RAM tier smaller than the non-resident frames: frames go GPU -> RAM ->
    disk and back; every frame keeps its bytes, decode over each step's
    frames matches the oracle, decisions equal KVManager's LRU."""
    from kvx.tier import Tier
    U, C, S, H, steps, per = 6000, 1500, 600, 2000, 10, 500
    data = kvgen.normal(51, (U, 2, 1, 16, 128)).astype(np.float16)
    raw = data.reshape(U, -1).view(np.uint8)
    t = Tier(FB, U, C, S, device=0, host_frames=H, spill_path=tmp_path / "spill.bin")
    assert t.location(C + H) == ("disk", C + H)
    for f in range(U):
        t.write_frame(f, raw[f])
    ranks = kvgen.zipf_pages(52, steps * per, U, 1.1)
    stream = kvgen.permutation(53, U)[ranks].astype(np.int32).reshape(steps, per)
    q = kvgen.normal(54, (steps, 2, 3, 128))
    lens = torch.full((2,), 250 * 16, dtype=torch.int32, device="cuda")
    outs, evs = [], []
    for s in range(steps):
        slots, ev, hit, st = t.step(stream[s])
        evs.append(ev)
        t.wait_resident()
        outs.append(kvx.decode(t.paged(1), torch.from_numpy(slots.reshape(2, 250)).cuda(), lens,
                               torch.from_numpy(q[s]).cuda()))
        t.mark_read()
    t.sync()
    torch.cuda.synchronize()
    for s in range(steps):
        ref = oracle.paged_decode(data, stream[s].reshape(2, 250), np.full(2, 4000, np.int32), q[s])
        got = outs[s].cpu().numpy()
        assert (np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))).max() <= 0, s
    tiers = {"device": 0, "host": 0, "disk": 0}
    for f in range(U):
        tiers[t.location(f)[0]] += 1
        assert np.array_equal(t.read_frame(f), raw[f]), f
    assert tiers["device"] == C and tiers["host"] <= H and tiers["disk"] > 0
    ids = np.concatenate([np.arange(C, dtype=np.int32), stream.ravel()])
    want_ev, _ = oracle.lru_replay(ids, np.zeros(ids.size, np.uint8), C)
    assert np.array_equal(np.concatenate(evs), want_ev[C:])
    tot = t.totals()
    assert tot["frames_disk_read"] > 0 and tot["frames_disk_write"] > 0
    t.close()
