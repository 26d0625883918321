"""The engine's tiers and decode step, checked bit for bit where the data is
only moved and against the oracle where it is computed.

- GPU -> RAM -> GPU and GPU -> file -> GPU preserve every byte.
- GPU -> int8 -> GPU equals the oracle's KVCompressionEngine round trip
  (compressToINT8 / decompressINT8, native-engine/cpp/KVCompressionEngine.cpp:83-122)
  rounded to fp16.
- With fewer device slabs than layers, the layer evicted by each move to the
  GPU is the least recently used one, lowest index on ties
  (KVCacheGPU::findLRUPage, native-engine/cpp/KVCacheGPU.cpp:54-66).
- adaptive_engine_decode_step (host buffers in and out) equals the oracle's
  append + paged GQA decode, and leaves the pool as the oracle's append.
"""
import numpy as np
import pytest

import kvgen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-2
LAYERS, PAGES, HKV, HQ = 4, 32, 8, 24


@pytest.fixture()
def engine(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx.engine as E
    api = E.api()
    api.stop()
    yield E, api, tmp_path
    api.stop()


def start(E, api, tmp_path, slots=LAYERS, batch=4):
    E.configure(layers=LAYERS, pages_per_layer=PAGES, max_batch=batch, gpu_layer_slots=slots,
                offload_dir=str(tmp_path))
    api.start()
    assert api.getKvPages() == LAYERS


def slab(seed):
    return kvgen.normal(seed, (PAGES, 2, HKV, 16, 128)).astype(np.float16)


def test_tier_round_trips_preserve_bytes(engine):
    E, api, tmp = engine
    start(E, api, tmp)
    data = [slab(100 + l) for l in range(LAYERS)]
    for l in range(LAYERS):
        E.load_layer(l, data[l])
    assert api.moveKvToRam(0) > 0 and E.tier(0) == "RAM"
    assert api.offloadKv(1) > 0 and E.tier(1) == "OFFLOADED"
    assert api.moveKvToRam(1) > 0 and E.tier(1) == "RAM"
    assert api.offloadKv(2) > 0 and E.tier(2) == "OFFLOADED"
    for l in range(3):
        assert api.moveKvToGpu(l) > 0 and E.tier(l) == "GPU"
        back = np.empty_like(data[l])
        E.read_layer(l, back)
        assert np.array_equal(back.view(np.uint16), data[l].view(np.uint16)), l


def test_compress_tier_matches_reference_codec(engine, oracle):
    E, api, tmp = engine
    start(E, api, tmp)
    x = slab(7)
    x.reshape(-1)[::997] *= np.float16(20)
    E.load_layer(3, x)
    assert api.compressKv(3) > 0 and E.tier(3) == "COMPRESSED"
    assert api.moveKvToGpu(3) > 0 and E.tier(3) == "GPU"
    back = np.empty_like(x)
    E.read_layer(3, back)
    codes, stats = oracle.compress_int8_blocks(x, 2048)
    want = oracle.decompress_int8_blocks(codes, stats, 2048).astype(np.float16).reshape(x.shape)
    assert np.array_equal(back.view(np.uint16), want.view(np.uint16))


def test_lru_eviction_under_device_budget(engine):
    E, api, tmp = engine
    start(E, api, tmp, slots=2)
    # layers 0,1 start on the device (stamps 0), 2,3 in RAM
    stamp = {0: 0, 1: 0}
    clock = 0
    rng = np.random.default_rng(5)
    for step in range(40):
        l = int(rng.integers(0, LAYERS))
        resident = {k for k in range(LAYERS) if E.tier(k) == "GPU"}
        assert resident == set(stamp), step
        want_victim = None
        if l not in stamp and len(stamp) == 2:
            want_victim = min(sorted(stamp), key=lambda k: stamp[k])  # min stamp, lowest index
        clock += 1
        assert api.moveKvToGpu(l) > 0
        if want_victim is not None:
            assert E.tier(want_victim) == "RAM", step
            del stamp[want_victim]
        stamp[l] = clock
    assert api.keepLayer(0) >= 1  # pinned layers are never victims
    for l in (1, 2, 3, 1, 2, 3):
        assert api.moveKvToGpu(l) > 0
        assert E.tier(0) == "GPU"
    for _ in range(3):
        E.lib.adaptive_engine_test_release_layer(0)


def test_decode_step_through_host_buffers(engine, oracle):
    E, api, tmp = engine
    start(E, api, tmp, batch=4)
    lens = np.array([0, 15, 40, 100], np.int32)
    E.set_sequences(lens, reserve_tokens=20, seed=11)
    bt = E.block_table(len(lens))
    pools = [slab(300 + l) for l in range(LAYERS)]
    for l in range(LAYERS):
        E.load_layer(l, pools[l])
    q = kvgen.normal(1, (LAYERS, 4, HQ, 128)).astype(np.float16)
    k = kvgen.normal(2, (LAYERS, 4, HKV, 128)).astype(np.float16)
    v = kvgen.normal(3, (LAYERS, 4, HKV, 128)).astype(np.float16)
    out = np.zeros_like(q)
    for step in range(2):
        E.decode_step(q, k, v, out)
        for l in range(LAYERS):
            oracle.append(pools[l], bt, lens, k[l], v[l], 16)
            ref = oracle.paged_decode(pools[l], bt, lens + 1, q[l].astype(np.float32))
            got = out[l].astype(np.float32)
            excess = np.abs(got - ref) - (ATOL + RTOL * np.abs(ref))
            assert excess.max() <= 0, (step, l, excess.max())
            back = np.empty_like(pools[l])
            E.read_layer(l, back)
            assert np.array_equal(back.view(np.uint16), pools[l].view(np.uint16)), (step, l)
        lens = lens + 1
        assert [E.lib.adaptive_engine_seq_len(s) for s in range(4)] == list(lens)


def test_decode_step_with_layers_in_other_tiers(engine, oracle):
    E, api, tmp = engine
    start(E, api, tmp, slots=2, batch=2)
    lens = np.array([33, 64], np.int32)
    E.set_sequences(lens, reserve_tokens=4, seed=0)
    bt = E.block_table(2)
    pools = [slab(500 + l) for l in range(LAYERS)]
    for l in range(LAYERS):
        E.load_layer(l, pools[l])
    assert api.offloadKv(1) > 0
    q = kvgen.normal(4, (LAYERS, 2, HQ, 128)).astype(np.float16)
    k = kvgen.normal(5, (LAYERS, 2, HKV, 128)).astype(np.float16)
    v = kvgen.normal(6, (LAYERS, 2, HKV, 128)).astype(np.float16)
    out = np.zeros_like(q)
    E.decode_step(q, k, v, out)  # brings every layer through the two device slabs
    for l in range(LAYERS):
        oracle.append(pools[l], bt, lens, k[l], v[l], 16)
        ref = oracle.paged_decode(pools[l], bt, lens + 1, q[l].astype(np.float32))
        excess = np.abs(out[l].astype(np.float32) - ref) - (ATOL + RTOL * np.abs(ref))
        assert excess.max() <= 0, l


def test_decode_step_28_layers_with_split_contexts(engine, oracle, monkeypatch):
    """adaptive_engine_decode_step at the bench's depth: 28 layers, run in
    groups (dependent launches within a group, copies between groups) of 2,
    24 and 2 layers in the first step and 2, 7, 7, 7, 3 and 2 in the second
    (KVX_ENGINE_GROUP=7), batch 8 with contexts of 2,048-8,192 tokens so the
    longer sequences are split over several CTAs; every layer's output
    against the oracle and every pool bit for bit."""
    E, api, tmp = engine
    L, B = 28, 8
    lens = kvgen.randint(626, B, 2048, 8192).astype(np.int32)
    pages = int(((lens + 2 + 15) // 16).sum())
    E.configure(layers=L, kv_heads=HKV, q_heads=HQ, max_batch=B, pages_per_layer=pages, gpu_layer_slots=L,
                offload_dir=str(tmp))
    api.start()
    E.set_sequences(lens, reserve_tokens=2, seed=627)
    bt = E.block_table(B)
    g = torch.Generator(device="cuda")
    g.manual_seed(628)
    pools0 = []
    for l in range(L):
        p = torch.randn((pages, 2, HKV, 16, 128), generator=g, device="cuda", dtype=torch.float16)
        E.load_layer(l, p)
        pools0.append(p)
    q = kvgen.normal(629, (L, B, HQ, 128)).astype(np.float16)
    k = kvgen.normal(630, (L, B, HKV, 128)).astype(np.float16)
    v = kvgen.normal(631, (L, B, HKV, 128)).astype(np.float16)
    outs = [np.zeros_like(q) for _ in range(2)]
    for step in range(2):
        if step == 1:
            monkeypatch.setenv("KVX_ENGINE_GROUP", "7")
        E.decode_step(q, k, v, outs[step])
    assert [E.lib.adaptive_engine_seq_len(s) for s in range(B)] == list(lens + 2)
    back = torch.empty_like(pools0[0])
    for l in range(L):
        host = pools0[l].cpu().numpy()
        for step in range(2):
            pos = (lens + step).astype(np.int32)
            oracle.append(host, bt, pos, k[l], v[l], 16)
            ref = oracle.paged_decode(host, bt, pos + 1, q[l].astype(np.float32))
            excess = np.abs(outs[step][l].astype(np.float32) - ref) - (ATOL + RTOL * np.abs(ref))
            assert excess.max() <= 0, (step, l, excess.max())
        E.read_layer(l, back)
        assert np.array_equal(back.cpu().numpy().view(np.uint16), host.view(np.uint16)), l


def test_layer_move_overlaps_a_running_decode_step(engine, oracle):
    """A NativeEngineApi move of a layer the running decode step is done with
    runs while the step's later layers still decode: the step waits for its
    kernels with the engine lock released, and the move waits only for its
    own layer's last kernel (the output event of the step's first group of
    layers).  16 layers x 16 sequences x 32,768 tokens make a step of a few
    milliseconds; compressKv(0) is issued as soon as the step is in flight
    and must return while the step still is.  The step's outputs are then
    checked against the oracle (layer 0 was read before it was compressed)."""
    import threading
    E, api, tmp = engine
    L, B, T = 16, 16, 32768
    lens = np.full(B, T - 1, np.int32)
    pages = B * (T // 16 + 1)
    E.configure(layers=L, kv_heads=HKV, q_heads=HQ, max_batch=B, pages_per_layer=pages, gpu_layer_slots=L,
                ram_layer_slots=0, int8_layer_slots=1, offload_dir=str(tmp))
    api.start()
    E.set_sequences(lens, reserve_tokens=1, seed=641)
    bt = E.block_table(B)
    g = torch.Generator(device="cuda")
    g.manual_seed(642)
    pool = torch.randn((pages, 2, HKV, 16, 128), generator=g, device="cuda", dtype=torch.float16)
    for l in range(L):
        E.load_layer(l, pool)
    q = kvgen.normal(643, (L, B, HQ, 128)).astype(np.float16)
    k = kvgen.normal(644, (L, B, HKV, 128)).astype(np.float16)
    v = kvgen.normal(645, (L, B, HKV, 128)).astype(np.float16)
    # pinned host buffers: a copy to pageable memory would hold the calling
    # thread (and with it the engine lock) until the step's kernels are done
    h_q, h_k, h_v = (torch.from_numpy(a).pin_memory() for a in (q, k, v))
    h_out = torch.zeros(q.shape, dtype=torch.float16).pin_memory()
    E.decode_step(h_q, h_k, h_v, h_out)  # warm-up (lazy module loading), context now T
    lens = lens + 1
    E.set_sequences(lens - 1, reserve_tokens=1, seed=641)  # same pages, back to T - 1 tokens
    status = {}

    def run_step():
        try:
            E.decode_step(h_q, h_k, h_v, h_out)
            status["step"] = "ok"
        except Exception as e:  # noqa: BLE001
            status["step"] = repr(e)

    t = threading.Thread(target=run_step)
    t.start()
    for _ in range(2_000_000):
        if E.lib.adaptive_engine_step_in_flight():
            break
    else:
        t.join()
        pytest.fail("the step never showed as in flight")
    ms = api.compressKv(0)
    still_running = E.lib.adaptive_engine_step_in_flight()
    t.join()
    assert status.get("step") == "ok", status
    assert ms > 0 and E.tier(0) == "COMPRESSED"
    assert still_running == 1, "the move waited for the whole step"
    out = h_out.numpy()
    host = pool.cpu().numpy()
    for l in (0, 1, L - 1):
        pl = host.copy()
        oracle.append(pl, bt[:3], (lens[:3] - 1).astype(np.int32), k[l, :3], v[l, :3], 16)
        ref = oracle.paged_decode(pl, bt[:3], lens[:3].astype(np.int32), q[l, :3].astype(np.float32))
        excess = np.abs(out[l, :3].astype(np.float32) - ref) - (ATOL + RTOL * np.abs(ref))
        assert excess.max() <= 0, (l, excess.max())


def test_moves_use_the_slots_made_at_start(engine):
    """RAM and int8 tiers take slots of arenas made by start(): with one RAM
    slot, a second layer cannot move to RAM (-1) until the first leaves it."""
    E, api, tmp = engine
    E.configure(layers=LAYERS, pages_per_layer=PAGES, max_batch=4, gpu_layer_slots=LAYERS, ram_layer_slots=1,
                int8_layer_slots=1, offload_dir=str(tmp))
    api.start()
    data = [slab(700 + l) for l in range(LAYERS)]
    for l in range(LAYERS):
        E.load_layer(l, data[l])
    assert api.moveKvToRam(0) > 0
    assert api.moveKvToRam(1) == -1 and E.tier(1) == "GPU"
    assert api.compressKv(2) > 0
    assert api.compressKv(3) == -1 and E.tier(3) == "GPU"
    assert api.moveKvToGpu(0) > 0
    assert api.moveKvToRam(1) > 0 and E.tier(1) == "RAM"
    assert api.moveKvToGpu(2) > 0 and api.compressKv(3) > 0
    for l in (0, 1):
        assert api.moveKvToGpu(l) >= 0
        back = np.empty_like(data[l])
        E.read_layer(l, back)
        assert np.array_equal(back.view(np.uint16), data[l].view(np.uint16)), l


def test_age_policy_compresses_old_layers(engine, oracle):
    """The Java KVCompressionEngine's age policy
    (src/main/java/com/adaptivellm/kv/KVCompressionEngine.java:62-98) over
    the engine's layers: age = now - last access; >= compressedThreshold ->
    COMPRESSED (the NF4 tier here), else >= int8Threshold -> INT8 (the int8
    tier); only GPU-resident, unpinned layers change.  Decisions are checked
    at both thresholds' boundaries; applied, the NF4 round trip equals the
    oracle's compressToNF4 / decompressNF4 rounded to fp16, bit for bit."""
    from kvx import KvxError
    E, api, tmp = engine
    start(E, api, tmp)
    data = [slab(900 + l) for l in range(LAYERS)]
    for l in range(LAYERS):
        E.load_layer(l, data[l])
    a = [E.last_access_ms(l) for l in range(LAYERS)]
    lo, hi = min(a), max(a)
    for now in (lo + 99, lo + 100, hi + 99, hi + 100, hi + 999, hi + 1000, hi + 50000):
        n, d = E.compress_aged(100, 1000, now, apply=False)
        want = [2 if now - t >= 1000 else 1 if now - t >= 100 else 0 for t in a]
        assert n == 0 and list(d) == want, (now, a)
    for bad in ((0, 1000), (100, 0), (-5, 10)):
        with pytest.raises(KvxError):
            E.compress_aged(*bad, hi + 1000)
    assert api.keepLayer(3) >= 1             # pinned: left alone
    assert api.moveKvToRam(2) > 0            # not on the GPU: left alone
    n, d = E.compress_aged(100, 1000, hi + 1000)
    assert n == 2 and list(d) == [2, 2, 0, 0]
    assert [E.tier(l) for l in range(LAYERS)] == ["COMPRESSED_NF4", "COMPRESSED_NF4", "RAM", "GPU"]
    assert api.moveKvToGpu(0) > 0 and E.tier(0) == "GPU"
    back = np.empty_like(data[0])
    E.read_layer(0, back)
    codes, stats = oracle.compress_nf4_blocks(data[0], 2048)
    want = oracle.decompress_nf4_blocks(codes, stats, 2048).astype(np.float16).reshape(data[0].shape)
    assert np.array_equal(back.view(np.uint16), want.view(np.uint16))
    # INT8 branch: layer 0 written again (an access), 100 ms later it is INT8
    E.load_layer(0, data[0])
    t0 = E.last_access_ms(0)
    n, d = E.compress_aged(100, 1000, t0 + 100)
    assert n == 1 and d[0] == 1 and E.tier(0) == "COMPRESSED"
    assert api.moveKvToGpu(0) > 0
    E.read_layer(0, back)
    codes, stats = oracle.compress_int8_blocks(data[0], 2048)
    want = oracle.decompress_int8_blocks(codes, stats, 2048).astype(np.float16).reshape(data[0].shape)
    assert np.array_equal(back.view(np.uint16), want.view(np.uint16))
    for _ in range(2):
        E.lib.adaptive_engine_test_release_layer(3)
