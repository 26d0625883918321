"""The C++ drop-ins of the reference's cache / compression / scheduler
headers (include/kv_cache.h, kv_pager.h, kv_compress.h, scheduler.h),
exercised by C++ programs ported from the reference's own tests
(tests/kv_test.cpp, kv_pager_test.cpp, kv_integration_test.cpp) and checked
against the reference's golden outputs (tests/golden/)."""
import os
import subprocess

import numpy as np
import pytest

from conftest import golden

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CDIR = os.path.join(ROOT, "tests", "cpp")


@pytest.fixture(scope="module")
def built():
    subprocess.run(["make", "-s", "-C", CDIR], check=True)
    return os.path.join(CDIR, "_build")


def run(built, name, *args, stdin=None):
    r = subprocess.run([os.path.join(built, name), *map(str, args)], capture_output=True,
                       text=True, input=stdin, timeout=120)
    return r.returncode, r.stdout + r.stderr


def test_scheduler_depth_matches_reference(built):
    g = golden("prefetch_depth.npz")
    lines, want = [], []
    for li, size, cap, md, depth in g["grid"]:
        lat = g[f"lat{li}"]
        lines.append(" ".join([str(size), str(cap), str(md), str(lat.size)] + [repr(float(x)) for x in lat]))
        want.append(int(depth))
    rc, out = run(built, "scheduler_depth", stdin="\n".join(lines) + "\n")
    assert rc == 0, out
    assert [int(x) for x in out.split()] == want


def test_scheduler_c_entry_points_match_reference():
    """kvx_scheduler_* (include/kvx_scheduler.h) over the same golden grid:
    a fresh Scheduler per case, fed the case's latencies, asked once."""
    from kvx.scheduler import Scheduler
    g = golden("prefetch_depth.npz")
    for li, size, cap, md, depth in g["grid"]:
        s = Scheduler(int(md))
        for x in g[f"lat{li}"]:
            s.observe(float(x))
        assert s.depth(0, int(size), int(cap)) == int(depth), (li, size, cap, md)
        s.close()


def test_scheduler_c_entry_points_check_arguments():
    import ctypes
    from kvx import KvxError
    from kvx.scheduler import Scheduler, lib as slib
    with pytest.raises(KvxError):
        Scheduler(0)  # max_depth >= 1
    s = Scheduler(4)
    with pytest.raises(KvxError):
        s.observe(-1.0)
    with pytest.raises(KvxError):
        s.depth(0, -1, 10)
    assert slib.kvx_scheduler_depth(s.h, 0, 0, 10, None) == -1
    assert s.depth(0, 10, 10) == 1  # a full cache: depth 1 whatever the latency
    s.close()


def test_prefetcher_drop_in(built):
    """Prefetcher (prefetch/prefetcher.h:14-38): requests are served in FIFO
    order by the worker; a mover result of 0 is a hit (no load, nothing
    observed), < 0 a failure, > 0 a load whose latency goes to the
    Scheduler, which then decides exactly as one fed the same latencies;
    schedule(5, 8) requests layers 6 .. 5 + depth below 8
    (InferenceController::schedulePrefetch, runtime/inference.cpp:61-84)."""
    rc, out = run(built, "prefetcher_io")
    assert rc == 0, out
    lines = dict(line.split(" ", 1) for line in out.strip().splitlines() if " " in line)
    assert [int(x) for x in lines["order"].split()] == list(range(16))
    loads = [i for i in range(16) if i % 3 != 0 and i != 13]
    assert [int(x) for x in lines["counts"].split()] == [16, len(loads), 1]
    d_sched, d_twin = map(int, lines["depth"].split())
    assert d_sched == d_twin
    sched = [int(x) for x in lines["schedule"].split()]
    depth = sched[0]
    assert sched[1:] == [l for l in range(6, 6 + depth) if l < 8]
    assert out.strip().endswith("ok")


@pytest.mark.gpu
def test_prefetcher_moves_engine_layers(built, tmp_path):
    """The Prefetcher's default mover is the engine's move to the GPU tier:
    prefetched layers become GPU-resident, the least recently used ones go
    to RAM (KVCacheGPU's evict-then-retry), a resident layer is a hit."""
    rc, out = run(built, "prefetcher_engine", tmp_path)
    assert rc == 0 and out.strip().endswith("ok"), out


@pytest.mark.gpu
def test_kv_test_known_answers(built, tmp_path):
    # tests/kv_test.cpp of the reference prints 0.0999756, 1.09961, 2.09961
    rc, out = run(built, "kv_test", tmp_path / "pages")
    assert rc == 0, out
    assert "key[0]=0.0999756" in out and "key[0]=1.09961" in out and "key[0]=2.09961" in out
    assert "Eviction succeeded" in out


@pytest.mark.gpu
def test_kv_pager_prefetch(built, tmp_path):
    rc, out = run(built, "kv_pager_test", tmp_path / "pages")
    assert rc == 0, out


@pytest.mark.gpu
def test_kv_integration(built, tmp_path):
    rc, out = run(built, "kv_integration_test", tmp_path / "pages")
    assert rc == 0, out


@pytest.mark.gpu
def test_page_file_bytes_equal_reference(built, tmp_path):
    g = golden("disk_page.npz")
    d = tmp_path / "pages"
    d.mkdir()
    g["key"].astype(np.float32).tofile(tmp_path / "key.bin")
    g["value"].astype(np.float32).tofile(tmp_path / "value.bin")
    rc, out = run(built, "kv_disk_format", d, 5, tmp_path / "key.bin", tmp_path / "value.bin")
    assert rc == 0, out
    assert (d / "page_5.bin").read_bytes() == g["blob"].tobytes()
    back = np.fromfile(d / "back.bin", np.float32)
    nk = g["key_back"].size
    assert np.array_equal(back[:nk].view(np.uint32), g["key_back"].view(np.uint32))
    assert np.array_equal(back[nk:].view(np.uint32), g["value_back"].view(np.uint32))


RTOL, ATOL = 1e-3, 1e-2


def close(got, want):
    excess = np.abs(np.asarray(got, np.float64) - want) - (ATOL + RTOL * np.abs(want))
    return excess.max() <= 0


@pytest.mark.gpu
def test_cuda_softmax_matches_tensorops(built, tmp_path):
    g = golden("attention.npz")
    x = np.array([[1, 2], [3, 2]], np.float32)
    (tmp_path / "in.bin").write_bytes(np.array([2, 2], np.uint64).tobytes() + x.tobytes())
    rc, out = run(built, "cuda_executor_io", "softmax", tmp_path / "in.bin", tmp_path / "out.bin")
    assert rc == 0, out
    assert close(np.fromfile(tmp_path / "out.bin", np.float32).reshape(2, 2), g["softmax"])


@pytest.mark.gpu
def test_cuda_attention_matches_tensorops(built, tmp_path):
    import kvgen
    g = golden("attention.npz")
    cases = [(np.array([[1, 0], [0, 1]], np.float32),) * 3]
    wants = [g["identity"]]
    for i, T in enumerate((1, 2, 3, 16, 33, 257)):
        q = kvgen.normal(400 + i, (128,))
        cases.append((np.tile(q, (T, 1)), kvgen.normal(500 + i, (T, 128)), kvgen.normal(600 + i, (T, 128))))
        wants.append(np.tile(g["rows"][i], (T, 1)))  # TensorOps::attention of a repeated query
    for (Q, K, V), want in zip(cases, wants):
        seq, dim = Q.shape
        blob = np.array([seq, dim], np.uint64).tobytes() + b"".join(
            np.ascontiguousarray(a, np.float32).tobytes() for a in (Q, K, V))
        (tmp_path / "in.bin").write_bytes(blob)
        rc, out = run(built, "cuda_executor_io", "attention", tmp_path / "in.bin", tmp_path / "out.bin")
        assert rc == 0, out
        assert close(np.fromfile(tmp_path / "out.bin", np.float32).reshape(seq, dim), want), seq


@pytest.mark.gpu
def test_kv_attention_backend_matches_oracle(built, tmp_path, oracle):
    import kvgen
    L, hkv, hq, pages, B, steps = 3, 2, 6, 16, 2, 20
    (tmp_path / "cfg.txt").write_text(
        f"layers = {L}\nkv_heads = {hkv}\nq_heads = {hq}\npages_per_layer = {pages}\n"
        f"max_batch = {B}\nbatch = {B}\n")
    xs = kvgen.normal(77, (steps, L, B, hq + 2 * hkv, 128))
    with open(tmp_path / "in.bin", "wb") as f:
        for s in range(steps):
            for l in range(L):
                f.write(np.array([xs[s, l].size], np.uint64).tobytes())
                f.write(xs[s, l].astype(np.float32).tobytes())
    rc, out = run(built, "kv_backend_io", tmp_path / "cfg.txt", tmp_path / "in.bin", tmp_path / "out.bin",
                  steps)
    assert rc == 0, out
    got = np.fromfile(tmp_path / "out.bin", np.float32).reshape(steps, L, B, hq, 128)
    # engine state: zero pools, sequences of length 0, pages handed out in order
    per_seq = (pages * 16 // B + 15) // 16
    bt = np.arange(B * per_seq, dtype=np.int32).reshape(B, per_seq)
    pools = [np.zeros((pages, 2, hkv, 16, 128), np.float16) for _ in range(L)]
    for s in range(steps):
        for l in range(L):
            x = xs[s, l]
            q, k, v = x[:, :hq], x[:, hq:hq + hkv].astype(np.float16), x[:, hq + hkv:].astype(np.float16)
            pos = np.full(B, s, np.int32)
            oracle.append(pools[l], bt, pos, k, v, 16)
            ref = oracle.paged_decode(pools[l], bt, pos + 1, q)
            assert close(got[s, l], ref), (s, l)


@pytest.mark.gpu
def test_kv_compression_engine_dropin_matches_reference(built, tmp_path, oracle):
    """include/KVCompressionEngine.h (the reference's native-engine class) on the
    GPU: every mode's ratio, stats, compressed bytes and round trip equal the
    reference's (through the oracle, itself pinned to the reference's golden
    outputs), one block per call as the reference computes it."""
    g = golden("nf4.npz")
    blocks, off = [], 0
    for n in g["lens"]:
        blocks.append(g["data"][off:off + int(n)])
        off += int(n)
    blocks.append(golden("fp16_wrap.npz")["x"])
    cases = [(t, b) for b in blocks for t in (0, 1, 2, 3)]
    with open(tmp_path / "in.bin", "wb") as f:
        for t, b in cases:
            f.write(np.int32(t).tobytes() + np.uint64(b.size).tobytes() + np.ascontiguousarray(b, np.float32).tobytes())
    rc, out = run(built, "kv_compression_engine_io", tmp_path / "in.bin", tmp_path / "out.bin")
    assert rc == 0, out
    raw = (tmp_path / "out.bin").read_bytes()
    pos = 0
    for t, b in cases:
        ratio, = np.frombuffer(raw, np.float32, 1, pos)
        stats = np.frombuffer(raw, np.float32, 4, pos + 4)
        typ, = np.frombuffer(raw, np.int32, 1, pos + 20)
        nbytes, = np.frombuffer(raw, np.uint64, 1, pos + 24)
        pos += 32
        comp = np.frombuffer(raw, np.uint8, int(nbytes), pos)
        pos += int(nbytes)
        back = np.frombuffer(raw, np.float32, b.size, pos)
        pos += 4 * b.size
        assert typ == t and ratio == (1.0, 0.5, 0.25, 0.125)[t]
        if t == 0:
            want_c, want_s, want_b = b.view(np.uint8), None, b
        elif t == 1:
            enc = oracle.fp16_wrap_encode(b)
            want_c, want_s, want_b = enc.view(np.uint8), None, oracle.fp16_wrap_decode(enc)
        elif t == 2:
            c, s = oracle.compress_int8(b)
            want_c, want_s, want_b = c.view(np.uint8), s, oracle.decompress_int8(c, s)
        else:
            c, s = oracle.compress_nf4(b)
            want_c, want_s, want_b = c, s, oracle.decompress_nf4(c, s, b.size)
        assert np.array_equal(comp, want_c), (t, b.size)
        if want_s is not None:
            assert np.array_equal(stats.view(np.uint32), want_s.view(np.uint32)), (t, b.size)
        assert np.array_equal(back.view(np.uint32), want_b.view(np.uint32)), (t, b.size)
    assert pos == len(raw)


@pytest.mark.gpu
def test_kvcache_gpu_dropin_matches_reference(built):
    """include/KVCacheGPU.h on the device slot pool against the reference's
    KVCacheGPU (golden traces): the same result and byte count after every op,
    one call per op and with transfers batched; page bytes intact."""
    g = golden("kvcache_gpu.npz")
    for i in range(int(g["n_traces"])):
        ops, res, used = g[f"ops{i}"], g[f"result{i}"], g[f"used{i}"]
        text = f"{int(g[f'budget{i}'])} {int(g[f'page{i}'])}\n" + "".join(f"{o} {a} {b}\n" for o, a, b in ops)
        rc, out = run(built, "kv_cache_gpu_io", stdin=text)
        assert rc == 0, out[-500:]
        lines = out.split("\n")
        p1 = lines.index("pass 1")
        p2 = lines.index("pass 2")
        one = [tuple(map(int, ln.split())) for ln in lines[p1 + 1:p2]]
        assert one == [(int(r), int(u)) for r, u in zip(res, used)], i
        k = 0
        for ln in lines[p2 + 1:]:
            if ln.startswith("corrupt"):
                assert ln == "corrupt 0", ln
                break
            a, b = ln.split()
            if a == "used":  # end of a batch of transfers
                assert int(b) == int(used[k - 1]), (i, k)
            elif b == "-":
                assert ops[k][0] == 0 and int(a) == int(res[k]), (i, k)
                k += 1
            else:
                assert (int(a), int(b)) == (int(res[k]), int(used[k])), (i, k)
                k += 1
        assert k == len(ops)


@pytest.mark.gpu
def test_kvcache_gpu_manager_natives():
    """The KVCacheGPUManager natives' C entry points (include/kvx_gpu_cache.h):
    handles, byte count, LRU eviction, copy back + release, stale handles."""
    import ctypes as C
    import kvx
    L = kvx.lib
    L.kvx_gpu_cache_transfer_to_gpu.restype = C.c_int64
    L.kvx_gpu_cache_transfer_to_gpu.argtypes = [C.c_void_p, C.c_int64, C.c_int32]
    L.kvx_gpu_cache_transfer_from_gpu.restype = C.c_int32
    L.kvx_gpu_cache_transfer_from_gpu.argtypes = [C.c_int64, C.c_void_p, C.c_int64]
    L.kvx_gpu_cache_used_memory.restype = C.c_int64
    L.kvx_gpu_cache_evict_lru.restype = C.c_int32
    L.kvx_gpu_cache_mark_page_used.argtypes = [C.c_int32, C.c_int64]
    L.kvx_gpu_cache_init.argtypes = [C.c_uint64, C.c_uint64]
    page = 64 * 1024
    assert L.kvx_gpu_cache_init(3 * page, page) == 0
    try:
        data = [np.random.default_rng(s).integers(0, 256, page, dtype=np.uint8) for s in range(4)]
        h = [L.kvx_gpu_cache_transfer_to_gpu(d.ctypes.data, page, i) for i, d in enumerate(data[:3])]
        assert all(x > 0 for x in h) and len(set(h)) == 3
        assert L.kvx_gpu_cache_used_memory() == 3 * page
        for pid, tok in ((0, 30), (1, 10), (2, 20)):
            L.kvx_gpu_cache_mark_page_used(pid, tok)
        h3 = L.kvx_gpu_cache_transfer_to_gpu(data[3].ctypes.data, page, 3)  # evicts page 1 (token 10)
        assert h3 > 0 and L.kvx_gpu_cache_used_memory() == 3 * page
        back = np.zeros(page, np.uint8)
        assert L.kvx_gpu_cache_transfer_from_gpu(h[1], back.ctypes.data, page) == 0  # evicted
        assert L.kvx_gpu_cache_transfer_from_gpu(h[2], back.ctypes.data, page) == 1
        assert np.array_equal(back, data[2]) and L.kvx_gpu_cache_used_memory() == 2 * page
        assert L.kvx_gpu_cache_transfer_from_gpu(h[2], back.ctypes.data, page) == 0  # handle spent
        assert L.kvx_gpu_cache_evict_lru() == 1  # page 3 (token 0)
        assert L.kvx_gpu_cache_transfer_from_gpu(h[0], back.ctypes.data, page) == 1
        assert np.array_equal(back, data[0]) and L.kvx_gpu_cache_used_memory() == 0
        assert L.kvx_gpu_cache_evict_lru() == 0
    finally:
        L.kvx_gpu_cache_shutdown()
