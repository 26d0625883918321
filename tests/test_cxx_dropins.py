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
