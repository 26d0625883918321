"""Pin the C restatement (oracle/kvx_oracle.c) to the reference's own outputs.

The fixtures in tests/golden/ were produced by the reference sources compiled
unmodified (tests/golden/make_golden.py).  Integer / bit results must match
exactly; the attention rows also match bit for bit, because the restatement
keeps the reference's loop order and is built without FMA contraction.
"""
import hashlib

import numpy as np
import pytest

import kvgen
from conftest import golden


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_f16_trunc_encode(oracle):
    g = golden("kv_compress.npz")
    assert np.array_equal(oracle.f32_to_f16_trunc(g["x"]), g["enc"])


def test_f16_trunc_decode_all_patterns(oracle):
    g = golden("kv_compress.npz")
    dec = oracle.f16_trunc_to_f32(np.arange(65536, dtype=np.uint16))
    assert np.array_equal(dec.view(np.uint32), g["dec_bits"])


def test_kv_test_known_answers(oracle):
    # tests/kv_test.cpp prints key[0] after a disk round trip: 0.0999756, 1.09961, 2.09961
    x = np.array([0.1, 1.1, 2.1], np.float32)
    back = oracle.f16_trunc_to_f32(oracle.f32_to_f16_trunc(x))
    assert [f"{v:.6g}" for v in back] == ["0.0999756", "1.09961", "2.09961"]


def test_int8_codes_stats_exact(oracle):
    g = golden("int8.npz")
    off = 0
    for i, n in enumerate(g["lens"]):
        data = g["data"][off:off + n]
        codes, stats = oracle.compress_int8(data)
        assert np.array_equal(codes, g["codes"][off:off + n]), g["names"][i]
        assert np.array_equal(stats.view(np.uint32), g["stats"][i].view(np.uint32)), g["names"][i]
        dec = oracle.decompress_int8(codes, stats)
        assert np.array_equal(dec.view(np.uint32), g["dec"][off:off + n].view(np.uint32))
        off += n


def test_int8_f16_page_blocks(oracle):
    g = golden("int8.npz")
    blocks = g["f16_blocks"].view(np.float16)
    codes, stats = oracle.compress_int8_blocks(blocks, 2048)
    names = list(g["names"])
    first = names.index("f16_page_block")
    off = int(np.sum(g["lens"][:first]))
    assert np.array_equal(codes, g["codes"][off:off + codes.size])
    assert np.array_equal(stats.view(np.uint32), g["stats"][first:first + 8].view(np.uint32))


def test_nf4_codes_stats_exact(oracle):
    """KVCompressionEngine NF4 (native-engine/cpp/KVCompressionEngine.cpp:124-180)."""
    g = golden("nf4.npz")
    off = coff = 0
    for i, n in enumerate(g["lens"]):
        data = g["data"][off:off + n]
        cb = (n + 1) // 2
        codes, stats = oracle.compress_nf4(data)
        assert np.array_equal(codes, g["codes"][coff:coff + cb]), g["names"][i]
        assert np.array_equal(stats.view(np.uint32), g["stats"][i].view(np.uint32)), g["names"][i]
        dec = oracle.decompress_nf4(codes, stats, n)
        assert np.array_equal(dec.view(np.uint32), g["dec"][off:off + n].view(np.uint32)), g["names"][i]
        off += n
        coff += cb
    blocks = g["f16_blocks"].view(np.float16)
    codes, stats = oracle.compress_nf4_blocks(blocks, 2048)
    first = list(g["names"]).index("f16_page_block")
    start = int(np.sum((g["lens"][:first] + 1) // 2))
    assert np.array_equal(codes, g["codes"][start:start + codes.size])
    assert np.array_equal(stats.view(np.uint32), g["stats"][first:first + 8].view(np.uint32))


def test_fp16_wrap_exact(oracle):
    """KVCompressionEngine FP16 (native-engine/cpp/KVCompressionEngine.cpp:36-80): the
    exponent-wrapping conversion, not IEEE; every half decoded."""
    g = golden("fp16_wrap.npz")
    assert np.array_equal(oracle.fp16_wrap_encode(g["x"]), g["enc"])
    dec = oracle.fp16_wrap_decode(np.arange(65536, dtype=np.uint16))
    assert np.array_equal(dec.view(np.uint32), g["dec_bits"])
    assert dec[0] == np.float32(2.0 ** -15) and dec[0x7C00] == np.float32(65536.0)  # the quirks kept


def test_attention_rows(oracle):
    g = golden("attention.npz")
    for i, T in enumerate((1, 2, 3, 16, 33, 257)):
        q = kvgen.normal(400 + i, (128,))
        k = kvgen.normal(500 + i, (T, 128))
        v = kvgen.normal(600 + i, (T, 128))
        assert np.array_equal(oracle.attention_row(q, k, v), g["rows"][i])


def test_attention_identity_property():
    # tests/cpu_ops_test.cpp:35-47: each row weights itself and sums to 1
    out = golden("attention.npz")["identity"]
    assert out[0, 0] > out[0, 1] and out[1, 1] > out[1, 0]
    assert abs(out[0].sum() - 1) < 1e-3 and abs(out[1].sum() - 1) < 1e-3


def _paged_inputs(g, dtype):
    B = len(g["seq_lens"])
    tmax = int(g["seq_lens"].max())
    hkv, hq, dim = int(g["hkv"]), int(g["hq"]), int(g["dim"])
    seed = int(g["seed"])
    K = kvgen.normal(seed + 1, (B, tmax, hkv, dim)).astype(dtype)
    V = kvgen.normal(seed + 2, (B, tmax, hkv, dim)).astype(dtype)
    Q = kvgen.normal(seed + 3, (B, hq, dim)).astype(np.float32)
    assert sha(K, V, Q) == str(g["input_sha"]), "input generator drifted"
    return K, V, Q


def _fill_pool(oracle, g, K, V):
    """Append every token in order through the oracle's paged append."""
    pt, dim, hkv = int(g["pt"]), int(g["dim"]), int(g["hkv"])
    pool = np.zeros((int(g["num_pages"]), 2, hkv, pt, dim), K.dtype)
    bt = g["block_table"]
    lens = g["seq_lens"]
    for t in range(int(lens.max())):
        rows = np.nonzero(lens > t)[0]
        oracle.append(pool, bt[rows], np.full(rows.size, t, np.int32), K[rows, t], V[rows, t], pt)
    return pool


@pytest.mark.parametrize("name,dtype", [("paged_cfg1.npz", np.float32),
                                        ("paged_fp16.npz", np.float16),
                                        ("paged_gqa8.npz", np.float16)])
def test_paged_decode_matches_reference(oracle, name, dtype):
    g = golden(name)
    K, V, Q = _paged_inputs(g, dtype)
    pool = _fill_pool(oracle, g, K, V)
    out = oracle.paged_decode(pool, g["block_table"], g["seq_lens"], Q)
    assert np.array_equal(out, g["out"])


def test_int8_decode_matches_reference(oracle):
    g = golden("int8_decode.npz")
    seed, pt, dim, hkv, hq = int(g["seed"]), int(g["pt"]), int(g["dim"]), int(g["hkv"]), int(g["hq"])
    num_pages = int(g["num_pages"])
    pool = kvgen.normal(seed + 1, (num_pages, 2, hkv, pt, dim)).astype(np.float16)
    mask = kvgen.uniform(seed + 5, pool.size).reshape(pool.shape) < 0.01
    pool = (pool.astype(np.float32) * np.where(mask, 20.0, 1.0)).astype(np.float16)
    Q = kvgen.normal(seed + 3, (len(g["seq_lens"]), hq, dim))
    assert sha(pool, Q) == str(g["input_sha"])
    codes, stats = oracle.compress_int8_blocks(pool, pt * dim)
    assert sha(codes.reshape(-1, pt * dim)) == str(g["codes_sha"])
    assert np.array_equal(stats.view(np.uint32), g["stats"].view(np.uint32))
    out = oracle.paged_decode(codes.reshape(pool.shape), g["block_table"], g["seq_lens"], Q,
                              stats=stats)
    assert np.array_equal(out, g["out"])


def test_lru_replay_matches_kvmanager(oracle):
    g = golden("lru.npz")
    for i in range(int(g["n_traces"])):
        ev, hit = oracle.lru_replay(g[f"ids{i}"], g[f"ops{i}"], int(g[f"cap{i}"]))
        assert np.array_equal(ev, g[f"evicted{i}"]), i
        assert np.array_equal(hit, g[f"hit{i}"]), i


def test_kv_test_eviction_order(oracle):
    # tests/kv_test.cpp: capacity 2, pages 0,1,2 saved; loading 0,1,2 evicts 0 last
    g = golden("lru.npz")
    ev = g["evicted0"]
    assert list(ev) == [-1, -1, 0, 1, 2, 0]


def test_lru_select(oracle):
    g = golden("lru.npz")
    for st, n, want in zip(g["select_stamps"], g["select_n"], g["select_out"]):
        assert oracle.lru_select(st[:n]) == want


def test_prefetch_depth(oracle):
    g = golden("prefetch_depth.npz")
    for li, size, cap, md, want in g["grid"]:
        assert oracle.prefetch_depth(g[f"lat{li}"], int(size), int(cap), int(md)) == want


def test_disk_page_format():
    from oracle import persist_bytes
    g = golden("disk_page.npz")
    assert persist_bytes(g["key"], g["value"]) == g["blob"].tobytes()


def test_eviction_policies_exact(oracle):
    """AdvancedEvictionPolicy (native-engine/cpp/AdvancedEvictionPolicy.cpp): every
    policy's calculateScore(m, 0) and selectPageToEvict, the currentToken = 0
    wrap-around kept; Predictive from replayed access histories; composite."""
    from oracle import EVICT_METRICS
    g = golden("evict.npz")
    for c in range(12):
        m = g[f"pages{c}"].view(EVICT_METRICS)
        hist, hl = g[f"hist{c}"], g[f"hist_len{c}"]
        pred = np.array([oracle.predict_next_access(hist[i, :hl[i]]) for i in range(m.size)], np.float32)
        for pol in (0, 1, 2, 3):
            p = pred if pol == 3 else None
            assert oracle.evict_select(pol, m, 0.95, p) == int(g[f"sel{c}_{pol}"]), (c, pol)
            assert np.array_equal(oracle.evict_scores(pol, m, 0.95, p).view(np.uint32),
                                  g[f"scores{c}_{pol}"].view(np.uint32)), (c, pol)
        got = oracle.evict_select_composite(np.array([0, 1, 2], np.int32), g[f"composite_w{c}"], m)
        assert got == int(g[f"composite{c}"]), c


def test_kvcache_gpu_policy_matches_reference(oracle):
    """KVCacheGPU (native-engine/cpp/KVCacheGPU.cpp): every transfer's
    success, evictions, lookups and the byte count after each op, replayed
    on the reference's own class (golden) and on the restatement."""
    g = golden("kvcache_gpu.npz")
    for i in range(int(g["n_traces"])):
        res, used = oracle.kvcache_gpu_replay(g[f"ops{i}"], int(g[f"budget{i}"]), int(g[f"page{i}"]))
        assert np.array_equal(res, g[f"result{i}"]), i
        assert np.array_equal(used, g[f"used{i}"]), i
