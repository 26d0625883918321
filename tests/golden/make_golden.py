"""Generate the golden fixtures of tests/golden/ from the reference itself.

Run in a checkout that has the reference sources (the library is built from
them by oracle/Makefile, target `ref`):

    python tests/golden/make_golden.py

Every array in the fixtures is an output of the reference's own functions
(oracle/_ref/libkvref.so), on inputs that are either stored in the fixture or
regenerated from a seed by tests/kvgen.py (a seed plus a sha256 of the input
bytes is stored, so drift in the generator is caught).
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(HERE))

import kvgen  # noqa: E402
from oracle import Reference, build_reference  # noqa: E402


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def special_floats() -> np.ndarray:
    vals = [0.1, 1.1, 2.1, 0.0, -0.0, np.inf, -np.inf, np.nan, 65504.0, 65519.0, 65520.0,
            1e5, 6.1e-5, 6.0e-5, 2.0 ** -14, 2.0 ** -15, 2.0 ** -24, 1e-8, -3e-5, 1.0,
            -1.0, 0.5, 3.14159, -2.71828, 1.0009765625, 1.00048828125]
    return np.array(vals, dtype=np.float32)


def gen_kv_compress(R: Reference):
    x = np.concatenate([special_floats(),
                        kvgen.normal(11, (2048,)) * np.float32(100.0),
                        kvgen.splitmix64(12, 2048).astype(np.uint32).view(np.float32)])
    enc = R.f32_to_f16_trunc(x)
    halves = np.arange(65536, dtype=np.uint16)
    dec = R.f16_trunc_to_f32(halves).view(np.uint32)
    np.savez_compressed(os.path.join(HERE, "kv_compress.npz"), x=x, enc=enc, dec_bits=dec)


def gen_int8(R: Reference):
    blocks, codes, stats, dec = [], [], [], []
    cases = []
    for n in (1, 2, 3, 17, 2048):
        base = kvgen.normal(100 + n, (n,))
        cases.append(("normal", base))
        out = base.copy()
        mask = kvgen.uniform(200 + n, n) < 0.01
        out[mask] *= np.float32(20.0)
        cases.append(("outliers", out))
        cases.append(("constant", np.full(n, 3.0, np.float32)))
        z = np.abs(base)
        z[n // 2] = 0.0
        z[0] = -0.0
        cases.append(("signed_zero_min", z))
        cases.append(("all_zero", np.zeros(n, np.float32)))
    nanfirst = kvgen.normal(300, (64,))
    nanfirst[0] = np.nan
    cases.append(("nan_first", nanfirst))
    nanmid = kvgen.normal(301, (64,))
    nanmid[7] = np.nan
    cases.append(("nan_mid", nanmid))
    big = kvgen.normal(302, (64,)) * np.float32(1e30)
    cases.append(("huge", big))
    tiny = kvgen.normal(303, (64,)) * np.float32(1e-42)
    cases.append(("denormal", tiny))
    inf = kvgen.normal(304, (64,))
    inf[3] = np.inf
    cases.append(("inf", inf))
    # fp16 page blocks (16 tokens x 128 dims) as the engine stores them
    f16 = (kvgen.normal(305, (8, 2048)) *
           np.where(kvgen.uniform(306, 8 * 2048).reshape(8, 2048) < 0.01, 20.0, 1.0)
           ).astype(np.float16)
    for b in range(8):
        cases.append(("f16_page_block", f16[b].astype(np.float32)))
    lens, names = [], []
    for name, v in cases:
        c, s = R.compress_int8(v)
        d = R.decompress_int8(c, s)
        blocks.append(v)
        codes.append(c)
        stats.append(s)
        dec.append(d)
        lens.append(v.size)
        names.append(name)
    np.savez_compressed(os.path.join(HERE, "int8.npz"), data=np.concatenate(blocks),
                        codes=np.concatenate(codes), stats=np.stack(stats),
                        dec=np.concatenate(dec), lens=np.array(lens), names=np.array(names),
                        f16_blocks=f16.view(np.uint16))


def codec_cases(seed0):
    """Edge-case blocks shared by the block codecs: sizes 1..2048 (odd ones
    too), outliers, constants, signed zeros, NaN first / inside, huge,
    denormal, Inf, and fp16 page blocks as the engine stores them."""
    cases = []
    for n in (1, 2, 3, 17, 2048):
        base = kvgen.normal(seed0 + n, (n,))
        cases.append(("normal", base))
        out = base.copy()
        out[kvgen.uniform(seed0 + 100 + n, n) < 0.01] *= np.float32(20.0)
        cases.append(("outliers", out))
        cases.append(("constant", np.full(n, 3.0, np.float32)))
        z = np.abs(base)
        z[n // 2] = 0.0
        z[0] = -0.0
        cases.append(("signed_zero_min", z))
    for name, fill in (("nan_first", 0), ("nan_mid", 7)):
        v = kvgen.normal(seed0 + 300 + fill, (65,))
        v[fill] = np.nan
        cases.append((name, v))
    cases.append(("huge", kvgen.normal(seed0 + 302, (64,)) * np.float32(1e30)))
    cases.append(("denormal", kvgen.normal(seed0 + 303, (64,)) * np.float32(1e-42)))
    inf = kvgen.normal(seed0 + 304, (64,))
    inf[3] = np.inf
    cases.append(("inf", inf))
    ties = ((np.arange(2048) % 16) + 0.5) / 15.0 * 7.0  # quotients on k + 1/2
    ties[0], ties[1] = 0.0, 7.0
    cases.append(("half_ties", ties.astype(np.float32)))
    f16 = (kvgen.normal(seed0 + 305, (8, 2048)) *
           np.where(kvgen.uniform(seed0 + 306, 8 * 2048).reshape(8, 2048) < 0.01, 20.0, 1.0)
           ).astype(np.float16)
    for b in range(8):
        cases.append(("f16_page_block", f16[b].astype(np.float32)))
    return cases, f16


def gen_nf4(R: Reference):
    """KVCompressionEngine NF4 (native-engine/cpp/KVCompressionEngine.cpp:124-180)."""
    cases, f16 = codec_cases(700)
    data, codes, stats, dec, lens, names = [], [], [], [], [], []
    for name, v in cases:
        c, st = R.compress_nf4(v)
        data.append(v)
        codes.append(c)
        stats.append(st)
        dec.append(R.decompress_nf4(c, st, v.size))
        lens.append(v.size)
        names.append(name)
    np.savez_compressed(os.path.join(HERE, "nf4.npz"), data=np.concatenate(data),
                        codes=np.concatenate(codes), stats=np.stack(stats), dec=np.concatenate(dec),
                        lens=np.array(lens), names=np.array(names), f16_blocks=f16.view(np.uint16))


def gen_fp16_wrap(R: Reference):
    """KVCompressionEngine FP16 (native-engine/cpp/KVCompressionEngine.cpp:36-80):
    every half decoded, special and random floats encoded."""
    h = np.arange(65536, dtype=np.uint16)
    rnd = kvgen.randint(900, 20000, 0, 2 ** 32 - 1).astype(np.uint32).view(np.float32)
    x = np.concatenate([special_floats(), kvgen.normal(901, (4096,)) * np.float32(1e3),
                        np.ldexp(np.float32(1.5), np.arange(-40, 40)).astype(np.float32), rnd])
    np.savez_compressed(os.path.join(HERE, "fp16_wrap.npz"), x=x, enc=R.fp16_wrap_encode(x),
                        dec_bits=R.fp16_wrap_decode(h).view(np.uint32))


def gen_evict(R: Reference):
    """AdvancedEvictionPolicy selectPageToEvict and calculateScore(m, 0) of
    every policy (native-engine/cpp/AdvancedEvictionPolicy.cpp), Predictive
    after replaying per-page access histories, and one composite manager."""
    from oracle import EVICT_METRICS
    res = {}
    for c in range(12):
        n = int(kvgen.randint(1000 + c, 1, 1, 400)[0])
        m = np.zeros(n, EVICT_METRICS)
        m["last_access_token"] = kvgen.randint(1100 + c, n, 0, 10 ** 6).astype(np.uint64)
        m["last_access_token"][kvgen.uniform(1200 + c, n) < (0.0 if c % 3 == 0 else 0.1)] = 0
        if c == 5:
            m["last_access_token"][:] = 0
        if c == 7:
            m["last_access_token"][0] = np.uint64(2 ** 64 - 5)
        m["average_attention"] = kvgen.uniform(1300 + c, n).astype(np.float32)
        m["average_attention"][n // 2] = m["average_attention"][0]
        m["page_id"] = kvgen.permutation(1400 + c, n) + 100
        hl = kvgen.randint(1500 + c, n, 0, 10).astype(np.int32)
        hist = np.zeros((n, 10), np.uint64)
        for i in range(n):
            hist[i, :hl[i]] = np.sort(kvgen.randint(1600 + c * 1000 + i, int(hl[i]), 0, 10 ** 6)).astype(np.uint64)
        res[f"pages{c}"] = m.view(np.uint8)
        res[f"hist{c}"] = hist
        res[f"hist_len{c}"] = hl
        for pol in (0, 1, 2, 3):
            sel, sc = R.evict_select(pol, m, 0.95, hist if pol == 3 else None, hl if pol == 3 else None)
            res[f"sel{c}_{pol}"] = np.int32(sel)
            res[f"scores{c}_{pol}"] = sc
        sel, nw = R.evict_composite([0, 1, 2], np.array([1.0, 2.0, 0.5], np.float32), m)
        res[f"composite{c}"] = np.int32(sel)
        res[f"composite_w{c}"] = nw
    np.savez_compressed(os.path.join(HERE, "evict.npz"), **res)


def gen_attention(R: Reference):
    # cpu_ops_test (tests/cpu_ops_test.cpp:35-47) identity case + seeded rows
    out = {}
    q = np.array([[1, 0], [0, 1]], np.float32)
    out["identity"] = R.attention(q, q, q)
    rows = []
    for i, T in enumerate((1, 2, 3, 16, 33, 257)):
        qq = kvgen.normal(400 + i, (128,))
        k = kvgen.normal(500 + i, (T, 128))
        v = kvgen.normal(600 + i, (T, 128))
        r = R.attention_row(qq, k, v)
        full = R.attention(np.tile(qq, (T, 1)), k, v)
        assert np.array_equal(r, full[0]), "composed row must equal TensorOps::attention"
        rows.append(r)
    out["rows"] = np.stack(rows)
    out["softmax"] = R.softmax(np.array([[1, 2], [3, 2]], np.float32))
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


def paged_case(R: Reference, seed, seq_lens, hq, hkv, dim, pt, dtype, permute):
    """Reference decode for a paged cache: tokens of each sequence appended in
    order, q-head h reads kv-head h // (hq // hkv)."""
    B = len(seq_lens)
    bt, num_pages = kvgen.paged_layout(seq_lens, pt, 0, seed + 7 if permute else None)
    tmax = max(seq_lens)
    K = kvgen.normal(seed + 1, (B, tmax, hkv, dim)).astype(dtype)
    V = kvgen.normal(seed + 2, (B, tmax, hkv, dim)).astype(dtype)
    Q = kvgen.normal(seed + 3, (B, hq, dim)).astype(np.float32)
    out = np.zeros((B, hq, dim), np.float32)
    g = hq // hkv
    for s in range(B):
        T = seq_lens[s]
        for h in range(hq):
            kh = h // g
            k = K[s, :T, kh, :].astype(np.float32)
            v = V[s, :T, kh, :].astype(np.float32)
            out[s, h] = R.attention_row(Q[s, h], k, v)
    return dict(seed=seed, seq_lens=np.array(seq_lens, np.int32), hq=hq, hkv=hkv, dim=dim,
                pt=pt, block_table=bt, num_pages=num_pages, out=out,
                input_sha=sha(K, V, Q))


def gen_paged(R: Reference):
    # Llama-3.2-3B attention geometry, one layer, 1024 tokens, fp32, sequential pages
    c1 = paged_case(R, 1000, [1024], 24, 8, 128, 16, np.float32, permute=False)
    np.savez_compressed(os.path.join(HERE, "paged_cfg1.npz"), **c1)
    # fragmented fp16 batch with ragged lengths (incl. 1 token and page-boundary lengths)
    c2 = paged_case(R, 2000, [1, 15, 16, 17, 100, 256, 511, 700], 24, 8, 128, 16, np.float16,
                    permute=True)
    np.savez_compressed(os.path.join(HERE, "paged_fp16.npz"), **c2)
    # GQA group 8 (70B geometry, fewer heads kept: 16 q / 2 kv)
    c3 = paged_case(R, 3000, [33, 300, 64], 16, 2, 128, 16, np.float16, permute=True)
    np.savez_compressed(os.path.join(HERE, "paged_gqa8.npz"), **c3)


def gen_int8_decode(R: Reference):
    """Decode over pages quantised per (page, kv, head) block by the reference."""
    seed, seq_lens, hq, hkv, dim, pt = 4000, [48, 130, 16, 257], 24, 8, 128, 16
    bt, num_pages = kvgen.paged_layout(seq_lens, pt, 0, seed + 7)
    pool = kvgen.normal(seed + 1, (num_pages, 2, hkv, pt, dim)).astype(np.float16)
    out_mask = kvgen.uniform(seed + 5, pool.size).reshape(pool.shape) < 0.01
    pool = (pool.astype(np.float32) * np.where(out_mask, 20.0, 1.0)).astype(np.float16)
    blocks = pool.reshape(-1, pt * dim).astype(np.float32)
    codes = np.empty(blocks.shape, np.int8)
    stats = np.empty((blocks.shape[0], 4), np.float32)
    deq = np.empty(blocks.shape, np.float32)
    for b in range(blocks.shape[0]):
        codes[b], stats[b] = R.compress_int8(blocks[b])
        deq[b] = R.decompress_int8(codes[b], stats[b])
    deq = deq.reshape(num_pages, 2, hkv, pt, dim)
    Q = kvgen.normal(seed + 3, (len(seq_lens), hq, dim))
    out = np.zeros((len(seq_lens), hq, dim), np.float32)
    g = hq // hkv
    for s, T in enumerate(seq_lens):
        for h in range(hq):
            kh = h // g
            pages = bt[s, :(T + pt - 1) // pt]
            k = deq[pages, 0, kh].reshape(-1, dim)[:T]
            v = deq[pages, 1, kh].reshape(-1, dim)[:T]
            out[s, h] = R.attention_row(Q[s, h], k, v)
    np.savez_compressed(os.path.join(HERE, "int8_decode.npz"), seed=seed,
                        seq_lens=np.array(seq_lens, np.int32), hq=hq, hkv=hkv, dim=dim, pt=pt,
                        block_table=bt, num_pages=num_pages, codes_sha=sha(codes),
                        stats=stats, out=out, input_sha=sha(pool, Q))


def gen_lru(R: Reference):
    traces = []
    # tests/kv_test.cpp:11-33: save 0,1,2 (cap 2) then load 0,1,2
    traces.append((np.array([0, 1, 2, 0, 1, 2]), np.array([1, 1, 1, 0, 0, 0]), 2))
    # tests/kv_integration_test.cpp:29-45: 4 appends at cap 2, reload 0
    traces.append((np.array([0, 1, 2, 3, 0]), np.array([1, 1, 1, 1, 0]), 2))
    for i, (n, ids, cap) in enumerate(((300, 10, 4), (500, 40, 16), (400, 8, 1))):
        t = kvgen.randint(700 + i, n, 0, ids - 1)
        o = (kvgen.uniform(800 + i, n) < 0.3).astype(np.uint8)
        traces.append((t, o, cap))
    z = kvgen.zipf_pages(900, 2000, 64)
    traces.append((z, np.zeros(z.size, np.uint8), 16))
    res = {}
    for i, (ids, ops, cap) in enumerate(traces):
        with tempfile.TemporaryDirectory() as d:
            ev, hit = R.lru_replay(ids.astype(np.int32), ops.astype(np.uint8), cap, d)
        res[f"ids{i}"] = ids.astype(np.int32)
        res[f"ops{i}"] = ops.astype(np.uint8)
        res[f"cap{i}"] = np.int64(cap)
        res[f"evicted{i}"] = ev
        res[f"hit{i}"] = hit
    sel_in, sel_out = [], []
    for i in range(20):
        n = 1 + i * 7
        st = kvgen.randint(1000 + i, n, 0, 5 + i).astype(np.uint64)
        sel_in.append(np.pad(st, (0, 134 - n), constant_values=np.iinfo(np.uint64).max))
        sel_out.append(R.lru_select(st))
    res["select_stamps"] = np.stack(sel_in)
    res["select_n"] = np.array([1 + i * 7 for i in range(20)])
    res["select_out"] = np.array(sel_out)
    res["n_traces"] = np.int64(len(traces))
    np.savez_compressed(os.path.join(HERE, "lru.npz"), **res)


def gen_depth(R: Reference):
    rows = []
    lats = [np.array([]), np.array([10.0]), np.array([100.0] * 3), np.array([24.9, 25.1]),
            kvgen.uniform(1100, 40) * 120.0, np.array([50.0] * 20), np.array([37.5, 62.5])]
    for li, lat in enumerate(lats):
        for size, cap in ((0, 4), (1, 4), (2, 4), (4, 4), (3, 8), (0, 1)):
            for md in (1, 2, 4, 8):
                rows.append((li, size, cap, md, R.prefetch_depth(lat, size, cap, md)))
    np.savez_compressed(os.path.join(HERE, "prefetch_depth.npz"),
                        **{f"lat{i}": l for i, l in enumerate(lats)},
                        grid=np.array(rows, np.int64))


def gen_disk(R: Reference):
    """One page persisted by KVManager::save_page (cache/kv_cache.cpp:21-41)."""
    key = np.concatenate([special_floats(), kvgen.normal(1200, (64,))])
    value = kvgen.normal(1201, (40,)) * np.float32(7.0)
    with tempfile.TemporaryDirectory() as d:
        cwd = os.getcwd()
        os.chdir(d)
        try:
            assert R.save_page(5, key, value, "pages") == 0
            name = [f for f in os.listdir(".") if f.endswith("page_5.bin")][0]
            blob = open(name, "rb").read()
            k2, v2 = R.load_page(5, "pages")
        finally:
            os.chdir(cwd)
    np.savez_compressed(os.path.join(HERE, "disk_page.npz"), key=key, value=value,
                        blob=np.frombuffer(blob, np.uint8), key_back=k2, value_back=v2)


def kvcache_gpu_traces():
    """Op traces for KVCacheGPU: (op, a, b) rows as in oracle/kvx_oracle.h,
    with the budget and page size of each trace.  Mostly page-size
    transfers, some half and double size, re-sent page ids, tokens that
    grow, explicit evictions, lookups and a clear now and then."""
    rng = np.random.default_rng(2024)
    traces = []
    for t in range(8):
        page = (131072, 4096, 65536, 131072)[t % 4]
        budget = page * int(rng.integers(3, 14)) + (0 if t % 3 else page // 2)
        ids = int(rng.integers(6, 40))
        token = 1
        ops = []
        for _ in range(int(rng.integers(150, 400))):
            u = rng.random()
            if u < 0.45:
                size = page * (2 if rng.random() < 0.08 else 1) // (2 if rng.random() < 0.15 else 1)
                ops.append((0, int(rng.integers(0, ids)), int(size)))
            elif u < 0.75:
                token += int(rng.integers(1, 50))
                ops.append((1, int(rng.integers(-1, ids + 2)), token if rng.random() < 0.9 else 0))
            elif u < 0.83:
                ops.append((2, 0, 0))
            elif u < 0.98:
                ops.append((4, int(rng.integers(-1, ids + 2)), 0))
            else:
                ops.append((3, 0, 0))
        traces.append((budget, page, np.array(ops, np.int64)))
    return traces


def gen_kvcache_gpu(R: Reference):
    """KVCacheGPU (native-engine/cpp/KVCacheGPU.cpp) replayed by
    oracle/_ref/kvcachegpu_ref: the reference's class compiled unmodified
    against a host-memory stand-in for its four CUDA calls."""
    import subprocess
    exe = os.path.join(ROOT, "oracle", "_ref", "kvcachegpu_ref")
    out = {}
    for i, (budget, page, ops) in enumerate(kvcache_gpu_traces()):
        text = f"{budget} {page}\n" + "".join(f"{o} {a} {b}\n" for o, a, b in ops)
        r = subprocess.run([exe], input=text, capture_output=True, text=True, check=True,
                           env=dict(os.environ, ADAPTIVE_LOG_LEVEL="0"))
        rows = np.array([list(map(int, ln.split())) for ln in r.stdout.split("\n") if ln.strip()], np.int64)
        assert rows.shape == (len(ops), 2)
        out[f"ops{i}"] = ops
        out[f"budget{i}"] = np.int64(budget)
        out[f"page{i}"] = np.int64(page)
        out[f"result{i}"] = rows[:, 0]
        out[f"used{i}"] = rows[:, 1].astype(np.uint64)
    out["n_traces"] = np.int64(len(kvcache_gpu_traces()))
    np.savez_compressed(os.path.join(HERE, "kvcache_gpu.npz"), **out)


def main():
    os.environ.setdefault("ADAPTIVE_LOG_LEVEL", "ERROR")
    # the reference checkout: KVX_REFERENCE_DIR, or the first argument
    if not build_reference(sys.argv[1] if len(sys.argv) > 1 else None):
        raise SystemExit("reference checkout not found: set KVX_REFERENCE_DIR or pass its path")
    R = Reference()
    gens = {"kv_compress": gen_kv_compress, "int8": gen_int8, "attention": gen_attention,
            "paged": gen_paged, "int8_decode": gen_int8_decode, "lru": gen_lru, "depth": gen_depth,
            "disk": gen_disk, "nf4": gen_nf4, "fp16_wrap": gen_fp16_wrap, "evict": gen_evict,
            "kvcache_gpu": gen_kvcache_gpu}
    for name in (sys.argv[1:] or gens):  # e.g. `make_golden.py nf4 fp16_wrap` for one fixture
        gens[name](R)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
