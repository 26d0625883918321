"""GPU parity: every kernel of libadaptive_engine.so against the oracle.

Integer / byte / index results (append, int8 codes + stats, fp16 truncation
codec, LRU victims, frame migration) must be bit-exact.  Attention outputs
must satisfy |gpu - ref| <= ATOL + RTOL * |ref| with the tolerance the
reference comparison is specified at: RTOL = 1e-3, ATOL = 1e-2.
"""
import numpy as np
import pytest

import kvgen
from conftest import golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-2


@pytest.fixture(scope="module")
def kvx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kvx as k
    assert k.lib.kvx_device_check() == 0, "not an sm_100 device"
    return k


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_close(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
    assert err.max() <= 0, f"max excess {err.max():.3e}, max abs err {np.abs(got - want).max():.3e}"


# ---------------------------------------------------------------- append ---

@pytest.mark.parametrize("np_dtype", [np.float32, np.float16])
def test_append_bitexact(kvx, oracle, np_dtype):
    lens = np.array([0, 5, 15, 16, 17, 100, 255, 300], np.int64)
    bt, num_pages = kvgen.paged_layout(lens, 16, 1, seed=77)
    hkv = 8
    pool = kvgen.normal(78, (num_pages, 2, hkv, 16, 128)).astype(np_dtype)
    nk = kvgen.normal(79, (lens.size, hkv, 128)).astype(np_dtype)
    nv = kvgen.normal(80, (lens.size, hkv, 128)).astype(np_dtype)
    pos = lens.astype(np.int32)
    g_pool = dev(pool)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvx.append(g_pool, dev(bt), dev(pos), dev(nk), dev(nv), error_flag=err)
    oracle.append(pool, bt, pos, nk, nv, 16)
    assert np.array_equal(g_pool.cpu().numpy().view(np.uint8), pool.view(np.uint8))
    assert err.item() == 0


@pytest.mark.parametrize("np_dtype", [np.float32, np.float16])
@pytest.mark.parametrize("page_tokens,dim", [(8, 64), (32, 256)])
def test_append_other_page_geometry_bitexact(kvx, oracle, np_dtype, page_tokens, dim):
    """Page sizes and head dims other than 16 x 128 (the element-wise
    kernel) against the oracle's KVManager::save_page per token."""
    lens = np.array([0, 5, 7, 8, 9, 63, 64, 100], np.int64)
    bt, num_pages = kvgen.paged_layout(lens, page_tokens, 1, seed=81)
    hkv = 4
    pool = kvgen.normal(82, (num_pages, 2, hkv, page_tokens, dim)).astype(np_dtype)
    nk = kvgen.normal(83, (lens.size, hkv, dim)).astype(np_dtype)
    nv = kvgen.normal(84, (lens.size, hkv, dim)).astype(np_dtype)
    pos = lens.astype(np.int32)
    g_pool = dev(pool)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvx.append(g_pool, dev(bt), dev(pos), dev(nk), dev(nv), error_flag=err)
    oracle.append(pool, bt, pos, nk, nv, page_tokens)
    assert np.array_equal(g_pool.cpu().numpy().view(np.uint8), pool.view(np.uint8))
    assert err.item() == 0


@pytest.mark.parametrize("np_dtype", [np.float32, np.float16])
@pytest.mark.parametrize("n_new", [1, 5, 16, 17, 100, 256])
def test_append_chunk_bitexact(kvx, oracle, np_dtype, n_new):
    """A chunk of n_new tokens per sequence from ragged start positions
    (page starts, mid-page, page ends) equals n_new single-token appends of
    the oracle (KVManager::save_page per token)."""
    start = np.array([0, 1, 15, 16, 31, 100, 7, 250], np.int64)
    bt, num_pages = kvgen.paged_layout(start, 16, n_new, seed=97 + n_new)
    hkv = 8
    pool = kvgen.normal(98, (num_pages, 2, hkv, 16, 128)).astype(np_dtype)
    nk = kvgen.normal(99, (start.size, n_new, hkv, 128)).astype(np_dtype)
    nv = kvgen.normal(100, (start.size, n_new, hkv, 128)).astype(np_dtype)
    g_pool = dev(pool)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvx.append_chunk(g_pool, dev(bt), dev(start.astype(np.int32)), dev(nk), dev(nv), error_flag=err)
    for t in range(n_new):
        oracle.append(pool, bt, (start + t).astype(np.int32), nk[:, t], nv[:, t], 16)
    assert np.array_equal(g_pool.cpu().numpy().view(np.uint8), pool.view(np.uint8))
    assert err.item() == 0


def test_append_chunk_out_of_range_rows_are_reported_not_written(kvx):
    """Rows past the block table (or of a negative start) are skipped and
    flagged; the rows that fit are written."""
    bt = np.array([[0, 1], [2, -1]], np.int32)
    pool = torch.zeros((3, 2, 1, 16, 128), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows = torch.ones((2, 20, 1, 128), dtype=torch.float16, device="cuda")
    kvx.append_chunk(pool, dev(bt), dev(np.array([20, 10], np.int32)), rows, rows, error_flag=err)
    torch.cuda.synchronize()
    assert err.item() & 2
    # sequence 0: tokens 20..31 land in page 1 (12 rows), 32..39 have no page
    assert int(pool[1, :, 0, 4:].sum().item()) == 2 * 12 * 128 and int(pool[1, :, 0, :4].abs().sum().item()) == 0
    # sequence 1: tokens 10..15 land in page 2, 16..29 have no page
    assert int(pool[2, :, 0, 10:].sum().item()) == 2 * 6 * 128 and int(pool[2, :, 0, :10].abs().sum().item()) == 0
    assert int(pool[0].abs().sum().item()) == 0


def test_append_out_of_range_is_reported_not_written(kvx):
    bt = np.array([[0, 1]], np.int32)
    pool = torch.zeros((2, 2, 1, 16, 128), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ones = torch.ones((1, 1, 128), dtype=torch.float16, device="cuda")
    kvx.append(pool, dev(bt), dev(np.array([32], np.int32)), ones, ones, error_flag=err)
    torch.cuda.synchronize()
    assert err.item() & 2
    assert pool.abs().sum().item() == 0


# ---------------------------------------------------------------- decode ---

def fill_pool_gpu(kvx, g, dtype_np):
    """Append every token of the golden case through the GPU append kernel."""
    B = len(g["seq_lens"])
    tmax = int(g["seq_lens"].max())
    hkv, hq, dim, seed = int(g["hkv"]), int(g["hq"]), int(g["dim"]), int(g["seed"])
    K = kvgen.normal(seed + 1, (B, tmax, hkv, dim)).astype(dtype_np)
    V = kvgen.normal(seed + 2, (B, tmax, hkv, dim)).astype(dtype_np)
    Q = kvgen.normal(seed + 3, (B, hq, dim)).astype(np.float32)
    pool = torch.zeros((int(g["num_pages"]), 2, hkv, 16, dim),
                       dtype=torch.float32 if dtype_np == np.float32 else torch.float16,
                       device="cuda")
    bt = dev(g["block_table"])
    lens = g["seq_lens"]
    Kd, Vd = dev(K), dev(V)
    for t in range(tmax):
        rows = np.nonzero(lens > t)[0]
        r = torch.from_numpy(rows).cuda()
        kvx.append(pool, bt[r].contiguous(), dev(np.full(rows.size, t, np.int32)),
                   Kd[r, t].contiguous(), Vd[r, t].contiguous())
    return pool, K, V, Q


@pytest.mark.parametrize("name,dtype", [("paged_cfg1.npz", np.float32),
                                        ("paged_fp16.npz", np.float16),
                                        ("paged_gqa8.npz", np.float16)])
def test_decode_matches_reference_golden(kvx, oracle, name, dtype):
    g = golden(name)
    pool, K, V, Q = fill_pool_gpu(kvx, g, dtype)
    # cache contents: bit-exact with the oracle's paged append of the same tokens
    ref_pool = np.zeros(tuple(pool.shape), dtype)
    lens = g["seq_lens"]
    for t in range(int(lens.max())):
        rows = np.nonzero(lens > t)[0]
        oracle.append(ref_pool, g["block_table"][rows], np.full(rows.size, t, np.int32),
                      K[rows, t], V[rows, t], 16)
    assert np.array_equal(pool.cpu().numpy().view(np.uint8), ref_pool.view(np.uint8))
    for io in (torch.float32, torch.float16):
        q = dev(Q).to(io)
        out = kvx.decode(pool, dev(g["block_table"]), dev(g["seq_lens"]), q)
        torch.cuda.synchronize()
        want = g["out"] if io == torch.float32 else g["out"].astype(np.float16).astype(np.float32)
        assert_close(out.float().cpu().numpy(), want)


def test_decode_empty_and_single_token(kvx, oracle):
    lens = np.array([0, 1, 0, 2], np.int64)
    bt, num_pages = kvgen.paged_layout(np.maximum(lens, 1), 16, 0, seed=5)
    pool = kvgen.normal(6, (num_pages, 2, 2, 16, 128)).astype(np.float16)
    q = kvgen.normal(7, (4, 6, 128))
    out = kvx.decode(dev(pool), dev(bt), dev(lens.astype(np.int32)), dev(q)).cpu().numpy()
    ref = oracle.paged_decode(pool, bt, lens.astype(np.int32), q)
    assert np.all(out[0] == 0) and np.all(out[2] == 0)
    assert_close(out, ref)


def config2_layer(seed=2024, batch=32, lo=512, hi=8192):
    """One layer of the batched fragmented decode workload: fp16 K/V N(0,1),
    context lengths U[lo, hi], physical pages a seeded permutation."""
    lens = kvgen.randint(seed, batch, lo, hi)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed + 1)
    pool = kvgen.normal(seed + 2, (num_pages, 2, 8, 16, 128)).astype(np.float16)
    q = kvgen.normal(seed + 3, (batch, 24, 128))
    return lens.astype(np.int32), bt, pool, q


def test_decode_config2_layer_against_oracle(kvx, oracle):
    lens, bt, pool, q = config2_layer()
    out = kvx.decode(dev(pool), dev(bt), dev(lens), dev(q)).cpu().numpy()
    ref = oracle.paged_decode(pool, bt, lens, q)
    assert_close(out, ref)


@pytest.mark.parametrize("chunk", ["4", "8", "64"])
def test_decode_split_invariance(kvx, monkeypatch, chunk):
    """Size-independent property: the result does not depend on how the
    context is split across CTAs (flash-decoding combine)."""
    lens, bt, pool, q = config2_layer(seed=99, batch=8, lo=1, hi=3000)
    base = kvx.decode(dev(pool), dev(bt), dev(lens), dev(q)).cpu().numpy()
    monkeypatch.setenv("KVX_DECODE_CHUNK", chunk)
    other = kvx.decode(dev(pool), dev(bt), dev(lens), dev(q)).cpu().numpy()
    assert np.abs(base - other).max() < 1e-4


def test_decode_many_ragged_sequences(kvx, oracle):
    """Many short, empty and long sequences in one launch; the workspace is
    reused, so the split counters must be back at zero after each launch."""
    lens = kvgen.randint(81, 300, 0, 2000)
    lens[::17] = 0
    lens[5] = 16
    lens[6] = 1
    bt, num_pages = kvgen.paged_layout(np.maximum(lens, 1), 16, 0, seed=82)
    pool = kvgen.normal(83, (num_pages, 2, 8, 16, 128)).astype(np.float16)
    q = kvgen.normal(84, (lens.size, 24, 128))
    ws = kvx.decode_workspace(lens.size, 24, bt.shape[1])
    for _ in range(2):  # counters must come back to zero between launches
        out = kvx.decode(dev(pool), dev(bt), dev(lens.astype(np.int32)), dev(q), workspace=ws)
    out = out.cpu().numpy()
    ref = oracle.paged_decode(pool, bt, lens.astype(np.int32), q)
    assert_close(out, ref)
    assert np.all(out[lens == 0] == 0)


@pytest.mark.parametrize("np_dtype", [np.float16, np.float32])
def test_append_decode_fused_matches_append_then_decode(kvx, oracle, np_dtype):
    lens = kvgen.randint(41, 12, 0, 900)
    lens[0], lens[1], lens[2] = 0, 15, 16  # first token, page end, page start
    bt, num_pages = kvgen.paged_layout(lens, 16, 1, seed=42)
    pool = kvgen.normal(43, (num_pages, 2, 8, 16, 128)).astype(np_dtype)
    nk = kvgen.normal(44, (lens.size, 8, 128)).astype(np_dtype)
    nv = kvgen.normal(45, (lens.size, 8, 128)).astype(np_dtype)
    q = kvgen.normal(46, (lens.size, 24, 128))
    pos = lens.astype(np.int32)
    g_pool = dev(pool)
    ws = kvx.decode_workspace(lens.size, 24, bt.shape[1])
    for rep in range(2):  # second call reuses the workspace: counters must be back at zero
        out = kvx.append_decode(g_pool, dev(bt), dev(pos), dev(nk), dev(nv), dev(q), workspace=ws)
        torch.cuda.synchronize()
    ref_pool = pool.copy()
    oracle.append(ref_pool, bt, pos, nk, nv, 16)
    assert np.array_equal(g_pool.cpu().numpy().view(np.uint8), ref_pool.view(np.uint8))
    ref = oracle.paged_decode(ref_pool, bt, pos + 1, q)
    assert_close(out.cpu().numpy(), ref)
    assert int(ws[-lens.size * 24 * 4:].view(torch.int32).abs().sum().item()) == 0


def test_compress_int8_fp16_nan_and_inf_blocks(kvx, oracle):
    data = kvgen.normal(61, (6, 2048)).astype(np.float16)
    bits = data.view(np.uint16)
    bits[0, 0] = 0x7E00          # quiet NaN first
    bits[1, 0] = 0x7C01          # signaling NaN first (payload kept, quieted)
    bits[2, 100] = 0xFE00        # NaN later (ignored)
    bits[3, 0] = 0x7C00          # +inf first
    bits[4, 7] = 0xFC00          # -inf inside
    bits[5, :] = 0x0000
    bits[5, 3] = 0x8000          # -0 after +0: min/max keep the first zero
    codes, stats = kvx.compress_int8(dev(data))
    rc, rs = oracle.compress_int8_blocks(data, 2048)
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    dec = kvx.decompress_int8(codes, stats).cpu().numpy()
    assert np.array_equal(dec.view(np.uint32), oracle.decompress_int8_blocks(rc, rs, 2048).view(np.uint32))


@pytest.mark.parametrize("hkv,hq", [(8, 8), (8, 24), (2, 16), (1, 16), (4, 8)])
def test_decode_tensor_core_path_matches_oracle(kvx, oracle, monkeypatch, hkv, hq):
    """fp16 pools run on the tensor-core kernel (GQA group as the mma M
    dimension, up to 16); the SIMT kernel must agree with it and both with
    the oracle."""
    lens = kvgen.randint(70 + hq, 6, 1, 1500)
    lens[0] = 1
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=71)
    pool = kvgen.normal(72, (num_pages, 2, hkv, 16, 128)).astype(np.float16)
    q = kvgen.normal(73, (lens.size, hq, 128))
    args = (dev(pool), dev(bt), dev(lens.astype(np.int32)), dev(q))
    tc = kvx.decode(*args).cpu().numpy()
    monkeypatch.setenv("KVX_DECODE_SIMT", "1")
    simt = kvx.decode(*args).cpu().numpy()
    ref = oracle.paged_decode(pool, bt, lens.astype(np.int32), q)
    assert_close(tc, ref)
    assert_close(simt, ref)


@pytest.mark.parametrize("hkv,hq", [(8, 24), (1, 12), (2, 32)])
def test_decode_outlier_keys_keep_fp32_query_accuracy(kvx, oracle, hkv, hq):
    """Keys with outlier channels (1% of entries x20, as K caches have):
    the query must not be rounded to fp16 on its way into the mma."""
    lens = kvgen.randint(110 + hq, 6, 1, 900)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=111)
    pool = kvgen.normal(112, (num_pages, 2, hkv, 16, 128))
    pool[kvgen.uniform(113, pool.size).reshape(pool.shape) < 0.01] *= 20
    pool = pool.astype(np.float16)
    q = kvgen.normal(114, (lens.size, hq, 128)) * 2.0
    out = kvx.decode(dev(pool), dev(bt), dev(lens.astype(np.int32)), dev(q)).cpu().numpy()
    assert_close(out, oracle.paged_decode(pool, bt, lens.astype(np.int32), q))


@pytest.mark.parametrize("hq", [24, 64])
def test_decode_dominant_scores_fp16_weights(kvx, oracle, hq):
    """A few keys aligned with the query take almost all the softmax mass
    (scores 12, 11.5, 11 against ~N(0,1) for the rest: weights 1, 0.61, 0.37
    and ~1e-5 each), over values with 1% outliers x20.  The fp16 pool's
    kernel rounds the softmax weights to fp16 for the P.V mma (relative error
    2^-11 per weight); the output must still meet the tolerance."""
    hkv = 8
    G = hq // hkv
    lens = kvgen.randint(140 + hq, 8, 300, 4000)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=141)
    pool = kvgen.normal(142, (num_pages, 2, hkv, 16, 128))
    vals = pool[:, 1]
    vals[kvgen.uniform(143, vals.size).reshape(vals.shape) < 0.01] *= 20
    q = kvgen.normal(144, (lens.size, hq, 128))
    pick = kvgen.uniform(145, lens.size * hkv * 3).reshape(lens.size, hkv, 3)
    for s in range(lens.size):
        for h in range(hkv):
            qd = q[s, h * G]  # the group's first q-head sets the direction
            unit = qd / np.linalg.norm(qd)
            for j, a in enumerate((12.0, 11.5, 11.0)):
                t = int(pick[s, h, j] * lens[s])
                page = bt[s, t // 16]
                # score = q . k / sqrt(128) = a for the direction head
                pool[page, 0, h, t % 16] = a * np.sqrt(128.0) / np.linalg.norm(qd) * unit
    pool = pool.astype(np.float16)
    out = kvx.decode(dev(pool), dev(bt), dev(lens.astype(np.int32)), dev(q)).cpu().numpy()
    assert_close(out, oracle.paged_decode(pool, bt, lens.astype(np.int32), q))


def test_decode_gqa_grouping_matches_mha_expansion(kvx):
    """Property: GQA with group G equals MHA on a pool whose kv heads are
    repeated G times."""
    lens = np.array([40, 333], np.int32)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=11)
    pool = kvgen.normal(12, (num_pages, 2, 2, 16, 128)).astype(np.float16)
    q = kvgen.normal(13, (2, 6, 128))
    gqa = kvx.decode(dev(pool), dev(bt), dev(lens), dev(q)).cpu().numpy()
    mha_pool = np.repeat(pool, 3, axis=2)
    mha = kvx.decode(dev(mha_pool), dev(bt), dev(lens), dev(q)).cpu().numpy()
    # the pools differ in size, so the work is split differently: fp32
    # summation order differs, nothing else
    assert np.abs(gqa - mha).max() < 2e-4


# ------------------------------------------------------------------ int8 ---

def test_compress_int8_golden_cases(kvx):
    g = golden("int8.npz")
    off = 0
    for i, n in enumerate(g["lens"]):
        data = dev(g["data"][off:off + n])
        codes, stats = kvx.compress_int8(data, block_elems=int(n))
        torch.cuda.synchronize()
        assert np.array_equal(codes.cpu().numpy(), g["codes"][off:off + n]), g["names"][i]
        assert np.array_equal(stats.cpu().numpy().view(np.uint32).ravel(),
                              g["stats"][i].view(np.uint32)), g["names"][i]
        dec = kvx.decompress_int8(codes, stats, block_elems=int(n)).cpu().numpy()  # any size
        assert np.array_equal(dec.view(np.uint32), g["dec"][off:off + n].view(np.uint32))
        off += n


@pytest.mark.parametrize("np_dtype", [np.float16, np.float32])
def test_compress_int8_pages_bitexact(kvx, oracle, np_dtype):
    nb = 3000
    data = kvgen.normal(31, (nb, 2048))
    data[kvgen.uniform(32, data.size).reshape(data.shape) < 0.01] *= 20
    data[5, :] = 0.0
    data[6, ::2] = -0.0
    data[7, :] = 1.5
    data = data.astype(np_dtype)
    codes, stats = kvx.compress_int8(dev(data))
    rc, rs = oracle.compress_int8_blocks(data, 2048)
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    dec = kvx.decompress_int8(codes, stats).cpu().numpy()
    assert np.array_equal(dec.view(np.uint32), oracle.decompress_int8_blocks(rc, rs, 2048).view(np.uint32))


@pytest.mark.parametrize("np_dtype", [np.float16, np.float32])
def test_compress_int8_half_ties_bitexact(kvx, oracle, np_dtype):
    """Quotients (x - min) / scale on and next to k + 1/2, where a
    reciprocal-multiply could round differently from the division."""
    rows = []
    k = np.arange(2048) % 255
    rows.append(np.where(k == 0, 0.0, k + 0.5))                   # scale 1: exact ties
    rows[-1][1] = 255.0
    for span in (1.0, 3.0, 0.1, 7.0, 1e-3, 6e4):
        t = (np.arange(2048) % 256 + 0.5) / 255.0 * span         # ties for a non-dyadic scale
        t[0], t[1] = 0.0, span
        rows.append(t)
        for ulps in (-2, -1, 1, 2):
            r = t.astype(np_dtype)
            bits = r.view(np.uint16 if np_dtype == np.float16 else np.uint32).copy()
            bits[2:] = bits[2:] + ulps * (bits[2:] > 0)
            rows.append(bits.view(np_dtype).astype(np.float64))
    data = np.stack(rows).astype(np_dtype)
    codes, stats = kvx.compress_int8(dev(data))
    rc, rs = oracle.compress_int8_blocks(data, 2048)
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(codes.cpu().numpy(), rc)
    dec16 = kvx.decompress_int8(codes, stats, dtype=torch.float16).cpu().numpy()
    want = oracle.decompress_int8_blocks(rc, rs, 2048).astype(np.float16)
    assert np.array_equal(dec16.view(np.uint16), want.view(np.uint16))


def test_nf4_golden_cases(kvx):
    """KVCompressionEngine NF4 (native-engine/cpp/KVCompressionEngine.cpp:124-180) on the
    reference's own outputs: edge blocks of 1..2048 elements (odd ones too)."""
    g = golden("nf4.npz")
    off = coff = 0
    for i, n in enumerate(g["lens"]):
        n = int(n)
        cb = (n + 1) // 2
        codes, stats = kvx.compress_nf4(dev(g["data"][off:off + n]), block_elems=n)
        torch.cuda.synchronize()
        assert np.array_equal(codes.cpu().numpy(), g["codes"][coff:coff + cb]), g["names"][i]
        assert np.array_equal(stats.cpu().numpy().view(np.uint32).ravel(), g["stats"][i].view(np.uint32)), g["names"][i]
        dec = kvx.decompress_nf4(codes, stats, block_elems=n).cpu().numpy()
        assert np.array_equal(dec.view(np.uint32), g["dec"][off:off + n].view(np.uint32)), g["names"][i]
        off += n
        coff += cb


@pytest.mark.parametrize("np_dtype", [np.float16, np.float32])
def test_nf4_pages_bitexact(kvx, oracle, np_dtype):
    nb = 3000
    data = kvgen.normal(61, (nb, 2048))
    data[kvgen.uniform(62, data.size).reshape(data.shape) < 0.01] *= 20
    data[5, :] = 0.0
    data[6, ::2] = -0.0
    data[7, :] = 1.5
    ties = ((np.arange(2048) % 16) + 0.5) / 15.0 * 3.0  # quotients on k + 1/2
    ties[0], ties[1] = 0.0, 3.0
    data[8] = ties
    data[9] = np.nextafter(ties.astype(np_dtype), np_dtype(np.inf)).astype(np.float64)
    data[10, 100] = np.nan
    data = data.astype(np_dtype)
    codes, stats = kvx.compress_nf4(dev(data))
    rc, rs = oracle.compress_nf4_blocks(data, 2048)
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(codes.cpu().numpy(), rc)
    dec = kvx.decompress_nf4(codes, stats).cpu().numpy()
    want = oracle.decompress_nf4_blocks(rc, rs, 2048)
    assert np.array_equal(dec.view(np.uint32), want.view(np.uint32))
    dec16 = kvx.decompress_nf4(codes, stats, dtype=torch.float16).cpu().numpy()
    assert np.array_equal(dec16.view(np.uint16), want.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("block_elems", [17, 2047, 4096])
def test_nf4_other_block_sizes(kvx, oracle, block_elems):
    data = (kvgen.normal(63, (40, block_elems)) * 3).astype(np.float32)
    codes, stats = kvx.compress_nf4(dev(data), block_elems=block_elems)
    rc, rs = oracle.compress_nf4_blocks(data, block_elems)
    assert np.array_equal(codes.cpu().numpy(), rc)
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    dec = kvx.decompress_nf4(codes, stats, block_elems=block_elems).cpu().numpy()
    assert np.array_equal(dec.view(np.uint32), oracle.decompress_nf4_blocks(rc, rs, block_elems).view(np.uint32))


def test_fp16_wrap_codec_bitexact(kvx):
    """KVCompressionEngine FP16 (native-engine/cpp/KVCompressionEngine.cpp:36-80), the
    exponent-wrapping conversion, on the reference's own outputs."""
    g = golden("fp16_wrap.npz")
    enc = kvx.fp16_wrap_encode(dev(g["x"])).cpu().numpy().view(np.uint16)
    assert np.array_equal(enc, g["enc"])
    h = torch.arange(65536, dtype=torch.int32).to(torch.int16).cuda()
    dec = kvx.fp16_wrap_decode(h).cpu().numpy()
    assert np.array_equal(dec.view(np.uint32), g["dec_bits"])
    odd = kvx.fp16_wrap_encode(dev(g["x"])[1:]).cpu().numpy().view(np.uint16)  # unaligned: scalar path
    assert np.array_equal(odd, g["enc"][1:])
    # decode: misaligned start, and aligned starts with a partial last tile
    for sl in (slice(3, None), slice(8, None), slice(None, -5), slice(8, 8 + 2048 + 1)):
        d = kvx.fp16_wrap_decode(h[sl]).cpu().numpy()
        assert np.array_equal(d.view(np.uint32), g["dec_bits"][sl]), sl


def test_compress_roundtrip_error_bound(kvx):
    """Property at scale: |x - dequant(quant(x))| <= scale/2 (+1 ulp) per block."""
    nb = 65536  # 128 Mi elements = 256 MiB fp16, larger than L2
    x = torch.randn((nb, 2048), dtype=torch.float16, device="cuda")
    codes, stats = kvx.compress_int8(x)
    back = kvx.decompress_int8(codes, stats).view(nb, 2048)
    err = (back - x.float()).abs().amax(dim=1)
    assert bool((err <= stats[:, 2] * 0.5001 + 1e-6).all())


def test_int8_decode_matches_reference_golden(kvx, oracle):
    g = golden("int8_decode.npz")
    seed, pt, dim, hkv = int(g["seed"]), int(g["pt"]), int(g["dim"]), int(g["hkv"])
    num_pages = int(g["num_pages"])
    pool = kvgen.normal(seed + 1, (num_pages, 2, hkv, pt, dim)).astype(np.float16)
    mask = kvgen.uniform(seed + 5, pool.size).reshape(pool.shape) < 0.01
    pool = (pool.astype(np.float32) * np.where(mask, 20.0, 1.0)).astype(np.float16)
    Q = kvgen.normal(seed + 3, (len(g["seq_lens"]), int(g["hq"]), dim))
    codes, stats = kvx.compress_int8(dev(pool))
    assert np.array_equal(stats.cpu().numpy().view(np.uint32), g["stats"].view(np.uint32))
    cpool = codes.view(num_pages, 2, hkv, pt, dim)
    out = kvx.decode(cpool, dev(g["block_table"]), dev(g["seq_lens"]), dev(Q), stats=stats)
    assert_close(out.cpu().numpy(), g["out"])


@pytest.mark.parametrize("hkv,hq,io", [(8, 24, "f32"), (8, 24, "f16"), (2, 16, "f32"), (1, 12, "f32"),
                                       (4, 4, "f32")])
def test_int8_decode_tensor_core_path_matches_oracle(kvx, oracle, monkeypatch, hkv, hq, io):
    """int8 pools run on the tensor-core kernel (codes widened in registers,
    scale / zero point folded into scores and weights); the SIMT kernel
    must agree with it and both with the oracle's dequantise-then-attend."""
    lens = kvgen.randint(90 + hq, 7, 1, 1200)
    lens[0], lens[1] = 1, 16
    bt, num_pages = kvgen.paged_layout(lens, 16, 5, seed=91)
    pool = kvgen.normal(92, (num_pages, 2, hkv, 16, 128))
    pool[kvgen.uniform(93, pool.size).reshape(pool.shape) < 0.01] *= 20
    pool[0] += 3.0  # blocks far from zero: the zero-point terms matter
    pool = pool.astype(np.float16)
    codes, stats = kvx.compress_int8(dev(pool))
    cpool = codes.view(num_pages, 2, hkv, 16, 128)
    q = kvgen.normal(94, (lens.size, hq, 128))
    qd = dev(q) if io == "f32" else dev(q.astype(np.float16))
    args = (cpool, dev(bt), dev(lens.astype(np.int32)), qd)
    tc = kvx.decode(*args, stats=stats).float().cpu().numpy()
    monkeypatch.setenv("KVX_DECODE_SIMT", "1")
    simt = kvx.decode(*args, stats=stats).float().cpu().numpy()
    qref = q if io == "f32" else q.astype(np.float16).astype(np.float32)
    ref = oracle.paged_decode(codes.cpu().numpy().reshape(cpool.shape), bt, lens.astype(np.int32), qref,
                              stats=stats.cpu().numpy().reshape(num_pages, 2, hkv, 4))
    assert_close(tc, ref)
    assert_close(simt, ref)


@pytest.mark.parametrize("hq", [24, 64])
def test_int8_decode_long_contexts(kvx, oracle, hq):
    """int8 pools with long contexts: 256-page CTAs (one split for 4,096
    tokens, five folded for 20,000) match the oracle's dequantise-then-attend."""
    hkv = 8
    lens = np.array([4096, 20000, 777, 16, 4095], np.int32)
    bt, num_pages = kvgen.paged_layout(lens, 16, 1, seed=191)
    pool = kvgen.normal(192, (num_pages, 2, hkv, 16, 128))
    pool[kvgen.uniform(193, pool.size).reshape(pool.shape) < 0.01] *= 20
    pool = pool.astype(np.float16)
    codes, stats = kvx.compress_int8(dev(pool))
    cpool = codes.view(num_pages, 2, hkv, 16, 128)
    q = kvgen.normal(194, (lens.size, hq, 128))
    got = kvx.decode(cpool, dev(bt), dev(lens), dev(q), stats=stats).float().cpu().numpy()
    ref = oracle.paged_decode(codes.cpu().numpy().reshape(cpool.shape), bt, lens, q,
                              stats=stats.cpu().numpy().reshape(num_pages, 2, hkv, 4))
    assert_close(got, ref)


@pytest.mark.parametrize("qscale", [20.0, 200.0])
def test_int8_decode_query_outlier_channels(kvx, oracle, qscale):
    """Queries with outlier channels (two dims x20 / x200) over int8 pages
    with outlier keys and values stay within the attention tolerance: q
    enters the mma as fp16 hi + lo, each element with its own exponent (q
    as 16-bit integers per row, one scale for all dims, misses it at x200)."""
    hkv, hq = 8, 24
    lens = kvgen.randint(130, 6, 200, 2500)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=131)
    pool = kvgen.normal(132, (num_pages, 2, hkv, 16, 128))
    pool[kvgen.uniform(133, pool.size).reshape(pool.shape) < 0.01] *= 20
    pool = pool.astype(np.float16)
    codes, stats = kvx.compress_int8(dev(pool))
    cpool = codes.view(num_pages, 2, hkv, 16, 128)
    q = kvgen.normal(134, (lens.size, hq, 128))
    q[:, :, 17] *= qscale
    q[:, :, 90] *= -qscale
    out = kvx.decode(cpool, dev(bt), dev(lens.astype(np.int32)), dev(q), stats=stats).cpu().numpy()
    ref = oracle.paged_decode(codes.cpu().numpy().reshape(cpool.shape), bt, lens.astype(np.int32), q,
                              stats=stats.cpu().numpy().reshape(num_pages, 2, hkv, 4))
    assert_close(out, ref)


def test_attention_dense_and_softmax_match_reference_rows(kvx, oracle):
    """kvx.attention_dense / kvx.softmax_rows (the cuda_attention and
    cuda_softmax kernels) against TensorOps::attention rows of the golden
    fixture and the restatement's row attention."""
    g = golden("attention.npz")
    for i, T in enumerate((1, 2, 3, 16, 33, 257)):
        q = kvgen.normal(400 + i, (128,))
        k = kvgen.normal(500 + i, (T, 128))
        v = kvgen.normal(600 + i, (T, 128))
        out = kvx.attention_dense(dev(q[None, :].copy()), dev(k), dev(v)).cpu().numpy()[0]
        assert_close(out, g["rows"][i])
    x = kvgen.normal(77, (5, 300)) * 4
    sm = kvx.softmax_rows(dev(x)).cpu().numpy()
    e = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    assert np.abs(sm - e / e.sum(axis=1, keepdims=True)).max() < 1e-6


@pytest.mark.parametrize("dim,offset", [(128, 1), (64, 0), (96, 0), (256, 0), (1000, 0)])
def test_attention_dense_cuda_core_paths_match_fp64(kvx, dim, offset):
    """The CUDA-core kernels of the dense attention: head dim 128 whose Q /
    out rows are not 16-byte aligned (attention_dense128_kernel) and other
    head dims up to 1024 (attention_dense_kernel), against float64."""
    seq_q, seq_k = 37, 300
    g = torch.Generator(device="cuda")
    g.manual_seed(dim * 13 + offset)
    qbuf = torch.randn(seq_q * dim + offset, generator=g, device="cuda")
    q = qbuf[offset:].view(seq_q, dim)  # offset 1: rows start 4 bytes past a 16-byte boundary
    k = torch.randn((seq_k, dim), generator=g, device="cuda")
    v = torch.randn((seq_k, dim), generator=g, device="cuda")
    obuf = torch.zeros(seq_q * dim + offset, device="cuda")
    out = obuf[offset:].view(seq_q, dim)
    kvx.attention_dense(q, k, v, out=out)
    s = (q.double() @ k.double().T) / np.sqrt(float(dim))
    ref = torch.softmax(s, dim=1) @ v.double()
    assert_close(out.cpu().numpy(), ref.cpu().numpy())
    assert obuf[:offset].abs().sum().item() == 0


@pytest.mark.parametrize("seq_q,seq_k,mag", [(1024, 1024, 1.0), (1000, 777, 1.0), (1, 1, 1.0), (17, 65, 1.0),
                                             (300, 2049, 1.0), (64, 500, 1e5), (128, 300, 1e-3),
                                             (4096, 4096, 1.0), (20000, 300, 1.0), (128, 40001, 1.0)])
def test_attention_dense_tensor_core_matches_fp64(kvx, seq_q, seq_k, mag):
    """The head-dim-128 dense attention (tensor cores, 3xTF32 products)
    over ragged query / key counts (partial key tiles, rows past the last
    query), key tiles split over CTAs one each (1024 x 1024), several per
    CTA (4096 x 4096: 4 splits of 16 tiles; 128 x 40001: 126 splits of 5,
    the last with one tile of one key) or all in one CTA that writes the
    output itself (20000 x 300: more row tiles than SMs), and magnitudes
    far outside fp16's range, against
    softmax(Q K^T / sqrt(128)) V in float64 (TensorOps::attention,
    runtime/tensor_ops.cpp:179-219)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seq_q * 7 + seq_k)
    q = torch.randn((seq_q, 128), generator=g, device="cuda") * mag
    k = torch.randn((seq_k, 128), generator=g, device="cuda") * mag
    v = torch.randn((seq_k, 128), generator=g, device="cuda")
    v[torch.rand(v.shape, generator=g, device="cuda") < 0.01] *= 20
    out = kvx.attention_dense(q, k, v)
    s = (q.double() @ k.double().T) / np.sqrt(128.0)
    ref = torch.softmax(s, dim=1) @ v.double()
    assert_close(out.cpu().numpy(), ref.cpu().numpy())


# ------------------------------------------------------- fp16 trunc codec ---

def test_f16_trunc_codec_bitexact(kvx):
    g = golden("kv_compress.npz")
    enc = kvx.f32_to_f16_trunc(dev(g["x"])).cpu().numpy().view(np.uint16)
    assert np.array_equal(enc, g["enc"])
    allh = dev(np.arange(65536, dtype=np.uint16).view(np.int16))
    dec = kvx.f16_trunc_to_f32(allh).cpu().numpy().view(np.uint32)
    assert np.array_equal(dec, g["dec_bits"])
    # misaligned views take the element-wise path, same bits
    enc_odd = kvx.f32_to_f16_trunc(dev(g["x"])[1:]).cpu().numpy().view(np.uint16)
    assert np.array_equal(enc_odd, g["enc"][1:])
    dec_odd = kvx.f16_trunc_to_f32(allh[3:]).cpu().numpy().view(np.uint32)
    assert np.array_equal(dec_odd, g["dec_bits"][3:])
    # 16-byte aligned starts whose length is not a whole number of 2048-element
    # tiles: the tile kernel takes the prefix, the element-wise kernel the rest
    for sl in (slice(8, None), slice(None, -5), slice(8, 8 + 2048 + 1)):
        dec_tail = kvx.f16_trunc_to_f32(allh[sl]).cpu().numpy().view(np.uint32)
        assert np.array_equal(dec_tail, g["dec_bits"][sl]), sl


# ------------------------------------------------------------- eviction ---

def test_lru_select_matches_reference(kvx, oracle):
    g = golden("lru.npz")
    for st, n, want in zip(g["select_stamps"], g["select_n"], g["select_out"]):
        v = kvx.lru_select(dev(st[:n].copy())).item()
        assert v == want
    big = kvgen.randint(55, 1_000_001, 0, 5000).astype(np.uint64)
    big[::7] = np.iinfo(np.uint64).max
    assert kvx.lru_select(dev(big)).item() == oracle.lru_select(big)
    allmax = np.full(10, np.iinfo(np.uint64).max, np.uint64)
    assert kvx.lru_select(dev(allmax)).item() == -1


# ------------------------------------------------------------- migration ---

def test_migrate_frames_roundtrip(kvx):
    frame = 64 * 1024
    nf_dev, nf_host = 64, 96
    devbuf = torch.randint(-128, 127, (nf_dev * frame,), dtype=torch.int8, device="cuda")
    host = torch.zeros(nf_host * frame, dtype=torch.int8).pin_memory()
    dsel = kvgen.permutation(3, nf_dev)[:40].astype(np.int32)
    hsel = kvgen.permutation(4, nf_host)[:40].astype(np.int32)
    kvx.migrate_frames(devbuf, nf_dev, host, nf_host, dev(dsel), dev(hsel), frame, 0, ctas=8)
    torch.cuda.synchronize()
    d = devbuf.cpu().numpy().reshape(nf_dev, frame)
    h = host.numpy().reshape(nf_host, frame)
    assert np.array_equal(h[hsel], d[dsel])
    back = torch.zeros_like(devbuf)
    kvx.migrate_frames(back, nf_dev, host, nf_host, dev(dsel), dev(hsel), frame, 1, ctas=8)
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy().reshape(nf_dev, frame)[dsel], d[dsel])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    kvx.migrate_frames(back, nf_dev, host, nf_host, dev(np.array([nf_dev], np.int32)),
                       dev(np.array([0], np.int32)), frame, 1, error_flag=err)
    torch.cuda.synchronize()
    assert err.item() & 2


def test_eviction_policies_on_device_match_reference(kvx, oracle):
    """kvx_evict_select / _composite against the reference's selectPageToEvict
    (golden), for 12 page sets of up to 400 pages, and against the oracle on a
    large set (1,000,000 pages, single-CTA scan)."""
    from oracle import EVICT_METRICS
    g = golden("evict.npz")
    for c in range(12):
        m = g[f"pages{c}"].view(EVICT_METRICS)
        hist, hl = g[f"hist{c}"], g[f"hist_len{c}"]
        pred = np.array([oracle.predict_next_access(hist[i, :hl[i]]) for i in range(m.size)], np.float32)
        pages = dev(m.view(np.uint8))
        for pol in (0, 1, 2, 3):
            got = kvx.evict_select(pol, pages, 0.95, dev(pred) if pol == 3 else None).item()
            assert got == int(g[f"sel{c}_{pol}"]), (c, pol)
        got = kvx.evict_select_composite([0, 1, 2], g[f"composite_w{c}"], pages).item()
        assert got == int(g[f"composite{c}"]), c
    n = 1_000_000
    m = np.zeros(n, EVICT_METRICS)
    m["last_access_token"] = kvgen.randint(71, n, 1, 10 ** 9).astype(np.uint64)
    m["average_attention"] = kvgen.uniform(72, n).astype(np.float32)
    m["average_attention"][[17, 500_000]] = -0.25  # the best score twice: the lower index wins
    m["page_id"] = np.arange(n) + 7
    pages = dev(m.view(np.uint8))
    for pol in (0, 1, 2):
        assert kvx.evict_select(pol, pages).item() == oracle.evict_select(pol, m), pol
    assert kvx.evict_select(2, pages).item() == 17 + 7
    assert kvx.evict_select(0, pages[:0]).item() == -1


def _page_mass_ref(pool_f, bt, lens, q, hkv):
    """float64 softmax per (sequence, q-head), summed per page, mean over q-heads."""
    B, hq, _ = q.shape
    G = hq // hkv
    mp = bt.shape[1]
    mass = np.zeros((B, mp))
    for s in range(B):
        T = int(lens[s])
        if T == 0:
            continue
        npg = (T + 15) // 16
        K = pool_f[bt[s, :npg], 0].transpose(1, 0, 2, 3).reshape(hkv, npg * 16, 128)[:, :T]
        for h in range(hq):
            sc = K[h // G].astype(np.float64) @ q[s, h].astype(np.float64) / np.sqrt(128.0)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            mass[s, :npg] += np.add.reduceat(p, np.arange(0, T, 16)) / hq
    return mass


@pytest.mark.parametrize("kind,hkv,hq", [("f16", 8, 24), ("f16", 1, 12), ("i8", 8, 24)])
def test_decode_attention_mass(kvx, monkeypatch, kind, hkv, hq):
    """kvx_decode_attn: same output as kvx_decode, each page's softmax mass
    (mean over q-heads) as a float64 softmax gives it, masses summing to 1,
    independent of the split."""
    lens = kvgen.randint(130 + hq, 6, 1, 1500)
    lens[0] = 1
    bt, num_pages = kvgen.paged_layout(lens, 16, 3, seed=131)
    pool = kvgen.normal(132, (num_pages, 2, hkv, 16, 128)).astype(np.float16)
    q = kvgen.normal(133, (lens.size, hq, 128))
    args = [dev(bt), dev(lens.astype(np.int32)), dev(q)]
    if kind == "f16":
        gpool, stats, pool_f = dev(pool), None, pool.astype(np.float32)
    else:
        codes, stats = kvx.compress_int8(dev(pool))
        gpool = codes.view(num_pages, 2, hkv, 16, 128)
        pool_f = kvx.decompress_int8(codes, stats).view(num_pages, 2, hkv, 16, 128).cpu().numpy()
    out, mass = kvx.decode_attn(gpool, *args, stats=stats)
    plain = kvx.decode(gpool, *args, stats=stats)
    assert torch.equal(out, plain)
    mass = mass.cpu().numpy()
    ref = _page_mass_ref(pool_f, bt, lens, q, hkv)
    assert np.abs(mass - ref).max() < 2e-4
    assert np.abs(mass.sum(1) - 1.0).max() < 1e-4
    monkeypatch.setenv("KVX_DECODE_CHUNK", "4")
    _, mass4 = kvx.decode_attn(gpool, *args, stats=stats)
    assert np.abs(mass4.cpu().numpy() - mass).max() < 1e-5


def test_attention_based_eviction_from_measured_attention(kvx):
    """decode -> per-page attention -> EvictionMetrics -> AttentionBased victim:
    the least-attended page of the step (the reference's policy on measured
    attention instead of its stub)."""
    from oracle import EVICT_METRICS
    lens = np.array([300, 41, 700], np.int64)
    bt, num_pages = kvgen.paged_layout(lens, 16, 0, seed=141)
    pool = kvgen.normal(142, (num_pages, 2, 8, 16, 128)).astype(np.float16)
    q = kvgen.normal(143, (3, 24, 128)) * 3
    m = np.zeros(num_pages, EVICT_METRICS)
    m["page_id"] = np.arange(num_pages)
    metrics = dev(m.view(np.uint8))
    gbt, glens = dev(bt), dev(lens.astype(np.int32))
    _, mass = kvx.decode_attn(dev(pool), gbt, glens, dev(q))
    kvx.attn_to_metrics(mass, gbt, glens, metrics, 12345)
    got = metrics.cpu().numpy().view(EVICT_METRICS)
    mass = mass.cpu().numpy()
    want_avg = np.zeros(num_pages, np.float32)
    for s in range(3):
        npg = (int(lens[s]) + 15) // 16
        want_avg[bt[s, :npg]] = mass[s, :npg]
    assert np.array_equal(got["average_attention"], want_avg)
    assert np.all(got["last_access_token"] == 12345) and np.all(got["access_frequency"] == 1)
    victim = kvx.evict_select(kvx.EVICT_ATTENTION_BASED, metrics).item()
    assert victim == int(np.argmin(want_avg))
