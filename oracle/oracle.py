"""ctypes + numpy front end of the parity checker (test infrastructure only).

Two libraries sit behind this module:

* ``Oracle``   -- oracle/_build/libkvx_oracle.so, the C restatement of the
  reference algorithms (oracle/kvx_oracle.c).  It is what the GPU parity tests
  compare against; it is pinned to the reference by tests/golden/.
* ``Reference`` -- oracle/_ref/libkvref.so, the reference's own CPU sources
  compiled unmodified plus extern "C" marshalling (oracle/ref_harness.cpp).
  Used to generate the golden vectors and, on the GPU box, as the timed CPU
  baseline of bench.py.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libkvx_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkvref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)


def build_reference(ref_dir: str | None = None) -> bool:
    """Compile the reference CPU sources from the checkout at `ref_dir`
    (default: the KVX_REFERENCE_DIR environment variable); False when no
    checkout is given or present."""
    ref = ref_dir or os.environ.get("KVX_REFERENCE_DIR")
    if not ref or not os.path.isdir(ref):
        return False
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)
    return True


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


EVICT_METRICS = np.dtype([("last_access_token", "<u8"), ("total_attention", "<f4"),
                          ("average_attention", "<f4"), ("access_frequency", "<f4"), ("_pad0", "<u4"),
                          ("creation_time", "<u8"), ("page_size", "<u8"), ("page_id", "<i4"),
                          ("_pad1", "<u4")])
assert EVICT_METRICS.itemsize == 48


class Oracle:
    """The C restatement (oracle/kvx_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build_oracle()
        L = C.CDLL(path)
        self.L = L
        L.kvo_encode_f16_trunc.argtypes = [_f32p, _u16p, _sz]
        L.kvo_decode_f16_trunc.argtypes = [_u16p, _f32p, _sz]
        L.kvo_compress_int8.argtypes = [_f32p, _i8p, _sz, _f32p]
        L.kvo_decompress_int8.argtypes = [_i8p, _f32p, _sz, _f32p]
        L.kvo_compress_int8_blocks_f16.argtypes = [_u16p, _i8p, _f32p, _sz, _sz]
        L.kvo_compress_int8_blocks_f32.argtypes = [_f32p, _i8p, _f32p, _sz, _sz]
        L.kvo_decompress_int8_blocks.argtypes = [_i8p, _f32p, _f32p, _sz, _sz]
        L.kvo_compress_nf4.argtypes = [_f32p, _u8p, _sz, _f32p]
        L.kvo_decompress_nf4.argtypes = [_u8p, _f32p, _sz, _f32p]
        L.kvo_compress_nf4_blocks_f16.argtypes = [_u16p, _u8p, _f32p, _sz, _sz]
        L.kvo_compress_nf4_blocks_f32.argtypes = [_f32p, _u8p, _f32p, _sz, _sz]
        L.kvo_decompress_nf4_blocks.argtypes = [_u8p, _f32p, _f32p, _sz, _sz]
        L.kvo_evict_select.argtypes = [C.c_int, C.c_void_p, _sz, C.c_float, C.c_void_p]
        L.kvo_evict_select.restype = C.c_int
        L.kvo_evict_score.argtypes = [C.c_int, C.c_void_p, C.c_float, C.c_float]
        L.kvo_evict_score.restype = C.c_float
        L.kvo_evict_select_composite.argtypes = [_i32p, _f32p, C.c_int, C.c_void_p, _sz, C.c_float,
                                                 C.c_void_p]
        L.kvo_evict_select_composite.restype = C.c_int
        L.kvo_predict_next_access.argtypes = [_u64p, _sz]
        L.kvo_predict_next_access.restype = C.c_float
        L.kvo_fp16_wrap_encode_n.argtypes = [_f32p, _u16p, _sz]
        L.kvo_fp16_wrap_decode_n.argtypes = [_u16p, _f32p, _sz]
        L.kvo_append.argtypes = [C.c_void_p, _sz, C.c_int, C.c_int, C.c_int, C.c_int,
                                 _i32p, C.c_int, _i32p, C.c_int, C.c_void_p, C.c_void_p]
        L.kvo_append.restype = C.c_int
        L.kvo_attention_row.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _f32p]
        L.kvo_paged_decode.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                       C.c_int, C.c_int, _i32p, C.c_int, _i32p, C.c_int,
                                       C.c_int, _f32p, _f32p]
        L.kvo_paged_decode.restype = C.c_int
        L.kvo_lru_select.argtypes = [_u64p, _sz]
        L.kvo_lru_select.restype = C.c_int
        L.kvo_lru_replay.argtypes = [_i32p, _u8p, _sz, _sz, _i32p, _u8p]
        L.kvo_lru_replay.restype = C.c_int
        L.kvo_prefetch_depth.argtypes = [_f64p, _sz, _sz, _sz, C.c_int]
        L.kvo_prefetch_depth.restype = C.c_int
        L.kvo_kvcache_gpu_replay.argtypes = [C.c_void_p, _sz, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]
        L.kvo_kvcache_gpu_replay.restype = C.c_int

    # compression/kv_compress.cpp
    def f32_to_f16_trunc(self, x):
        x = _c(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.kvo_encode_f16_trunc(x, out, x.size)
        return out

    def f16_trunc_to_f32(self, h):
        h = _c(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.kvo_decode_f16_trunc(h, out, h.size)
        return out

    # KVCompressionEngine INT8
    def compress_int8(self, x):
        x = _c(x, np.float32).ravel()
        codes = np.empty(x.size, np.int8)
        stats = np.empty(4, np.float32)
        self.L.kvo_compress_int8(x, codes, x.size, stats)
        return codes, stats

    def decompress_int8(self, codes, stats):
        codes = _c(codes, np.int8).ravel()
        out = np.empty(codes.size, np.float32)
        self.L.kvo_decompress_int8(codes, out, codes.size, _c(stats, np.float32))
        return out

    def compress_int8_blocks(self, data, block_elems):
        """data: fp16 (np.float16) or fp32 array; one reference call per block."""
        flat = np.ascontiguousarray(data).ravel()
        nb = flat.size // block_elems
        codes = np.empty(flat.size, np.int8)
        stats = np.empty(nb * 4, np.float32)
        if flat.dtype == np.float16:
            self.L.kvo_compress_int8_blocks_f16(flat.view(np.uint16), codes, stats, nb,
                                                block_elems)
        else:
            self.L.kvo_compress_int8_blocks_f32(_c(flat, np.float32), codes, stats, nb,
                                                block_elems)
        return codes, stats.reshape(nb, 4)

    def decompress_int8_blocks(self, codes, stats, block_elems):
        codes = _c(codes, np.int8).ravel()
        nb = codes.size // block_elems
        out = np.empty(codes.size, np.float32)
        self.L.kvo_decompress_int8_blocks(codes, _c(stats, np.float32).ravel(), out, nb,
                                          block_elems)
        return out

    # KVCompressionEngine NF4 (uniform 4-bit) and FP16 (exponent-wrap)
    def compress_nf4(self, x):
        x = _c(x, np.float32).ravel()
        codes = np.empty((x.size + 1) // 2, np.uint8)
        stats = np.empty(4, np.float32)
        self.L.kvo_compress_nf4(x, codes, x.size, stats)
        return codes, stats

    def decompress_nf4(self, codes, stats, count):
        out = np.empty(count, np.float32)
        self.L.kvo_decompress_nf4(_c(codes, np.uint8).ravel(), out, count, _c(stats, np.float32))
        return out

    def compress_nf4_blocks(self, data, block_elems):
        flat = np.ascontiguousarray(data).ravel()
        nb = flat.size // block_elems
        codes = np.empty(nb * ((block_elems + 1) // 2), np.uint8)
        stats = np.empty(nb * 4, np.float32)
        if flat.dtype == np.float16:
            self.L.kvo_compress_nf4_blocks_f16(flat.view(np.uint16), codes, stats, nb, block_elems)
        else:
            self.L.kvo_compress_nf4_blocks_f32(_c(flat, np.float32), codes, stats, nb, block_elems)
        return codes, stats.reshape(nb, 4)

    def decompress_nf4_blocks(self, codes, stats, block_elems):
        st = _c(stats, np.float32).ravel()
        nb = st.size // 4
        out = np.empty(nb * block_elems, np.float32)
        self.L.kvo_decompress_nf4_blocks(_c(codes, np.uint8).ravel(), st, out, nb, block_elems)
        return out

    def fp16_wrap_encode(self, x):
        x = _c(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.kvo_fp16_wrap_encode_n(x, out, x.size)
        return out

    # AdvancedEvictionPolicy (pages: EVICT_METRICS records)
    def evict_select(self, policy, pages, decay=0.95, predicted=None):
        pages = np.ascontiguousarray(pages, EVICT_METRICS)
        pred = None if predicted is None else _c(predicted, np.float32)
        return self.L.kvo_evict_select(policy, pages.ctypes.data, pages.size, decay,
                                       None if pred is None else pred.ctypes.data)

    def evict_scores(self, policy, pages, decay=0.95, predicted=None):
        pages = np.ascontiguousarray(pages, EVICT_METRICS)
        out = np.empty(pages.size, np.float32)
        for i in range(pages.size):
            p = -1.0 if predicted is None else float(predicted[i])
            out[i] = self.L.kvo_evict_score(policy, pages[i:i + 1].ctypes.data, decay, p)
        return out

    def evict_select_composite(self, policies, weights, pages, decay=0.95, predicted=None):
        pages = np.ascontiguousarray(pages, EVICT_METRICS)
        pred = None if predicted is None else _c(predicted, np.float32)
        return self.L.kvo_evict_select_composite(_c(policies, np.int32), _c(weights, np.float32),
                                                 len(policies), pages.ctypes.data, pages.size, decay,
                                                 None if pred is None else pred.ctypes.data)

    def predict_next_access(self, times):
        t = _c(times, np.uint64)
        return self.L.kvo_predict_next_access(t, t.size)

    def fp16_wrap_decode(self, h):
        h = _c(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.kvo_fp16_wrap_decode_n(h, out, h.size)
        return out

    def append(self, pool, block_table, positions, new_k, new_v, page_tokens):
        """pool: [pages][2][hkv][page_tokens][dim] numpy array, modified in place."""
        num_pages, _, hkv, pt, dim = pool.shape
        assert pt == page_tokens and pool.flags.c_contiguous
        bt = _c(block_table, np.int32)
        nk = np.ascontiguousarray(new_k, dtype=pool.dtype)
        nv = np.ascontiguousarray(new_v, dtype=pool.dtype)
        rc = self.L.kvo_append(pool.ctypes.data, pool.itemsize, num_pages, hkv, dim,
                               page_tokens, bt, bt.shape[1], _c(positions, np.int32),
                               bt.shape[0], nk.ctypes.data, nv.ctypes.data)
        if rc != 0:
            raise ValueError("append: page out of range")

    def attention_row(self, q, k, v):
        q = _c(q, np.float32)
        k = _c(k, np.float32)
        v = _c(v, np.float32)
        out = np.empty(q.size, np.float32)
        self.L.kvo_attention_row(q, k, v, k.shape[0], q.size, out)
        return out

    def paged_decode(self, pool, block_table, seq_lens, q, stats=None):
        """pool: [pages][2][hkv][pt][dim] fp32 / fp16 / int8 (stats [pages][2][hkv][4])."""
        num_pages, _, hkv, pt, dim = pool.shape
        kind = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int8): 2}[pool.dtype]
        pool = np.ascontiguousarray(pool)
        st = None if stats is None else _c(stats, np.float32)
        bt = _c(block_table, np.int32)
        q = _c(q, np.float32)
        batch, hq, _ = q.shape
        out = np.zeros_like(q)
        rc = self.L.kvo_paged_decode(pool.ctypes.data, kind,
                                     None if st is None else st.ctypes.data, num_pages, hkv,
                                     dim, pt, bt, bt.shape[1], _c(seq_lens, np.int32), batch,
                                     hq, q, out)
        if rc != 0:
            raise ValueError("paged_decode: bad geometry or page id")
        return out

    def lru_select(self, stamps):
        s = _c(stamps, np.uint64)
        return self.L.kvo_lru_select(s, s.size)

    def lru_replay(self, ids, ops, capacity):
        ids = _c(ids, np.int32)
        ops = _c(ops, np.uint8)
        ev = np.empty(ids.size, np.int32)
        hit = np.empty(ids.size, np.uint8)
        rc = self.L.kvo_lru_replay(ids, ops, ids.size, capacity, ev, hit)
        if rc != 0:
            raise ValueError("lru_replay: negative id")
        return ev, hit

    def kvcache_gpu_replay(self, ops, total, page_size):
        """KVCacheGPU (native-engine/cpp/KVCacheGPU.cpp) over ops [n][3] =
        (op, a, b); returns (result[n], used[n]) (see kvx_oracle.h)."""
        ops = _c(ops, np.int64).reshape(-1, 3)
        res = np.empty(len(ops), np.int64)
        used = np.empty(len(ops), np.uint64)
        rc = self.L.kvo_kvcache_gpu_replay(ops.ctypes.data, len(ops), int(total), int(page_size),
                                          res.ctypes.data, used.ctypes.data)
        if rc != 0:
            raise ValueError("kvcache_gpu_replay: negative page id in a transfer")
        return res, used

    def prefetch_depth(self, latencies, size, capacity, max_depth=4):
        lat = _c(latencies, np.float64)
        return self.L.kvo_prefetch_depth(lat, lat.size, size, capacity, max_depth)


class Reference:
    """The reference's own CPU code (oracle/_ref/libkvref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        self.L = L
        L.kvref_f32_to_f16.argtypes = [_f32p, _u16p, _sz]
        L.kvref_f16_to_f32.argtypes = [_u16p, _f32p, _sz]
        L.kvref_compress_int8.argtypes = [_f32p, _i8p, _sz, _f32p]
        L.kvref_decompress_int8.argtypes = [_i8p, _f32p, _sz, _f32p]
        L.kvref_compress_nf4.argtypes = [_f32p, _u8p, _sz, _f32p]
        L.kvref_decompress_nf4.argtypes = [_u8p, _f32p, _sz, _f32p]
        L.kvref_evict_select.argtypes = [C.c_int, C.c_void_p, _sz, C.c_float, C.c_void_p, C.c_void_p,
                                         C.c_void_p]
        L.kvref_evict_select.restype = C.c_int
        L.kvref_evict_composite.argtypes = [_i32p, _f32p, C.c_int, C.c_void_p, _sz, _f32p]
        L.kvref_evict_composite.restype = C.c_int
        L.kvref_fp16_wrap_encode.argtypes = [_f32p, _u16p, _sz]
        L.kvref_fp16_wrap_decode.argtypes = [_u16p, _f32p, _sz]
        L.kvref_attention.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _f32p]
        L.kvref_attention.restype = C.c_int
        L.kvref_softmax.argtypes = [_f32p, _sz, _sz, _f32p]
        L.kvref_softmax.restype = C.c_int
        L.kvref_attention_row.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _f32p]
        L.kvref_attention_row.restype = C.c_int
        L.kvref_lru_select.argtypes = [_u64p, _sz]
        L.kvref_lru_select.restype = C.c_int
        L.kvref_lru_replay.argtypes = [_i32p, _u8p, _sz, _sz, C.c_char_p, _i32p, _u8p]
        L.kvref_lru_replay.restype = C.c_int
        L.kvref_save_page.argtypes = [C.c_int, _f32p, _sz, _f32p, _sz, C.c_char_p, _sz]
        L.kvref_save_page.restype = C.c_int
        L.kvref_load_page.argtypes = [C.c_int, C.c_char_p, _f32p, _sz, _f32p, _sz,
                                      C.POINTER(C.c_size_t)]
        L.kvref_load_page.restype = C.c_long
        L.kvref_prefetch_depth.argtypes = [_f64p, _sz, _sz, _sz, C.c_int]
        L.kvref_prefetch_depth.restype = C.c_int
        L.kvref_time_decode.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, C.c_int, _f32p]
        L.kvref_time_decode.restype = C.c_double
        L.kvref_time_compress.argtypes = [_f32p, _i8p, _f32p, _sz, _sz, C.c_int]
        L.kvref_time_compress.restype = C.c_double
        L.kvref_time_tier.argtypes = [_i32p, _sz, _sz, _sz, _sz, C.c_char_p, C.POINTER(C.c_int64)]
        L.kvref_time_tier.restype = C.c_double
        L.kvref_time_append.argtypes = [_f32p, _sz, _sz, _sz, _sz, C.c_char_p]
        L.kvref_time_append.restype = C.c_double

    def f32_to_f16_trunc(self, x):
        x = _c(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.kvref_f32_to_f16(x, out, x.size)
        return out

    def f16_trunc_to_f32(self, h):
        h = _c(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.kvref_f16_to_f32(h, out, h.size)
        return out

    def compress_int8(self, x):
        x = _c(x, np.float32).ravel()
        codes = np.empty(x.size, np.int8)
        stats = np.empty(4, np.float32)
        self.L.kvref_compress_int8(x, codes, x.size, stats)
        return codes, stats

    def decompress_int8(self, codes, stats):
        codes = _c(codes, np.int8).ravel()
        out = np.empty(codes.size, np.float32)
        self.L.kvref_decompress_int8(codes, out, codes.size, _c(stats, np.float32))
        return out

    def compress_nf4(self, x):
        x = _c(x, np.float32).ravel()
        codes = np.empty((x.size + 1) // 2, np.uint8)
        stats = np.empty(4, np.float32)
        self.L.kvref_compress_nf4(x, codes, x.size, stats)
        return codes, stats

    def decompress_nf4(self, codes, stats, count):
        out = np.empty(count, np.float32)
        self.L.kvref_decompress_nf4(_c(codes, np.uint8).ravel(), out, count, _c(stats, np.float32))
        return out

    def fp16_wrap_encode(self, x):
        x = _c(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.kvref_fp16_wrap_encode(x, out, x.size)
        return out

    def fp16_wrap_decode(self, h):
        h = _c(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.kvref_fp16_wrap_decode(h, out, h.size)
        return out

    def evict_select(self, policy, pages, decay=0.95, hist=None, hist_len=None):
        """Returns (selected page id, every page's calculateScore(m, 0))."""
        pages = np.ascontiguousarray(pages, EVICT_METRICS)
        scores = np.empty(pages.size, np.float32)
        h = None if hist is None else _c(hist, np.uint64)
        hl = None if hist_len is None else _c(hist_len, np.int32)
        sel = self.L.kvref_evict_select(policy, pages.ctypes.data, pages.size, decay,
                                        None if h is None else h.ctypes.data,
                                        None if hl is None else hl.ctypes.data, scores.ctypes.data)
        return sel, scores

    def evict_composite(self, policies, weights, pages):
        """Returns (selected page id, the manager's normalised weights)."""
        pages = np.ascontiguousarray(pages, EVICT_METRICS)
        nw = np.empty(len(policies), np.float32)
        sel = self.L.kvref_evict_composite(_c(policies, np.int32), _c(weights, np.float32), len(policies),
                                           pages.ctypes.data, pages.size, nw)
        return sel, nw

    def attention(self, q, k, v):
        q, k, v = (_c(a, np.float32) for a in (q, k, v))
        out = np.empty_like(q)
        if self.L.kvref_attention(q, k, v, q.shape[0], q.shape[1], out) != 0:
            raise ValueError("attention failed")
        return out

    def softmax(self, logits):
        logits = _c(logits, np.float32)
        out = np.empty_like(logits)
        self.L.kvref_softmax(logits, logits.shape[0], logits.shape[1], out)
        return out

    def attention_row(self, q, k, v):
        q, k, v = (_c(a, np.float32) for a in (q, k, v))
        out = np.empty(q.size, np.float32)
        if self.L.kvref_attention_row(q, k, v, k.shape[0], q.size, out) != 0:
            raise ValueError("attention_row failed")
        return out

    def lru_select(self, stamps):
        s = _c(stamps, np.uint64)
        return self.L.kvref_lru_select(s, s.size)

    def lru_replay(self, ids, ops, capacity, workdir):
        """Replay through a real KVManager; run with cwd=workdir (page files land there)."""
        ids = _c(ids, np.int32)
        ops = _c(ops, np.uint8)
        ev = np.empty(ids.size, np.int32)
        hit = np.empty(ids.size, np.uint8)
        cwd = os.getcwd()
        os.chdir(workdir)
        try:
            for i in np.unique(ids):  # every page needs a file before load_page
                self.save_page(int(i), np.zeros(1, np.float32), np.zeros(1, np.float32),
                               "pages")
            rc = self.L.kvref_lru_replay(ids, ops, ids.size, capacity, b"pages", ev, hit)
        finally:
            os.chdir(cwd)
        if rc != 0:
            raise RuntimeError("kvref_lru_replay failed")
        return ev, hit

    def save_page(self, pid, key, value, dirname, capacity=4):
        k = _c(key, np.float32).ravel()
        v = _c(value, np.float32).ravel()
        return self.L.kvref_save_page(pid, k, k.size, v, v.size, dirname.encode(), capacity)

    def load_page(self, pid, dirname, cap=1 << 20):
        k = np.empty(cap, np.float32)
        v = np.empty(cap, np.float32)
        nv = C.c_size_t(0)
        nk = self.L.kvref_load_page(pid, dirname.encode(), k, cap, v, cap, C.byref(nv))
        if nk < 0:
            raise FileNotFoundError(pid)
        return k[:nk].copy(), v[: nv.value].copy()

    def time_tier(self, ids, universe, capacity, page_floats, workdir):
        """Seconds KVManager (capacity pages, fp16 page files in workdir) takes
        to serve load_page over `ids`, and how many of them read a file."""
        ids = _c(ids, np.int32)
        misses = C.c_int64()
        s = self.L.kvref_time_tier(ids, ids.size, universe, capacity, page_floats,
                                   workdir.encode(), C.byref(misses))
        if s < 0:
            raise RuntimeError("kvref_time_tier failed")
        return s, misses.value

    def kvcache_gpu_replay(self, ops, total, page_size):
        """KVCacheGPU (native-engine/cpp/KVCacheGPU.cpp) over ops [n][3] =
        (op, a, b); returns (result[n], used[n]) (see kvx_oracle.h)."""
        ops = _c(ops, np.int64).reshape(-1, 3)
        res = np.empty(len(ops), np.int64)
        used = np.empty(len(ops), np.uint64)
        rc = self.L.kvo_kvcache_gpu_replay(ops.ctypes.data, len(ops), int(total), int(page_size),
                                          res.ctypes.data, used.ctypes.data)
        if rc != 0:
            raise ValueError("kvcache_gpu_replay: negative page id in a transfer")
        return res, used

    def prefetch_depth(self, latencies, size, capacity, max_depth=4):
        lat = _c(latencies, np.float64)
        return self.L.kvref_prefetch_depth(lat, lat.size, size, capacity, max_depth)


def persist_bytes(key, value) -> bytes:
    """Bytes of a page file as KVManager::persist_to_disk writes them
    (cache/kv_cache.cpp:21-41): u8 flag=1, u64 n_key, n_key x u16 (truncating
    fp16 of compression/kv_compress.cpp:6-25), u64 n_value, n_value x u16."""
    o = Oracle()
    k = o.f32_to_f16_trunc(key)
    v = o.f32_to_f16_trunc(value)
    return (b"\x01" + np.uint64(k.size).tobytes() + k.tobytes() +
            np.uint64(v.size).tobytes() + v.tobytes())
