"""Python front end of libadaptive_engine.so (ctypes over the C ABI in
include/kvx.h and include/adaptive_engine.h).

Tensors are torch CUDA tensors; only their data pointers and the current
CUDA stream cross the ABI.  There is no fallback: importing this module on a
machine where the library cannot be loaded raises, and every call whose
status is not KVX_OK raises KvxError.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libadaptive_engine.so")

KVX_F32, KVX_F16, KVX_I8 = 0, 1, 2
HEAD_DIM, PAGE_TOKENS = 128, 16

STATUS = {0: "ok", -1: "invalid argument", -2: "object pinned", -3: "CUDA error",
          -4: "unsupported geometry or dtype", -5: "bounded device wait expired",
          -6: "workspace or pool too small", -7: "no sm_100 device",
          -8: "request exceeds the static scratch of kvx_decode_noalloc",
          -9: "another rank's part of the multi-GPU step failed"}


class KvxError(RuntimeError):
    def __init__(self, fn, status):
        super().__init__(f"{fn}: {STATUS.get(status, status)} ({status})")
        self.status = status


def build() -> str:
    """Compile the library in-tree (nvcc, sm_100a)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", PKG, "-j8"], check=True)
    return LIB_PATH


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `make -C {PKG}`")
    return C.CDLL(LIB_PATH)


lib = _load()


class KvPaged(C.Structure):
    _fields_ = [("pool", C.c_void_p), ("stats", C.c_void_p), ("dtype", C.c_int32),
                ("num_pages", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("page_tokens", C.c_int32)]


_vp, _i32, _sz, _f32 = C.c_void_p, C.c_int32, C.c_size_t, C.c_float
lib.kvx_version.restype = C.c_char_p
lib.kvx_status_string.restype = C.c_char_p
lib.kvx_status_string.argtypes = [C.c_int]
lib.kvx_device_check.restype = C.c_int
lib.kvx_append.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp]
lib.kvx_append_chunk.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp]
lib.kvx_append_chunk.restype = C.c_int
lib.kvx_decode_workspace_bytes.restype = _sz
lib.kvx_decode_workspace_bytes.argtypes = [_i32, _i32, _i32, _i32]
lib.kvx_decode.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _i32, _vp, _vp, _i32, _f32,
                           _vp, _sz, _vp, _vp]
lib.kvx_append_decode.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp,
                                  _vp, _i32, _f32, _vp, _sz, _vp, _vp]
lib.kvx_append_decode_signal.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _vp, _vp, _i32, _vp,
                                         _vp, _i32, _f32, _vp, _sz, _vp, _vp, C.c_uint32, _vp]
lib.kvx_stream_wait_geq.argtypes = [_vp, C.c_uint32, _vp]
lib.kvx_decode_workspace_init.argtypes = [_vp, _sz, _vp]
lib.kvx_decode_noalloc.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _i32, _vp, _vp, _i32,
                                   _f32, _vp, _vp]
lib.kvx_decode_noalloc.restype = C.c_int
lib.kvx_decode_noalloc_scratch_bytes.restype = _sz
lib.kvx_compress_int8.argtypes = [_vp, _i32, _vp, _vp, _sz, _i32, _vp]
lib.kvx_decompress_int8.argtypes = [_vp, _vp, _vp, _i32, _sz, _i32, _vp]
lib.kvx_compress_nf4.argtypes = [_vp, _i32, _vp, _vp, _sz, _i32, _vp]
lib.kvx_decompress_nf4.argtypes = [_vp, _vp, _vp, _i32, _sz, _i32, _vp]
lib.kvx_fp16_wrap_encode.argtypes = [_vp, _vp, _sz, _vp]
lib.kvx_fp16_wrap_decode.argtypes = [_vp, _vp, _sz, _vp]
lib.kvx_f32_to_f16_trunc.argtypes = [_vp, _vp, _sz, _vp]
lib.kvx_f16_trunc_to_f32.argtypes = [_vp, _vp, _sz, _vp]
lib.kvx_lru_select.argtypes = [_vp, _sz, _vp, _vp]
lib.kvx_migrate_frames.argtypes = [_vp, _i32, _vp, _i32, _vp, _vp, _i32, _sz, _i32, _i32, _vp, _vp]
lib.kvx_evict_select.argtypes = [_i32, _vp, _sz, _f32, _vp, _vp, _vp]
lib.kvx_decode_attn_workspace_bytes.restype = _sz
lib.kvx_decode_attn_workspace_bytes.argtypes = [_i32, _i32, _i32, _i32]
lib.kvx_decode_attn.argtypes = [C.POINTER(KvPaged), _vp, _i32, _vp, _i32, _i32, _vp, _vp, _i32, _f32,
                                _vp, _sz, _vp, _vp, _vp]
lib.kvx_decode_attn.restype = C.c_int
lib.kvx_attn_to_metrics.argtypes = [_vp, _vp, _i32, _vp, _i32, _vp, _i32, C.c_uint64, _vp]
lib.kvx_attn_to_metrics.restype = C.c_int
lib.kvx_evict_select_composite.argtypes = [_vp, _vp, _i32, _vp, _sz, _f32, _vp, _vp, _vp]
for _fn in ("kvx_append", "kvx_decode", "kvx_append_decode", "kvx_append_decode_signal", "kvx_stream_wait_geq",
            "kvx_decode_workspace_init", "kvx_compress_int8", "kvx_decompress_int8",
            "kvx_compress_nf4", "kvx_decompress_nf4", "kvx_fp16_wrap_encode", "kvx_fp16_wrap_decode",
            "kvx_f32_to_f16_trunc", "kvx_f16_trunc_to_f32", "kvx_lru_select",
            "kvx_migrate_frames", "kvx_evict_select", "kvx_evict_select_composite"):
    getattr(lib, _fn).restype = C.c_int


def _check(fn, rc):
    if rc != 0:
        raise KvxError(fn, rc)


def _torch():
    import torch
    return torch


def _stream(stream):
    if stream is not None:
        return C.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
    return C.c_void_p(_torch().cuda.current_stream().cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dtype_code(t):
    torch = _torch()
    return {torch.float32: KVX_F32, torch.float16: KVX_F16, torch.int8: KVX_I8}[t.dtype]


def paged(pool, stats=None) -> KvPaged:
    """Describe one layer's pool: a CUDA tensor [pages][2][hkv][16][128], or
    an existing KvPaged view (e.g. from kvx.engine.layer_view)."""
    if isinstance(pool, KvPaged):
        return pool
    assert pool.is_cuda and pool.is_contiguous() and pool.dim() == 5
    pages, two, hkv, pt, dim = pool.shape
    assert two == 2
    return KvPaged(pool.data_ptr(), 0 if stats is None else stats.data_ptr(), _dtype_code(pool),
                   pages, hkv, dim, pt)


class _DeviceArray:
    """__cuda_array_interface__ over a raw device address (no ownership)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


def pool_tensor(view):
    """A torch view [pages][2][hkv][16][128] of a KvPaged pool (e.g. an
    engine layer from kvx.engine.layer_view); the memory stays the owner's."""
    torch = _torch()
    typestr = {KVX_F32: "<f4", KVX_F16: "<f2", KVX_I8: "|i1"}[view.dtype]
    shape = (view.num_pages, 2, view.num_kv_heads, view.page_tokens, view.head_dim)
    return torch.as_tensor(_DeviceArray(view.pool, shape, typestr), device="cuda")


def append(pool, block_table, positions, new_k, new_v, error_flag=None, stream=None):
    kv = paged(pool)
    rc = lib.kvx_append(C.byref(kv), _ptr(block_table), block_table.shape[1], _ptr(positions),
                        positions.shape[0], _ptr(new_k), _ptr(new_v), _ptr(error_flag),
                        _stream(stream))
    _check("kvx_append", rc)


def append_chunk(pool, block_table, positions, new_k, new_v, error_flag=None, stream=None):
    """Append new_k / new_v [batch][n_new][hkv][128] at positions[s] ..
    positions[s] + n_new - 1 of each sequence."""
    kv = paged(pool)
    batch, n_new = new_k.shape[0], new_k.shape[1]
    rc = lib.kvx_append_chunk(C.byref(kv), _ptr(block_table), block_table.shape[1], _ptr(positions), batch,
                              n_new, _ptr(new_k), _ptr(new_v), _ptr(error_flag), _stream(stream))
    _check("kvx_append_chunk", rc)


def decode_workspace_bytes(batch, num_q_heads, max_pages):
    return lib.kvx_decode_workspace_bytes(batch, num_q_heads, max_pages, PAGE_TOKENS)


def decode_workspace(batch, num_q_heads, max_pages, device="cuda"):
    """A zero-filled decode workspace (the split counters start at zero)."""
    torch = _torch()
    return torch.zeros(max(decode_workspace_bytes(batch, num_q_heads, max_pages), 16),
                       dtype=torch.uint8, device=device)


def decode(pool, block_table, seq_lens, q, out=None, stats=None, workspace=None,
           error_flag=None, sm_scale=0.0, stream=None):
    """Paged GQA decode.  q: [batch][hq][128] fp32/fp16 CUDA tensor."""
    torch = _torch()
    kv = paged(pool, stats)
    batch, hq, _ = q.shape
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        workspace = decode_workspace(batch, hq, block_table.shape[1], q.device)
    rc = lib.kvx_decode(C.byref(kv), _ptr(block_table), block_table.shape[1], _ptr(seq_lens),
                        batch, hq, _ptr(q), _ptr(out), _dtype_code(q), sm_scale,
                        _ptr(workspace), workspace.numel() * workspace.element_size(),
                        _ptr(error_flag), _stream(stream))
    _check("kvx_decode", rc)
    return out


def append_decode(pool, block_table, positions, new_k, new_v, q, out=None, workspace=None,
                  error_flag=None, sm_scale=0.0, stream=None):
    """Append the token at `positions` and decode over positions+1 tokens, one launch."""
    torch = _torch()
    kv = paged(pool)
    batch, hq, _ = q.shape
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        workspace = decode_workspace(batch, hq, block_table.shape[1], q.device)
    rc = lib.kvx_append_decode(C.byref(kv), _ptr(block_table), block_table.shape[1],
                               _ptr(positions), batch, _ptr(new_k), _ptr(new_v), hq, _ptr(q),
                               _ptr(out), _dtype_code(q), sm_scale, _ptr(workspace),
                               workspace.numel() * workspace.element_size(), _ptr(error_flag),
                               _stream(stream))
    _check("kvx_append_decode", rc)
    return out


def append_decode_signal(pool, block_table, positions, new_k, new_v, q, done, epoch, out=None,
                         workspace=None, error_flag=None, sm_scale=0.0, stream=None):
    """append_decode that stores `epoch` to done[1] once the whole launch has
    finished (done: int32 CUDA tensor of 2, done[0] zero-filled once)."""
    torch = _torch()
    kv = paged(pool)
    batch, hq, _ = q.shape
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        workspace = decode_workspace(batch, hq, block_table.shape[1], q.device)
    rc = lib.kvx_append_decode_signal(C.byref(kv), _ptr(block_table), block_table.shape[1],
                                      _ptr(positions), batch, _ptr(new_k), _ptr(new_v), hq, _ptr(q),
                                      _ptr(out), _dtype_code(q), sm_scale, _ptr(workspace),
                                      workspace.numel() * workspace.element_size(), _ptr(error_flag),
                                      _ptr(done), epoch & 0xFFFFFFFF, _stream(stream))
    _check("kvx_append_decode_signal", rc)
    return out


def stream_wait_geq(word, value, stream=None):
    """Make `stream` wait until the device word reaches `value` (cyclic
    32-bit comparison).  word: a CUDA tensor whose first element is waited on."""
    _check("kvx_stream_wait_geq", lib.kvx_stream_wait_geq(_ptr(word), value & 0xFFFFFFFF, _stream(stream)))


def compress_int8(src, block_elems=PAGE_TOKENS * HEAD_DIM, codes=None, stats=None, stream=None):
    torch = _torch()
    n = src.numel()
    nb = n // block_elems
    if codes is None:
        codes = torch.empty(n, dtype=torch.int8, device=src.device)
    if stats is None:
        stats = torch.empty((nb, 4), dtype=torch.float32, device=src.device)
    rc = lib.kvx_compress_int8(_ptr(src), _dtype_code(src), _ptr(codes), _ptr(stats), nb,
                               block_elems, _stream(stream))
    _check("kvx_compress_int8", rc)
    return codes, stats


def decompress_int8(codes, stats, dtype=None, block_elems=PAGE_TOKENS * HEAD_DIM, out=None,
                    stream=None):
    torch = _torch()
    dtype = dtype or torch.float32
    if out is None:
        out = torch.empty(codes.numel(), dtype=dtype, device=codes.device)
    rc = lib.kvx_decompress_int8(_ptr(codes), _ptr(stats), _ptr(out), _dtype_code(out),
                                 codes.numel() // block_elems, block_elems, _stream(stream))
    _check("kvx_decompress_int8", rc)
    return out


def compress_nf4(src, block_elems=PAGE_TOKENS * HEAD_DIM, codes=None, stats=None, stream=None):
    """KVCompressionEngine NF4 per block: codes (uint8, two per byte) and stats."""
    torch = _torch()
    nb = src.numel() // block_elems
    if codes is None:
        codes = torch.empty(nb * ((block_elems + 1) // 2), dtype=torch.uint8, device=src.device)
    if stats is None:
        stats = torch.empty((nb, 4), dtype=torch.float32, device=src.device)
    rc = lib.kvx_compress_nf4(_ptr(src), _dtype_code(src), _ptr(codes), _ptr(stats), nb, block_elems,
                              _stream(stream))
    _check("kvx_compress_nf4", rc)
    return codes, stats


def decompress_nf4(codes, stats, dtype=None, block_elems=PAGE_TOKENS * HEAD_DIM, out=None, stream=None):
    torch = _torch()
    dtype = dtype or torch.float32
    nb = stats.numel() // 4
    if out is None:
        out = torch.empty(nb * block_elems, dtype=dtype, device=codes.device)
    rc = lib.kvx_decompress_nf4(_ptr(codes), _ptr(stats), _ptr(out), _dtype_code(out), nb, block_elems,
                                _stream(stream))
    _check("kvx_decompress_nf4", rc)
    return out


def fp16_wrap_encode(x, out=None, stream=None):
    """KVCompressionEngine FP16 (exponent-wrapping): fp32 -> uint16 bits as int16 tensor."""
    torch = _torch()
    if out is None:
        out = torch.empty(x.numel(), dtype=torch.int16, device=x.device)
    _check("kvx_fp16_wrap_encode", lib.kvx_fp16_wrap_encode(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def fp16_wrap_decode(h, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty(h.numel(), dtype=torch.float32, device=h.device)
    _check("kvx_fp16_wrap_decode", lib.kvx_fp16_wrap_decode(_ptr(h), _ptr(out), h.numel(), _stream(stream)))
    return out


def f32_to_f16_trunc(x, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty(x.numel(), dtype=torch.int16, device=x.device)
    _check("kvx_f32_to_f16_trunc", lib.kvx_f32_to_f16_trunc(_ptr(x), _ptr(out), x.numel(),
                                                            _stream(stream)))
    return out


def f16_trunc_to_f32(h, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty(h.numel(), dtype=torch.float32, device=h.device)
    _check("kvx_f16_trunc_to_f32", lib.kvx_f16_trunc_to_f32(_ptr(h), _ptr(out), h.numel(),
                                                            _stream(stream)))
    return out


def softmax_rows(x, out=None, stream=None):
    """Row softmax of a [rows][cols] fp32 CUDA tensor (TensorOps::softmax)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    _check("kvx_softmax_rows", lib.kvx_softmax_rows(_ptr(x), _ptr(out), C.c_int64(x.shape[0]),
                                                    C.c_int64(x.shape[1]), _stream(stream)))
    return out


def attention_dense(q, k, v, out=None, scale=0.0, stream=None):
    """softmax(q k^T * scale) v for fp32 CUDA tensors q [seq_q][dim],
    k / v [seq_k][dim] (TensorOps::attention; scale <= 0 -> 1/sqrt(dim))."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(q)
    _check("kvx_attention_dense",
           lib.kvx_attention_dense(_ptr(q), _ptr(k), _ptr(v), _ptr(out), C.c_int64(q.shape[0]),
                                   C.c_int64(k.shape[0]), C.c_int32(q.shape[1]), C.c_float(scale),
                                   _stream(stream)))
    return out


def lru_select(stamps, victim=None, stream=None):
    torch = _torch()
    if victim is None:
        victim = torch.empty(1, dtype=torch.int32, device=stamps.device)
    _check("kvx_lru_select", lib.kvx_lru_select(_ptr(stamps), stamps.numel(), _ptr(victim),
                                                _stream(stream)))
    return victim


def migrate_frames(dev_base, dev_capacity, host_base, host_capacity, dev_frames, host_frames,
                   frame_bytes, direction, ctas=0, error_flag=None, stream=None):
    """dev_base/host_base: raw addresses (int) or tensors; frames: int32 CUDA tensors."""
    def addr(x):
        return C.c_void_p(x if isinstance(x, int) else x.data_ptr())
    rc = lib.kvx_migrate_frames(addr(dev_base), dev_capacity, addr(host_base), host_capacity,
                                _ptr(dev_frames), _ptr(host_frames), dev_frames.numel(),
                                frame_bytes, direction, ctas, _ptr(error_flag), _stream(stream))
    _check("kvx_migrate_frames", rc)


EVICT_LRU, EVICT_TOKEN_WEIGHTED, EVICT_ATTENTION_BASED, EVICT_PREDICTIVE = 0, 1, 2, 3


def evict_select(policy, pages, decay=0.95, predicted=None, out=None, stream=None):
    """AdvancedEvictionPolicy selectPageToEvict on the device.  pages: CUDA
    uint8 tensor holding n EvictionMetrics records of 48 bytes."""
    torch = _torch()
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=pages.device)
    _check("kvx_evict_select", lib.kvx_evict_select(policy, _ptr(pages), pages.numel() // 48, decay,
                                                    _ptr(predicted), _ptr(out), _stream(stream)))
    return out


def evict_select_composite(policies, weights, pages, decay=0.95, predicted=None, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=pages.device)
    pol = (C.c_int32 * len(policies))(*policies)
    w = (C.c_float * len(weights))(*[float(x) for x in weights])
    _check("kvx_evict_select_composite",
           lib.kvx_evict_select_composite(pol, w, len(policies), _ptr(pages), pages.numel() // 48, decay,
                                          _ptr(predicted), _ptr(out), _stream(stream)))
    return out


def decode_attn(pool, block_table, seq_lens, q, out=None, stats=None, page_mass=None, workspace=None,
                error_flag=None, sm_scale=0.0, stream=None):
    """Paged decode plus each page's attention mass ([batch][max_pages], mean
    over q-heads).  Returns (out, page_mass)."""
    torch = _torch()
    kv = paged(pool, stats)
    batch, hq, _ = q.shape
    mp = block_table.shape[1]
    if out is None:
        out = torch.empty_like(q)
    if page_mass is None:
        page_mass = torch.empty((batch, mp), dtype=torch.float32, device=q.device)
    if workspace is None:
        workspace = torch.zeros(lib.kvx_decode_attn_workspace_bytes(batch, hq, mp, PAGE_TOKENS),
                                dtype=torch.uint8, device=q.device)
    rc = lib.kvx_decode_attn(C.byref(kv), _ptr(block_table), mp, _ptr(seq_lens), batch, hq, _ptr(q), _ptr(out),
                             _dtype_code(q), sm_scale, _ptr(workspace), workspace.numel(), _ptr(page_mass),
                             _ptr(error_flag), _stream(stream))
    _check("kvx_decode_attn", rc)
    return out, page_mass


def attn_to_metrics(page_mass, block_table, seq_lens, metrics, current_token, stream=None):
    """Fold one step's page_mass into EvictionMetrics records (CUDA uint8
    tensor of 48-byte records indexed by physical page)."""
    rc = lib.kvx_attn_to_metrics(_ptr(page_mass), _ptr(block_table), block_table.shape[1], _ptr(seq_lens),
                                 block_table.shape[0], _ptr(metrics), metrics.numel() // 48, current_token,
                                 _stream(stream))
    _check("kvx_attn_to_metrics", rc)
