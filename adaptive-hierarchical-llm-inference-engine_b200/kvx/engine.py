"""ctypes front end of the engine C ABI (include/adaptive_engine.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import KvPaged, KvxError, lib


class NativeEngineApi(C.Structure):
    _fields_ = [("start", C.CFUNCTYPE(None)), ("stop", C.CFUNCTYPE(None)),
                ("prefetchLayer", C.CFUNCTYPE(C.c_long, C.c_int)),
                ("evictLayer", C.CFUNCTYPE(C.c_long, C.c_int)),
                ("keepLayer", C.CFUNCTYPE(C.c_long, C.c_int)),
                ("moveKvToRam", C.CFUNCTYPE(C.c_long, C.c_long)),
                ("moveKvToGpu", C.CFUNCTYPE(C.c_long, C.c_long)),
                ("compressKv", C.CFUNCTYPE(C.c_long, C.c_long)),
                ("offloadKv", C.CFUNCTYPE(C.c_long, C.c_long)),
                ("getCurrentLayer", C.CFUNCTYPE(C.c_int)),
                ("getGpuMemory", C.CFUNCTYPE(C.c_long)),
                ("getKvPages", C.CFUNCTYPE(C.c_int)),
                ("getCachedLayers", C.CFUNCTYPE(C.c_int))]


class EngineConfig(C.Structure):
    _fields_ = [("layers", C.c_int32), ("kv_heads", C.c_int32), ("q_heads", C.c_int32),
                ("head_dim", C.c_int32), ("page_tokens", C.c_int32), ("max_batch", C.c_int32),
                ("pages_per_layer", C.c_int32), ("gpu_layer_slots", C.c_int32),
                ("device", C.c_int32), ("offload_dir", C.c_char * 256),
                ("ram_layer_slots", C.c_int32), ("int8_layer_slots", C.c_int32)]


lib.adaptive_engine_get_api.restype = C.POINTER(NativeEngineApi)
lib.adaptive_engine_test_release_layer.argtypes = [C.c_int]
lib.adaptive_engine_default_config.argtypes = [C.POINTER(EngineConfig)]
lib.adaptive_engine_configure.argtypes = [C.POINTER(EngineConfig)]
lib.adaptive_engine_configure.restype = C.c_int
lib.adaptive_engine_layer_view.argtypes = [C.c_int, C.POINTER(KvPaged)]
lib.adaptive_engine_layer_view.restype = C.c_int
lib.adaptive_engine_set_sequences.argtypes = [C.c_int32, C.c_void_p, C.c_int32, C.c_uint64]
lib.adaptive_engine_set_sequences.restype = C.c_int
lib.adaptive_engine_decode_step.argtypes = [C.c_void_p] * 4
lib.adaptive_engine_decode_step.restype = C.c_int
lib.adaptive_engine_seq_len.argtypes = [C.c_int32]
lib.adaptive_engine_seq_len.restype = C.c_int32
lib.adaptive_engine_layer_tier.argtypes = [C.c_int]
lib.adaptive_engine_layer_tier.restype = C.c_int
lib.adaptive_engine_device_bytes.restype = C.c_longlong
lib.adaptive_engine_load_layer.argtypes = [C.c_int, C.c_void_p]
lib.adaptive_engine_load_layer.restype = C.c_int
lib.adaptive_engine_read_layer.argtypes = [C.c_int, C.c_void_p]
lib.adaptive_engine_read_layer.restype = C.c_int
lib.adaptive_engine_block_table.argtypes = [C.c_void_p]
lib.adaptive_engine_block_table.restype = C.c_int32
lib.adaptive_engine_nccl_unique_id.argtypes = [C.c_void_p]
lib.adaptive_engine_nccl_unique_id.restype = C.c_int
lib.adaptive_engine_set_comm.argtypes = [C.c_int, C.c_int, C.c_void_p]
lib.adaptive_engine_set_comm.restype = C.c_int

lib.adaptive_engine_step_in_flight.restype = C.c_int
lib.adaptive_engine_set_readback_share.argtypes = [C.c_int]
lib.adaptive_engine_set_readback_share.restype = C.c_int

lib.adaptive_engine_compress_aged.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_void_p]
lib.adaptive_engine_compress_aged.restype = C.c_int
lib.adaptive_engine_layer_last_access_ms.argtypes = [C.c_int]
lib.adaptive_engine_layer_last_access_ms.restype = C.c_int64

TIERS = {0: "GPU", 1: "RAM", 2: "COMPRESSED", 3: "OFFLOADED", 4: "COMPRESSED_NF4"}


def api() -> NativeEngineApi:
    return lib.adaptive_engine_get_api().contents


def default_config() -> EngineConfig:
    c = EngineConfig()
    lib.adaptive_engine_default_config(C.byref(c))
    return c


def configure(**kw) -> EngineConfig:
    c = default_config()
    for k, v in kw.items():
        setattr(c, k, v.encode() if isinstance(v, str) else v)
    rc = lib.adaptive_engine_configure(C.byref(c))
    if rc != 0:
        raise KvxError("adaptive_engine_configure", rc)
    return c


def layer_view(layer: int) -> KvPaged:
    v = KvPaged()
    rc = lib.adaptive_engine_layer_view(layer, C.byref(v))
    if rc != 0:
        raise KvxError("adaptive_engine_layer_view", rc)
    return v


def set_sequences(lens, reserve_tokens=0, seed=0):
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    rc = lib.adaptive_engine_set_sequences(lens.size, lens.ctypes.data, reserve_tokens, seed)
    if rc != 0:
        raise KvxError("adaptive_engine_set_sequences", rc)


def decode_step(q, k, v, out):
    """q/k/v/out: host buffers (numpy fp16 or pinned torch CPU tensors); out
    may be None (no read-back)."""
    def ptr(a):
        if a is None:
            return None
        return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()
    rc = lib.adaptive_engine_decode_step(ptr(q), ptr(k), ptr(v), ptr(out))
    if rc != 0:
        raise KvxError("adaptive_engine_decode_step", rc)


def tier(layer: int) -> str:
    return TIERS.get(lib.adaptive_engine_layer_tier(layer), "invalid")


def _ptr(a):
    return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()


def load_layer(layer: int, src):
    rc = lib.adaptive_engine_load_layer(layer, _ptr(src))
    if rc != 0:
        raise KvxError("adaptive_engine_load_layer", rc)


def read_layer(layer: int, dst):
    rc = lib.adaptive_engine_read_layer(layer, _ptr(dst))
    if rc != 0:
        raise KvxError("adaptive_engine_read_layer", rc)


def block_table(batch: int) -> np.ndarray:
    mp = lib.adaptive_engine_block_table(None)
    out = np.empty((batch, max(mp, 1)), np.int32)
    lib.adaptive_engine_block_table(out.ctypes.data)
    return out


def nccl_unique_id() -> bytes:
    buf = (C.c_char * 128)()
    rc = lib.adaptive_engine_nccl_unique_id(buf)
    if rc != 0:
        raise KvxError("adaptive_engine_nccl_unique_id", rc)
    return bytes(buf)


def set_comm(rank: int, world: int, uid: bytes):
    buf = (C.c_char * 128).from_buffer_copy(uid)
    rc = lib.adaptive_engine_set_comm(rank, world, buf)
    if rc != 0:
        raise KvxError("adaptive_engine_set_comm", rc)


def set_readback_share(share: bool):
    """Multi-GPU read-back: each rank copies back only layers l % world == rank."""
    rc = lib.adaptive_engine_set_readback_share(1 if share else 0)
    if rc != 0:
        raise KvxError("adaptive_engine_set_readback_share", rc)


def compress_aged(int8_threshold_ms, compressed_threshold_ms, now_ms=-1, apply=True, layers=None):
    """The Java KVCompressionEngine's age policy over the engine's layers.
    Returns (layers compressed, per-layer decisions 0 none / 1 INT8 / 2 COMPRESSED)."""
    n = layers if layers is not None else lib.adaptive_engine_get_api().contents.getKvPages()
    d = np.zeros(max(n, 1), np.int32)
    rc = lib.adaptive_engine_compress_aged(int(int8_threshold_ms), int(compressed_threshold_ms), int(now_ms),
                                           1 if apply else 0, d.ctypes.data)
    if rc < 0:
        raise KvxError("adaptive_engine_compress_aged", rc)
    return rc, d[:n]


def last_access_ms(layer: int) -> int:
    return int(lib.adaptive_engine_layer_last_access_ms(layer))
