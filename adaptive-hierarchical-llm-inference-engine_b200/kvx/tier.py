"""Tiered page-frame store: ctypes front end of include/kvx_tier.h.

A device pool of fixed-size frames backed by a pinned host arena; the
reference's KVManager LRU (cache/kv_cache.cpp:86-148) decides which frames
are resident, and each step's loads and write-backs run as one batched copy
launch per direction on two copy streams.

    t = Tier(frame_bytes=65536, universe=U, capacity=C, spare=S)
    slots, evicted, hit, st = t.step(frame_ids)   # policy + copies enqueued
    t.wait_resident(stream)                       # decode waits for the loads
    ... decode over t.paged(kv_heads) with block tables built from `slots` ...
    t.mark_read(stream)                           # later steps respect the reads

`device=-1` gives a bookkeeping-only store (no GPU memory, no copies): the
policy and the slot assignment alone, usable on a machine without a GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import HEAD_DIM, KVX_F16, PAGE_TOKENS, KvPaged, _check, lib


class TierConfig(C.Structure):
    _fields_ = [("frame_bytes", C.c_size_t), ("universe", C.c_int64), ("capacity", C.c_int64),
                ("spare", C.c_int64), ("device", C.c_int32), ("load_ctas", C.c_int32),
                ("store_ctas", C.c_int32), ("host_frames", C.c_int64), ("spill_path", C.c_char_p),
                ("device_policy", C.c_int32), ("max_step", C.c_int64), ("lookahead", C.c_int32)]


_STAT_FIELDS = ("accesses", "hits", "misses", "evictions", "reloads", "frames_h2d", "frames_d2h",
                "frames_disk_read", "frames_disk_write")


class TierStats(C.Structure):
    _fields_ = [(n, C.c_int64) for n in _STAT_FIELDS]

    def as_dict(self):
        return {n: int(getattr(self, n)) for n in _STAT_FIELDS}


_vp, _i64 = C.c_void_p, C.c_int64
lib.kvx_tier_create.argtypes = [C.POINTER(TierConfig), C.POINTER(_vp)]
lib.kvx_tier_create.restype = C.c_int
lib.kvx_tier_destroy.argtypes = [_vp]
lib.kvx_tier_destroy.restype = None
lib.kvx_tier_device_arena.argtypes = [_vp, C.POINTER(_vp), C.POINTER(_i64)]
lib.kvx_tier_host_arena.argtypes = [_vp, C.POINTER(_vp), C.POINTER(_i64)]
lib.kvx_tier_location.argtypes = [_vp, _i64, C.POINTER(C.c_int32), C.POINTER(_i64)]
lib.kvx_tier_step.argtypes = [_vp, _vp, _i64, _vp, _vp, _vp, C.POINTER(TierStats)]
lib.kvx_tier_step_device.argtypes = [_vp, _vp, _i64, _vp, _vp, _vp, _vp]
lib.kvx_tier_plan_stream.argtypes = [_vp, C.POINTER(_vp)]
lib.kvx_tier_wait_resident.argtypes = [_vp, _vp]
lib.kvx_tier_mark_read.argtypes = [_vp, _vp]
lib.kvx_tier_sync.argtypes = [_vp]
lib.kvx_tier_totals.argtypes = [_vp, C.POINTER(TierStats)]
lib.kvx_tier_write_frame.argtypes = [_vp, _i64, _vp]
lib.kvx_tier_read_frame.argtypes = [_vp, _i64, _vp]
for _fn in ("kvx_tier_device_arena", "kvx_tier_host_arena", "kvx_tier_location", "kvx_tier_step",
            "kvx_tier_step_device", "kvx_tier_plan_stream",
            "kvx_tier_wait_resident", "kvx_tier_mark_read", "kvx_tier_sync", "kvx_tier_totals",
            "kvx_tier_write_frame", "kvx_tier_read_frame"):
    getattr(lib, _fn).restype = C.c_int


def _np_ptr(a):
    return None if a is None else a.ctypes.data_as(_vp)


def _stream_ptr(stream):
    if stream is None:
        import torch
        return _vp(torch.cuda.current_stream().cuda_stream)
    return _vp(stream if isinstance(stream, int) else stream.cuda_stream)


class _DeviceBytes:
    """__cuda_array_interface__ over a raw device range (zero-copy torch view)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class Tier:
    def __init__(self, frame_bytes, universe, capacity, spare, device=0, load_ctas=0, store_ctas=0,
                 host_frames=0, spill_path=None, device_policy=False, max_step=0, lookahead=0):
        """device_policy: the LRU bookkeeping runs as kernels on the device
        (step_device takes device tensors); max_step bounds a step's accesses.
        lookahead: steps that may be planned ahead of the reads (wait_resident
        and mark_read then address the oldest step not yet marked)."""
        self._path = None if spill_path is None else str(spill_path).encode()
        self.cfg = TierConfig(frame_bytes, universe, capacity, spare, device, load_ctas, store_ctas,
                              host_frames, self._path, 1 if device_policy else 0, max_step, lookahead)
        h = _vp()
        _check("kvx_tier_create", lib.kvx_tier_create(C.byref(self.cfg), C.byref(h)))
        self.h = h
        self.frame_bytes = frame_bytes

    def close(self):
        if self.h:
            lib.kvx_tier_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_arena(self):
        base, n = _vp(), _i64()
        _check("kvx_tier_device_arena", lib.kvx_tier_device_arena(self.h, C.byref(base), C.byref(n)))
        return base.value, n.value

    def host_arena(self):
        base, n = _vp(), _i64()
        _check("kvx_tier_host_arena", lib.kvx_tier_host_arena(self.h, C.byref(base), C.byref(n)))
        return base.value, n.value

    def device_tensor(self):
        """The device arena as a flat uint8 torch tensor (no copy)."""
        import torch
        base, n = self.device_arena()
        return torch.as_tensor(_DeviceBytes(base, n * self.frame_bytes), device="cuda")

    def host_array(self):
        """The pinned host arena as a flat uint8 numpy array (no copy)."""
        base, n = self.host_arena()
        return np.ctypeslib.as_array(C.cast(base, C.POINTER(C.c_uint8)), shape=(n * self.frame_bytes,))

    def paged(self, kv_heads):
        """The device arena as an fp16 kvx_paged pool (one frame = one page of
        [2][kv_heads][16][128])."""
        assert self.frame_bytes == 2 * kv_heads * PAGE_TOKENS * HEAD_DIM * 2
        base, n = self.device_arena()
        return KvPaged(base, 0, KVX_F16, n, kv_heads, HEAD_DIM, PAGE_TOKENS)

    def location(self, frame):
        tier, slot = C.c_int32(), _i64()
        _check("kvx_tier_location", lib.kvx_tier_location(self.h, frame, C.byref(tier), C.byref(slot)))
        return ("device", "host", "disk")[tier.value], slot.value

    def write_frame(self, frame, data):
        """Set frame's bytes wherever it lives (numpy array of frame_bytes)."""
        buf = np.ascontiguousarray(data).view(np.uint8)
        assert buf.size == self.frame_bytes
        _check("kvx_tier_write_frame", lib.kvx_tier_write_frame(self.h, frame, buf.ctypes.data))

    def read_frame(self, frame):
        out = np.empty(self.frame_bytes, np.uint8)
        _check("kvx_tier_read_frame", lib.kvx_tier_read_frame(self.h, frame, out.ctypes.data))
        return out

    def step(self, frames, dev_slot=None, evicted=True, hit=True):
        """Apply the policy to `frames` (int32, in order) and enqueue the copies.
        Returns (dev_slot, evicted or None, hit or None, stats dict)."""
        frames = np.ascontiguousarray(frames, dtype=np.int32)
        n = frames.size
        if dev_slot is None:
            dev_slot = np.empty(n, np.int32)
        ev = np.empty(n, np.int32) if evicted else None
        ht = np.empty(n, np.uint8) if hit else None
        st = TierStats()
        _check("kvx_tier_step", lib.kvx_tier_step(self.h, _np_ptr(frames), n, _np_ptr(dev_slot),
                                                  _np_ptr(ev), _np_ptr(ht), C.byref(st)))
        return dev_slot, ev, ht, st.as_dict()

    def step_device(self, frames, dev_slot, evicted=None, hit=None, stream=None):
        """A step planned on the device (device_policy stores): frames, dev_slot
        and the optional evicted (int32) / hit (uint8) are CUDA tensors; the
        plan runs after the work queued on `stream`, dev_slot is ready for work
        that waits with wait_resident."""
        def p(t):
            return None if t is None else _vp(t.data_ptr())
        _check("kvx_tier_step_device",
               lib.kvx_tier_step_device(self.h, p(frames), frames.numel(), p(dev_slot), p(evicted), p(hit),
                                        _stream_ptr(stream)))

    def plan_stream(self):
        """Device-policy stores: the stream the plans run on (torch ExternalStream)."""
        import torch
        st = _vp()
        _check("kvx_tier_plan_stream", lib.kvx_tier_plan_stream(self.h, C.byref(st)))
        return torch.cuda.ExternalStream(st.value)

    def _sp(self, stream):
        return _vp(0) if self.cfg.device < 0 else _stream_ptr(stream)

    def wait_resident(self, stream=None):
        _check("kvx_tier_wait_resident", lib.kvx_tier_wait_resident(self.h, self._sp(stream)))

    def mark_read(self, stream=None):
        _check("kvx_tier_mark_read", lib.kvx_tier_mark_read(self.h, self._sp(stream)))

    def sync(self):
        _check("kvx_tier_sync", lib.kvx_tier_sync(self.h))

    def totals(self):
        st = TierStats()
        _check("kvx_tier_totals", lib.kvx_tier_totals(self.h, C.byref(st)))
        return st.as_dict()
