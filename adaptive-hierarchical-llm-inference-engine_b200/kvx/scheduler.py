"""Prefetch depth: ctypes front end of include/kvx_scheduler.h (the
reference's Scheduler, scheduler/scheduler.cpp:15-37).

    s = Scheduler(max_depth=4)
    s.observe(load_ms)                      # observeLoadLatency
    d = s.depth(current, size, capacity)    # getPrefetchDepth over a cache of size/capacity
"""
from __future__ import annotations

import ctypes as C

from . import _check, lib

_vp = C.c_void_p
lib.kvx_scheduler_create.argtypes = [C.c_int32, C.POINTER(_vp)]
lib.kvx_scheduler_create.restype = C.c_int
lib.kvx_scheduler_destroy.argtypes = [_vp]
lib.kvx_scheduler_destroy.restype = None
lib.kvx_scheduler_observe.argtypes = [_vp, C.c_double]
lib.kvx_scheduler_observe.restype = C.c_int
lib.kvx_scheduler_depth.argtypes = [_vp, C.c_int32, C.c_int64, C.c_int64, C.POINTER(C.c_int32)]
lib.kvx_scheduler_depth.restype = C.c_int


class Scheduler:
    def __init__(self, max_depth=4):
        h = _vp()
        _check("kvx_scheduler_create", lib.kvx_scheduler_create(max_depth, C.byref(h)))
        self.h = h
        self.max_depth = max_depth

    def close(self):
        if self.h:
            lib.kvx_scheduler_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def observe(self, ms):
        _check("kvx_scheduler_observe", lib.kvx_scheduler_observe(self.h, float(ms)))

    def depth(self, current, size, capacity):
        d = C.c_int32()
        _check("kvx_scheduler_depth", lib.kvx_scheduler_depth(self.h, current, size, capacity, C.byref(d)))
        return d.value
