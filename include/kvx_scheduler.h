/*
 * kvx_scheduler.h -- C entry points over the Scheduler drop-in
 * (include/scheduler.h; the reference's scheduler/scheduler.cpp:15-37), for
 * hosts that drive prefetch from C or through an FFI the way the
 * reference's InferenceController::schedulePrefetch does
 * (runtime/inference.cpp:61-84): ask for a depth at the current position,
 * prefetch the next `depth` units, report each load's latency.
 *
 * The reference's Scheduler reads the cache's size() and capacity() when
 * asked for a depth; here the caller passes both with the question (for
 * the frame store: resident frames and capacity).
 */
#ifndef KVX_SCHEDULER_H
#define KVX_SCHEDULER_H

#include <stdint.h>

#include "kvx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kvx_scheduler kvx_scheduler;

/* A Scheduler with the reference's max_depth (its default: 4). */
KVX_API int kvx_scheduler_create(int32_t max_depth, kvx_scheduler **out);
KVX_API void kvx_scheduler_destroy(kvx_scheduler *s);
/* Scheduler::observeLoadLatency: one load took `ms` milliseconds. */
KVX_API int kvx_scheduler_observe(kvx_scheduler *s, double ms);
/* Scheduler::getPrefetchDepth(current) over a cache holding `size` of
 * `capacity` entries: clamp(round(max_depth * min(2, avg_ms / 50) *
 * (1 - size / capacity)), 1, max_depth). */
KVX_API int kvx_scheduler_depth(kvx_scheduler *s, int32_t current, int64_t size, int64_t capacity,
                                int32_t *depth);

#ifdef __cplusplus
}
#endif
#endif
