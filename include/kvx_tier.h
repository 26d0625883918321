/*
 * kvx_tier.h -- the tiered page-frame store: a device pool of fixed-size KV
 * frames backed by a pinned host arena, with the reference's LRU policy
 * deciding residency and batched copy kernels moving the frames.
 *
 * Replaces, for page frames:
 *   KVManager::load_page / evict_page / contains   cache/kv_cache.cpp:86-148
 *     (LRU list: a hit moves the page to the front; a miss with
 *      size >= capacity evicts lru_.back() first, then inserts at the front)
 *   KVCacheGPU::transferToGPU / transferToHost / evictLRUPage
 *                                                 native-engine/cpp/KVCacheGPU.cpp:68-152
 *     (one synchronous cudaMemcpy per page there; here one gather/scatter
 *      launch per step and direction, kvx_migrate_frames)
 *   RuntimeMemory::allocatePinnedHost             native-engine/cpp/RuntimeMemory.cpp:362-410
 *     (one pinned arena sliced into frames instead of a first-fit pool)
 *
 * Frames live in exactly one tier.  A frame id is any integer in
 * [0, universe); a frame's bytes are opaque (for the KV pools of this
 * library a frame is one page of all kv heads: [2][kv_heads][16][128] fp16,
 * 64 KiB for 8 heads, so the device arena is directly a kvx_paged pool with
 * num_pages = device frames).
 *
 * Initial state: frames 0 .. capacity-1 are resident in device slots
 * 0 .. capacity-1, in LRU order by id (frame 0 least recent), exactly as if
 * they had been loaded one by one in that order; every other frame f sits
 * in host slot f - capacity.  `spare` more device and host slots are free:
 * they let the loads of a step (H2D) run on one copy stream while the
 * write-backs of its victims (D2H) run on another, so both directions of
 * the host link are busy at once.
 *
 * A step takes the accesses of one decode step in order and applies the
 * policy serially (decisions bit-identical to replaying the same id stream
 * through KVManager with the same capacity), then enqueues the copies.  The
 * caller makes its decode wait for them (kvx_tier_wait_resident) and tells
 * the store when that decode has been enqueued (kvx_tier_mark_read), so a
 * later step never overwrites a frame before the decode that reads it ran.
 *
 * Disk tier (optional).  With host_frames > 0 the pinned arena holds at
 * most host_frames frames (plus `spare`); every other non-resident frame
 * lives in one spill file (spill_path) at offset frame * frame_bytes -- the
 * GPU -> RAM -> SSD chain of the reference's KVPageState
 * (src/main/java/com/adaptivellm/kv/KVPageState.java).  Initially frames
 * capacity .. capacity+host_frames-1 are in RAM (host slots 0..), the rest
 * on disk (their bytes: kvx_tier_write_frame).  The RAM tier is a FIFO of
 * arrivals: when a write-back needs a host slot and RAM is full, the frame
 * that entered RAM first goes to disk (pwrite, after any copy still writing
 * its slot finished); a miss on a disk frame is read into a host slot
 * during kvx_tier_step (pread) and then loaded like any RAM frame.  Device
 * residency decisions are unchanged (KVManager's LRU).
 *
 * Bookkeeping-only stores (device = -1) allocate no device or pinned memory
 * and copy nothing: they run the policy and the slot assignment alone.
 */
#ifndef KVX_TIER_H
#define KVX_TIER_H

#include <stddef.h>
#include <stdint.h>

#include "kvx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kvx_tier kvx_tier;

typedef struct kvx_tier_config {
    size_t frame_bytes;  /* bytes per frame, multiple of 16 */
    int64_t universe;    /* frame ids are [0, universe) */
    int64_t capacity;    /* frames resident on the device at most (the policy's capacity) */
    int64_t spare;       /* extra device and host slots; must cover the misses of one step */
    int32_t device;      /* CUDA device ordinal, or -1 for a bookkeeping-only store */
    int32_t load_ctas;   /* CTAs of a load launch (0: 16) */
    int32_t store_ctas;  /* CTAs of a write-back launch (0: 4).  Loads are reads of
                            host memory by the SMs and need more requests in
                            flight than write-backs; 16 + 4 keeps both directions
                            of the host link busy when they run together */
    int64_t host_frames; /* RAM tier size; 0: every non-resident frame in RAM (no disk) */
    const char *spill_path; /* disk tier file (created / truncated) when host_frames > 0 */
    int32_t device_policy;  /* 1: the policy's bookkeeping (recency, free slots, copy lists)
                               lives on the device and runs as kernels: steps take device
                               arrays (kvx_tier_step_device) and no host work is left per
                               step.  RAM tier only (host_frames 0), device >= 0 */
    int64_t max_step;       /* device_policy: accesses per step at most (< capacity) */
    int32_t lookahead;      /* L, 0..62: steps that may be planned ahead of the reads.  Step s
                               may be planned once the reads of steps up to s-L-2 are marked
                               (KVX_EBUSY otherwise); kvx_tier_wait_resident and
                               kvx_tier_mark_read then address the oldest step not yet
                               marked.  A device slot a victim frees is taken again no earlier
                               than L+1 steps later, so `spare` must cover about L+1 steps'
                               loads (KVX_ENOSPC otherwise).  0: plan, read, mark, one step
                               at a time (wait / mark address the last step planned) */
} kvx_tier_config;

typedef struct kvx_tier_stats {
    int64_t accesses;
    int64_t hits;
    int64_t misses;
    int64_t evictions;
    int64_t reloads;     /* victims of a step accessed again later in the same step */
    int64_t frames_h2d;  /* frames copied host -> device */
    int64_t frames_d2h;  /* frames copied device -> host */
    int64_t frames_disk_read;   /* frames read from the spill file */
    int64_t frames_disk_write;  /* frames written to the spill file */
} kvx_tier_stats;

/* Allocate the store (device arena of capacity + spare frames, pinned host
 * arena of universe - capacity + spare frames) and place the initial state.
 * KVX_EINVAL for a bad config, KVX_ENOSPC / KVX_ECUDA when memory cannot be
 * had. */
KVX_API int kvx_tier_create(const kvx_tier_config *cfg, kvx_tier **out);
/* Wait for outstanding copies and free everything. */
KVX_API void kvx_tier_destroy(kvx_tier *t);

/* Base address and slot count of the device arena (slot s at base + s *
 * frame_bytes) and of the pinned host arena (mapped: usable from kernels). */
KVX_API int kvx_tier_device_arena(kvx_tier *t, void **base, int64_t *slots);
KVX_API int kvx_tier_host_arena(kvx_tier *t, void **base, int64_t *slots);

/* Where frame f is now: *tier = 0 device / 1 host / 2 disk, *slot its slot
 * there (disk: the frame id, its file offset / frame_bytes). */
KVX_API int kvx_tier_location(kvx_tier *t, int64_t frame, int32_t *tier, int64_t *slot);
/* Copy frame f's bytes from / to host memory `buf` wherever the frame is
 * (synchronous; waits for the store's copies first).  For filling a store
 * and for checking it. */
KVX_API int kvx_tier_write_frame(kvx_tier *t, int64_t frame, const void *buf);
KVX_API int kvx_tier_read_frame(kvx_tier *t, int64_t frame, void *buf);

/* One step: accesses frames[0..n) in order.  For access i, dev_slot[i]
 * receives the device slot the frame occupies for this step's reads;
 * evicted[i] (optional) the frame evicted by this access or -1; hit[i]
 * (optional) 1 for a hit.  Copies are enqueued on the store's copy streams
 * and not waited for.  n must be smaller than capacity; KVX_ENOSPC when the
 * step misses more frames than `spare` can take (nothing is changed then). */
KVX_API int kvx_tier_step(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot,
                          int32_t *evicted, uint8_t *hit, kvx_tier_stats *stats);
/* A step with its bookkeeping on the device (config device_policy = 1):
 * frames, dev_slot, evicted, hit are DEVICE arrays; the policy's kernels run
 * on the store's own stream after the work queued so far on `stream` (so
 * `frames` may be written there), the copies follow them, and dev_slot is
 * ready for work that waits with kvx_tier_wait_resident (work queued on
 * `stream` after that wait may rewrite frames and the outputs).  Decisions are
 * KVManager's, exactly as kvx_tier_step makes them; placement (which free
 * slot a load takes) may differ.  n <= max_step.  A step with an id out of
 * range or more loads than free slots is rejected on the device (nothing
 * changes) and reported by kvx_tier_sync (KVX_EINVAL, KVX_ENOSPC).  Host-array
 * kvx_tier_step on such a store copies through the device and waits. */
KVX_API int kvx_tier_step_device(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot,
                                 int32_t *evicted, uint8_t *hit, void *stream);
/* Device-policy stores: the stream the plans (the policy's kernels) run on,
 * for ordering or timing other work against them; KVX_EUNSUPPORTED on a
 * host-policy store. */
KVX_API int kvx_tier_plan_stream(kvx_tier *t, void **stream);
/* Make `stream` wait until every frame of the reading step is resident:
 * the last step planned (lookahead 0) or the oldest step not yet marked. */
KVX_API int kvx_tier_wait_resident(kvx_tier *t, void *stream);
/* The reads of the reading step's frames have been enqueued on `stream`; a
 * later step that evicts one of them first waits for that work.  With a
 * lookahead, the next step becomes the reading step (every step is marked
 * once, in order; KVX_EINVAL when all planned steps are marked). */
KVX_API int kvx_tier_mark_read(kvx_tier *t, void *stream);
/* Block until all enqueued copies finished; KVX_EINVAL if a copy met a bad
 * slot (never expected), KVX_ECUDA on a CUDA error. */
KVX_API int kvx_tier_sync(kvx_tier *t);
/* Cumulative counters since create. */
KVX_API int kvx_tier_totals(kvx_tier *t, kvx_tier_stats *stats);

#ifdef __cplusplus
}
#endif
#endif
