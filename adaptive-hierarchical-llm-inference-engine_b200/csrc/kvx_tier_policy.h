// kvx_tier_policy.h -- the page-frame store's LRU bookkeeping on the device
// (private to the library: used by engine/tier.cpp, implemented in
// csrc/kvx_tier_dev.cu).  Plain C++: no CUDA syntax, so host-compiled code
// can include it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kvx_tier.h"

namespace kvx_tier_dev {

struct Policy;

// Device state for a store of `universe` frames, `capacity` of them
// resident: frames 0 .. resident0-1 start in device slots 0 .. resident0-1
// (frame 0 least recently used), frames resident0 .. resident0+host_cap-1 in
// host slots 0 .., the remaining device slots [resident0, dev_slots) and host
// slots [host_cap, host_slots) free.  max_step bounds the accesses of one
// step.  Returns a kvx_status.
int create(Policy **out, int64_t universe, int64_t capacity, int64_t resident0, int64_t dev_slots,
           int64_t host_slots, int64_t host_cap, int64_t max_step);
void destroy(Policy *p);

// One step (number step_no) over frames[0..n) (device array), enqueued on
// `st`, its copy lists in the buffers of `parity`:
// dev_slot[i] (device) receives the slot frame i occupies for this step's
// reads, hit[i] / evicted[i] (device, optional) the decisions; the step's
// copy lists are left on the device (lists()).  Decisions equal KVManager's
// serial LRU replay.  Free device slots form a FIFO; a load takes only a
// slot freed by step min_freed or earlier.  A step with more loads than such
// slots (or free host slots), or an id out of range, sets the policy's error
// word and changes nothing.
int step(Policy *p, int parity, int64_t step_no, int64_t min_freed, const int32_t *frames, int64_t n,
         int32_t *dev_slot, uint8_t *hit, int32_t *evicted, cudaStream_t st);

// Device arrays of the copies of the last step of that parity: loads
// (h2d_dev[i] <- h2d_host[i]) and write-backs (d2h_dev[i] -> d2h_host[i]);
// counts[0] loads, counts[1] write-backs (device int32).  A step of parity
// q rewrites parity q's arrays, so it must not start before the copies of
// the step two before it have read them.
void lists(Policy *p, int parity, const int32_t **h2d_dev, const int32_t **h2d_host, const int32_t **d2h_dev,
           const int32_t **d2h_host, const int32_t **counts);

// Synchronous reads and updates, ordered on  (the policy's stream).
int totals(Policy *p, kvx_tier_stats *stats, cudaStream_t st);
int location(Policy *p, int64_t frame, int32_t *tier, int64_t *slot, cudaStream_t st);
// The error word (bits: 1 id out of range, 2 more loads than free slots,
// 4 / 8 internal limits); `clear` resets it.
int error(Policy *p, int32_t *err, bool clear, cudaStream_t st);

// Frame migration with the frame count in device memory (count_dev[0]),
// at most max_frames frames.
int migrate_counted(void *dev_base, int32_t dev_capacity, void *host_base, int32_t host_capacity,
                    const int32_t *dev_frames, const int32_t *host_frames, const int32_t *count_dev,
                    int32_t max_frames, size_t frame_bytes, int32_t direction, int32_t ctas,
                    int32_t *error_flag, cudaStream_t st);

}  // namespace kvx_tier_dev
