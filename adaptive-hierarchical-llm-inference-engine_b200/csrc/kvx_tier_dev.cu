// kvx_tier_dev.cu -- the page-frame store's LRU bookkeeping on the device:
// KVManager's policy (cache/kv_cache.cpp:86-148: a hit moves the page to
// the front, a miss with a full cache evicts the back first) over one
// step's accesses, decisions identical to the serial replay, with the
// slots, free lists and copy lists kept in device memory.
//
// Recency is a stamp per frame (the position of its last access in one
// running sequence) and a log, log[stamp % W] = frame, appended for every
// access; an entry is current while stamp[frame] equals its position, so
// the least recently used resident frames are the current entries from the
// log's head on.  A step of n < capacity accesses (the store's own limit)
// touches fewer distinct frames than the capacity, so:
//  * a frame touched in the step is never a victim later in the step (an
//    older, untouched frame is always there), and
//  * the victim of a miss at access t is the first current log entry whose
//    frame is not touched before t; one touched later is evicted now and
//    misses again at its first touch (its slot and bytes are kept, its
//    write-back dropped: the host store's rule).
// Everything but that merge of misses with candidates is data-parallel:
// first touches (atomicMin), the misses of non-resident frames and their
// order (a block scan), slot assignment and copy lists (scans over the
// misses), stamps and log appends.  The merge runs in one CTA: its threads
// fetch and compact the next 1,024 log positions, one thread walks them
// against the misses in time order, a min-heap holding the second misses of
// evicted frames.  The log is compacted (current entries
// renumbered in order) when it fills.
#include <algorithm>
#include <climits>
#include <new>

#include "kvx_common.cuh"
#include "kvx_tier_policy.h"

namespace kvx_tier_dev {
namespace {

constexpr int kT = 1024;     // threads of the single-CTA kernels

// control block (device int64)
enum { kHead, kBase, kResident, kDevFree, kDevHead, kHostFree, kErr, kCompact, kAccesses, kHits, kMisses,
       kEvictions, kReloads, kH2d, kD2h, kCtlN };
// per-step counts (device int32): loads, write-backs, misses of non-resident
// frames, events (misses), evictions, step rejected, and the free lists'
// state before the step (device: count and head of the FIFO; host: stack top)
enum { cLoads, cWbs, cM0, cEvents, cEvict, cBad, cDevCount, cDevHead, cHostTop, cCountsN };

struct View {  // the policy's device arrays, passed by value to the kernels
    int64_t U, C, W, max_n, dev_slots;
    long long *stamp, *ctl, *freed_at;  // freed_at: per device slot, the step that freed it
    int32_t *dslot, *hslot, *first, *evict_ev, *log, *tmp, *dev_free, *host_free;
    int32_t *m0flag, *m0list, *ev_time, *ev_victim, *ev_of_time, *heap;
    int32_t *h2d_dev, *h2d_host, *d2h_dev, *d2h_host, *counts;
};

// Exclusive block scan of one int per thread (blockDim.x == kT); the total
// in *total.  Uses ws[33].
__device__ __forceinline__ int block_scan(int v, int *ws, int *total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) ws[w] = x;
    __syncthreads();
    if (w == 0) {
        const int s = ws[lane];
        int inc = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        ws[lane] = inc - s;
        if (lane == 31) ws[32] = inc;
    }
    __syncthreads();
    const int r = ws[w] + x - v;
    *total = ws[32];
    __syncthreads();
    return r;
}

__global__ void init_kernel(View s, int64_t resident0, int64_t host_cap, int64_t dev_slots, int64_t host_slots) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < s.U; f += stride) {
        const bool res = f < resident0;
        s.stamp[f] = res ? f : -1;
        s.dslot[f] = res ? (int32_t)f : -1;
        s.hslot[f] = (!res && f < resident0 + host_cap) ? (int32_t)(f - resident0) : -1;
        s.first[f] = INT_MAX;
        s.evict_ev[f] = -1;
        if (res) s.log[f] = (int32_t)f;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < s.max_n; i += stride) s.ev_of_time[i] = -1;
    for (int64_t d = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; d < dev_slots; d += stride) {
        if (d < dev_slots - resident0) s.dev_free[d] = (int32_t)(resident0 + d);  // a FIFO from slot resident0
        s.freed_at[d] = LLONG_MIN / 2;  // never used: free for any step
    }
    for (int64_t h = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; h < host_slots - host_cap; h += stride)
        s.host_free[h] = (int32_t)(host_slots - 1 - h);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        for (int i = 0; i < kCtlN; ++i) s.ctl[i] = 0;
        s.ctl[kBase] = resident0;
        s.ctl[kResident] = resident0;
        s.ctl[kDevFree] = dev_slots - resident0;
        s.ctl[kDevHead] = 0;
        s.ctl[kHostFree] = host_slots - host_cap;
    }
}

// first touch of every frame in the step; ids out of range reject the step
__global__ void touch_kernel(View s, const int32_t *__restrict__ frames, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int32_t f = frames[i];
        if (f < 0 || f >= s.U) {
            s.counts[cBad] = 1;
            continue;
        }
        atomicMin(&s.first[f], i);
    }
}

// misses of frames not resident at the step's start (their first touch)
__global__ void classify_kernel(View s, const int32_t *__restrict__ frames, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int32_t f = frames[i];
        s.m0flag[i] = (f >= 0 && f < s.U && s.first[f] == i && s.stamp[f] < 0) ? 1 : 0;
    }
}

// the misses in time order, and the step's room check (one CTA)
__global__ void __launch_bounds__(kT) scan_kernel(View s, int n, long long min_freed) {
    __shared__ int ws[33];
    int base = 0, tot = 0;
    for (int i0 = 0; i0 < n; i0 += kT) {
        const int i = i0 + threadIdx.x;
        const int v = i < n ? s.m0flag[i] : 0;
        const int o = block_scan(v, ws, &tot);
        if (v) s.m0list[base + o] = i;
        base += tot;
    }
    if (threadIdx.x == 0) {
        s.counts[cM0] = base;
        // every such miss loads into a free device slot freed by step
        // min_freed or earlier (the FIFO's first `base` entries), and a
        // write-back (at most one per such miss) takes a free host slot
        if ((long long)base > s.ctl[kDevFree] || (long long)base > s.ctl[kHostFree]) {
            s.counts[cBad] |= 2;
        } else if (base > 0) {
            const int32_t last = s.dev_free[(s.ctl[kDevHead] + base - 1) % s.dev_slots];
            if (s.freed_at[last] > min_freed) s.counts[cBad] |= 2;
        }
        if (s.counts[cBad]) atomicOr(reinterpret_cast<unsigned long long *>(&s.ctl[kErr]),
                                     (unsigned long long)s.counts[cBad]);
    }
}

// The sequential heart: misses in time order against the log's current
// entries from the head on (one CTA).  Most misses evict an untouched
// candidate and come before any pending second miss: such a run is a plain
// zip of the next misses with the next candidates, written by all threads at
// once.
// Thread 0 walks the rest one miss at a time (candidates touched in the
// step, second misses, which wait in a min-heap of times in device memory:
// at most one per eviction, so max_n entries always suffice).  All threads
// refill the candidate window: the next kWin log positions, current entries
// whose frame was not touched before the pending miss (those would only be
// skipped), with the indices of the touched ones listed.
constexpr int kWin = 2 * kT;
constexpr int kMinRun = 8;  // shorter runs are cheaper on thread 0 than a barrier
enum { aDone, aRefill, aZip, aZipRoom };

__global__ void __launch_bounds__(kT) merge_kernel(View s, int n) {
    __shared__ int cand[kWin], ctau[kWin], coff[kWin], tl[kWin];
    __shared__ int ws[33];
    __shared__ int s_act, s_run, s_p0, s_ci, s_k, s_nc, s_ntl, s_tnext, s_lim, s_bad;
    __shared__ long long s_fill, s_fill_end;
    if (s.counts[cBad]) return;
    const long long base = s.ctl[kBase];
    const int m0n = s.counts[cM0];
    const int32_t *__restrict__ m0 = s.m0list;
    int32_t *heap = s.heap;
    // thread 0's state
    long long room = s.C - s.ctl[kResident];  // misses left before the first eviction
    int p0 = 0, ci = 0, tp = 0, k = 0, hn = 0, htop = INT_MAX;
    if (threadIdx.x == 0) {
        s_fill = s_fill_end = s.ctl[kHead];
        s_nc = s_ntl = 0;
        s_bad = 0;
    }
    __syncthreads();
    for (;;) {
        if (threadIdx.x == 0) {
            const int nc = s_nc, ntl = s_ntl;
            int act = aDone, run = 0, tn = INT_MAX;
            for (;;) {
                const int tm = p0 < m0n ? m0[p0] : INT_MAX;
                tn = min(tm, htop);
                if (tn == INT_MAX) break;  // no miss left
                if (room > 0 && hn == 0) {  // free room, misses in m0 order: no victims
                    run = (int)min(room, (long long)(m0n - p0));
                    act = aZipRoom;
                    break;
                }
                if (room <= 0) {
                    while (ci < nc && ctau[ci] < tn) ++ci;  // touched before this miss: more recent now
                    if (ci == nc) {
                        act = aRefill;
                        break;
                    }
                    if (ctau[ci] == INT_MAX && tm < htop) {  // untouched candidates: a zip run?
                        while (tp < ntl && tl[tp] < ci) ++tp;
                        run = min((tp < ntl ? tl[tp] : nc) - ci, m0n - p0);
                        if (hn) run = min(run, kT);  // cut at the pending second miss below
                        if (run >= kMinRun) {
                            act = aZip;
                            break;
                        }
                    }
                }
                // one miss on thread 0: the earlier of the two streams
                int t;
                if (tm < htop) {
                    t = tm;
                    ++p0;
                } else {  // pop the heap's minimum
                    t = htop;
                    const int last = heap[--hn];
                    int i = 0;
                    for (;;) {
                        int c = 2 * i + 1;
                        if (c >= hn) break;
                        if (c + 1 < hn && heap[c + 1] < heap[c]) ++c;
                        if (heap[c] >= last) break;
                        heap[i] = heap[c];
                        i = c;
                    }
                    if (hn) heap[i] = last;
                    htop = hn ? heap[0] : INT_MAX;
                }
                int victim = -1;
                if (room > 0) {
                    --room;
                } else {  // ctau[ci] >= t here
                    victim = cand[ci];
                    const int tau = ctau[ci];
                    ++ci;
                    s.stamp[victim] = -1;
                    s.evict_ev[victim] = k;
                    if (tau != INT_MAX) {  // touched later: a second miss then (tau > t)
                        int i = hn++;
                        while (i > 0 && heap[(i - 1) / 2] > tau) {
                            heap[i] = heap[(i - 1) / 2];
                            i = (i - 1) / 2;
                        }
                        heap[i] = tau;
                        htop = min(htop, tau);
                    }
                }
                s.ev_time[k] = t;
                s.ev_victim[k] = victim;
                s.ev_of_time[t] = k;
                ++k;
            }
            s_act = act;
            s_run = run;
            s_p0 = p0;
            s_ci = ci;
            s_k = k;
            s_tnext = tn;
            s_lim = htop;
        }
        __syncthreads();
        const int act = s_act;
        if (act == aDone) break;
        if (act == aZip || act == aZipRoom) {
            const int q0 = s_p0, c0 = s_ci, k0 = s_k, lim = s_lim;
            int run = s_run;
            if (act == aZip && lim != INT_MAX) {
                // a second miss is pending at time lim: only the misses before
                // it (a prefix, the times are sorted; run <= kT) zip now
                run = __syncthreads_count(threadIdx.x < run && m0[q0 + threadIdx.x] < lim);
            }
            for (int i = threadIdx.x; i < run; i += kT) {
                const int t = m0[q0 + i];
                const int v = act == aZip ? cand[c0 + i] : -1;
                s.ev_time[k0 + i] = t;
                s.ev_victim[k0 + i] = v;
                s.ev_of_time[t] = k0 + i;
                if (v >= 0) {
                    s.stamp[v] = -1;
                    s.evict_ev[v] = k0 + i;
                }
            }
            if (threadIdx.x == 0) {
                p0 += run;
                k += run;
                if (act == aZip) ci += run; else room -= run;
            }
            __syncthreads();  // the zip's shared reads are done before thread 0 goes on
            continue;
        }
        // refill: the next kWin log positions below the step's base
        const long long h = s_fill_end;
        const long long end = min(h + (long long)kWin, base);
        if (h >= end) {  // no candidate left: impossible while n < capacity
            if (threadIdx.x == 0) s_bad = 8;
            break;
        }
        const int tn = s_tnext;
        int c[2], tau[2], valid[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const long long pos = h + 2 * threadIdx.x + j;
            c[j] = -1;
            tau[j] = 0;
            valid[j] = 0;
            if (pos < end) {
                c[j] = s.log[pos % s.W];
                if (c[j] >= 0 && c[j] < s.U && s.stamp[c[j]] == pos) {
                    tau[j] = s.first[c[j]];
                    valid[j] = tau[j] >= tn;  // touched before the pending miss: skipped anyway
                }
            }
        }
        const int touched0 = valid[0] && tau[0] != INT_MAX, touched1 = valid[1] && tau[1] != INT_MAX;
        int tot = 0;
        const int packed = (valid[0] + valid[1]) | ((touched0 + touched1) << 16);
        const int o = block_scan(packed, ws, &tot);
        int oc = o & 0xffff, ot = o >> 16;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (valid[j]) {
                cand[oc] = c[j];
                ctau[oc] = tau[j];
                coff[oc] = 2 * threadIdx.x + j;
                if (tau[j] != INT_MAX) tl[ot++] = oc;
                ++oc;
            }
        }
        if (threadIdx.x == 0) {
            s_fill = h;
            s_fill_end = end;
            s_nc = tot & 0xffff;
            s_ntl = tot >> 16;
            ci = 0;
            tp = 0;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        // the head: the first candidate not consumed (its position), or the
        // end of what was fetched
        s.ctl[kHead] = ci < s_nc ? s_fill + coff[ci] : s_fill_end;
        s.counts[cEvents] = k;
        if (s_bad) {
            s.counts[cBad] |= s_bad;
            atomicOr(reinterpret_cast<unsigned long long *>(&s.ctl[kErr]), (unsigned long long)s_bad);
        }
    }
}

// slots and copy lists of the misses (one CTA, scans over the events)
__global__ void __launch_bounds__(kT) apply_kernel(View s, const int32_t *__restrict__ frames) {
    __shared__ int ws[33];
    if (s.counts[cBad]) return;
    const int E = s.counts[cEvents];
    const long long dev_head = s.ctl[kDevHead], host_top = s.ctl[kHostFree];
    int lb = 0, wb = 0, vb = 0, tot = 0;
    for (int k0 = 0; k0 < E; k0 += kT) {
        const int k = k0 + threadIdx.x;
        int f = -1, v = -1, is_load = 0, is_wb = 0;
        if (k < E) {
            f = frames[s.ev_time[k]];
            v = s.ev_victim[k];
            is_load = s.evict_ev[f] < 0;                  // not evicted earlier in the step
            is_wb = v >= 0 && s.first[v] == INT_MAX;      // not touched again in the step
        }
        const int lo = block_scan(is_load, ws, &tot) + lb;
        lb += tot;
        const int wo = block_scan(is_wb, ws, &tot) + wb;
        wb += tot;
        block_scan(v >= 0 ? 1 : 0, ws, &tot);
        vb += tot;
        if (is_load) {
            const int32_t ds = s.dev_free[(dev_head + lo) % s.dev_slots];
            s.h2d_dev[lo] = ds;
            s.h2d_host[lo] = s.hslot[f];
            s.dslot[f] = ds;
            s.hslot[f] = -1;
        }
        if (is_wb) {
            const int32_t hs = s.host_free[host_top - 1 - wo];
            s.d2h_dev[wo] = s.dslot[v];
            s.d2h_host[wo] = hs;
            s.hslot[v] = hs;
            s.dslot[v] = -1;
        }
    }
    if (threadIdx.x == 0) {
        s.counts[cLoads] = lb;
        s.counts[cWbs] = wb;
        s.counts[cEvict] = vb;
        s.counts[cDevCount] = (int32_t)s.ctl[kDevFree];
        s.counts[cDevHead] = (int32_t)dev_head;
        s.counts[cHostTop] = (int32_t)host_top;
    }
}

// per access: outputs, stamps, log; then every first touch reset
__global__ void finish_kernel(View s, const int32_t *__restrict__ frames, int n, int32_t *dev_slot, uint8_t *hit,
                              int32_t *evicted) {
    const bool bad = s.counts[cBad] != 0;
    const long long base = s.ctl[kBase];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int32_t f = frames[i];
        if (f < 0 || f >= s.U) continue;
        if (!bad) {
            const int k = s.ev_of_time[i];
            dev_slot[i] = s.dslot[f];
            if (hit) hit[i] = k < 0 ? 1 : 0;
            if (evicted) evicted[i] = k >= 0 ? s.ev_victim[k] : -1;
            atomicMax(&s.stamp[f], base + i);
            s.log[(base + i) % s.W] = f;
            s.ev_of_time[i] = -1;
        }
    }
}

// after finish: first touches and eviction marks reset, freed slots pushed,
// counters and totals; the compaction flag when the log is nearly full
__global__ void commit_kernel(View s, const int32_t *__restrict__ frames, int n, long long step_no) {
    const bool bad = s.counts[cBad] != 0;
    const int loads = bad ? 0 : s.counts[cLoads], wbs = bad ? 0 : s.counts[cWbs];
    const int E = bad ? 0 : s.counts[cEvents];
    // the free lists as apply_kernel saw them (thread 0 of block 0 updates ctl below)
    const long long dev_cnt = s.counts[cDevCount], dev_head = s.counts[cDevHead], host_top = s.counts[cHostTop];
    const int stride = gridDim.x * blockDim.x, id = blockIdx.x * blockDim.x + threadIdx.x;
    for (int i = id; i < n; i += stride) {
        const int32_t f = frames[i];
        if (f >= 0 && f < s.U) s.first[f] = INT_MAX;
    }
    for (int k = id; k < E; k += stride) {
        const int32_t v = s.ev_victim[k];
        if (v >= 0) s.evict_ev[v] = -1;
    }
    for (int w = id; w < wbs; w += stride) {  // appended behind the FIFO's last entry
        const int32_t d = s.d2h_dev[w];
        s.dev_free[(dev_head + dev_cnt + w) % s.dev_slots] = d;
        s.freed_at[d] = step_no;
    }
    for (int l = id; l < loads; l += stride) s.host_free[host_top - wbs + l] = s.h2d_host[l];
    if (id == 0 && !bad) {
        s.ctl[kDevFree] = dev_cnt - loads + wbs;
        s.ctl[kDevHead] = (dev_head + loads) % s.dev_slots;
        s.ctl[kHostFree] = host_top - wbs + loads;
        s.ctl[kResident] += E - s.counts[cEvict];
        s.ctl[kAccesses] += n;
        s.ctl[kHits] += n - E;
        s.ctl[kMisses] += E;
        s.ctl[kEvictions] += s.counts[cEvict];
        s.ctl[kReloads] += E - loads;
        s.ctl[kH2d] += loads;
        s.ctl[kD2h] += wbs;
        s.ctl[kBase] += n;
        if (s.ctl[kBase] + s.max_n - s.ctl[kHead] > s.W) s.ctl[kCompact] = 1;
    }
}

// renumber the current log entries 0 .. in order when the log is nearly
// full (one CTA; a no-op otherwise)
__global__ void __launch_bounds__(kT) compact_kernel(View s) {
    __shared__ int ws[33];
    if (!s.ctl[kCompact]) return;
    const long long head = s.ctl[kHead], base = s.ctl[kBase];
    int cnt = 0, tot = 0;
    for (long long p0 = head; p0 < base; p0 += kT) {
        const long long pos = p0 + threadIdx.x;
        int c = -1, valid = 0;
        if (pos < base) {
            c = s.log[pos % s.W];
            valid = c >= 0 && c < s.U && s.stamp[c] == pos;
        }
        const int o = block_scan(valid, ws, &tot);
        if (valid) s.tmp[cnt + o] = c;
        cnt += tot;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < cnt; i += kT) {
        const int c = s.tmp[i];
        s.log[i] = c;
        s.stamp[c] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        s.ctl[kHead] = 0;
        s.ctl[kBase] = cnt;
        s.ctl[kCompact] = 0;
    }
}

__global__ void location_kernel(View s, int64_t f, long long *out) {
    out[0] = s.stamp[f];
    out[1] = s.dslot[f];
    out[2] = s.hslot[f];
}

}  // namespace

struct Policy {
    View v{};
    int device = 0;
    long long *scratch = nullptr;  // location_kernel output
};

namespace {
template <typename T>
bool dalloc(T **p, int64_t n) {
    return cudaMalloc(reinterpret_cast<void **>(p), (size_t)(n > 0 ? n : 1) * sizeof(T)) == cudaSuccess;
}
}  // namespace

int create(Policy **out, int64_t U, int64_t C, int64_t resident0, int64_t dev_slots, int64_t host_slots,
           int64_t host_cap, int64_t max_n) {
    if (!out || U <= 0 || C <= 0 || max_n <= 0 || max_n >= C || U > INT32_MAX) return KVX_EINVAL;
    Policy *p = new (std::nothrow) Policy;
    if (!p) return KVX_ENOSPC;
    View &v = p->v;
    v.U = U;
    v.C = C;
    v.max_n = max_n;
    v.dev_slots = dev_slots;
    v.W = 4 * C + 2 * max_n;
    bool ok = dalloc(&v.stamp, U) && dalloc(&v.ctl, kCtlN) && dalloc(&v.freed_at, dev_slots) && dalloc(&v.dslot, U) && dalloc(&v.hslot, U) &&
              dalloc(&v.first, U) && dalloc(&v.evict_ev, U) && dalloc(&v.log, v.W) && dalloc(&v.tmp, C) &&
              dalloc(&v.dev_free, dev_slots) && dalloc(&v.host_free, host_slots) && dalloc(&v.m0flag, max_n) &&
              dalloc(&v.m0list, max_n) && dalloc(&v.ev_time, max_n) && dalloc(&v.ev_victim, max_n) &&
              dalloc(&v.ev_of_time, max_n) && dalloc(&v.heap, max_n) && dalloc(&v.h2d_dev, 2 * max_n) && dalloc(&v.h2d_host, 2 * max_n) &&
              dalloc(&v.d2h_dev, 2 * max_n) && dalloc(&v.d2h_host, 2 * max_n) && dalloc(&v.counts, 2 * cCountsN) &&
              dalloc(&p->scratch, 4);
    if (!ok) {
        cudaGetLastError();
        destroy(p);
        return KVX_ENOSPC;
    }
    cudaGetDevice(&p->device);
    init_kernel<<<592, 256>>>(v, resident0, host_cap, dev_slots, host_slots);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        destroy(p);
        return KVX_ECUDA;
    }
    *out = p;
    return KVX_OK;
}

void destroy(Policy *p) {
    if (!p) return;
    View &v = p->v;
    void *ptrs[] = {v.stamp, v.ctl, v.freed_at, v.dslot, v.hslot, v.first, v.evict_ev, v.log, v.tmp, v.dev_free, v.host_free,
                    v.m0flag, v.m0list, v.ev_time, v.ev_victim, v.ev_of_time, v.heap, v.h2d_dev, v.h2d_host, v.d2h_dev,
                    v.d2h_host, v.counts, p->scratch};
    for (void *q : ptrs)
        if (q) cudaFree(q);
    delete p;
}

// The copy lists and counts are double-buffered by step parity: a step's
// migrations may still read its lists while the next step is planned.
View at_parity(const View &v0, int parity) {
    View v = v0;
    const int64_t o = parity ? v0.max_n : 0;
    v.h2d_dev += o;
    v.h2d_host += o;
    v.d2h_dev += o;
    v.d2h_host += o;
    v.counts += parity ? cCountsN : 0;
    return v;
}

int step(Policy *p, int parity, int64_t step_no, int64_t min_freed, const int32_t *frames, int64_t n,
         int32_t *dev_slot, uint8_t *hit, int32_t *evicted, cudaStream_t st) {
    if (!p || n < 0 || n > p->v.max_n || (n > 0 && (!frames || !dev_slot))) return KVX_EINVAL;
    const View v = at_parity(p->v, parity & 1);
    if (cudaMemsetAsync(v.counts, 0, cCountsN * sizeof(int32_t), st) != cudaSuccess) return KVX_ECUDA;
    const int ni = (int)n;
    const unsigned grid = (unsigned)std::min<int64_t>(std::max<int64_t>((n + 255) / 256, 1), 148 * 8);
    if (n > 0) {
        touch_kernel<<<grid, 256, 0, st>>>(v, frames, ni);
        classify_kernel<<<grid, 256, 0, st>>>(v, frames, ni);
        scan_kernel<<<1, kT, 0, st>>>(v, ni, (long long)min_freed);
        merge_kernel<<<1, kT, 0, st>>>(v, ni);
        apply_kernel<<<1, kT, 0, st>>>(v, frames);
        finish_kernel<<<grid, 256, 0, st>>>(v, frames, ni, dev_slot, hit, evicted);
        commit_kernel<<<grid, 256, 0, st>>>(v, frames, ni, (long long)step_no);
        compact_kernel<<<1, kT, 0, st>>>(v);
    }
    return kvx::launch_status();  // an empty step: zero counts, no copies
}

void lists(Policy *p, int parity, const int32_t **h2d_dev, const int32_t **h2d_host, const int32_t **d2h_dev,
           const int32_t **d2h_host, const int32_t **counts) {
    const View v = at_parity(p->v, parity & 1);
    *h2d_dev = v.h2d_dev;
    *h2d_host = v.h2d_host;
    *d2h_dev = v.d2h_dev;
    *d2h_host = v.d2h_host;
    *counts = v.counts;  // [0] loads, [1] write-backs
}

namespace {
int read_ctl(Policy *p, long long (&c)[kCtlN], cudaStream_t st) {
    if (cudaMemcpyAsync(c, p->v.ctl, sizeof(c), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return KVX_ECUDA;
    return KVX_OK;
}
}  // namespace

int totals(Policy *p, kvx_tier_stats *stats, cudaStream_t st) {
    long long c[kCtlN];
    const int rc = read_ctl(p, c, st);
    if (rc != KVX_OK) return rc;
    *stats = kvx_tier_stats{};
    stats->accesses = c[kAccesses];
    stats->hits = c[kHits];
    stats->misses = c[kMisses];
    stats->evictions = c[kEvictions];
    stats->reloads = c[kReloads];
    stats->frames_h2d = c[kH2d];
    stats->frames_d2h = c[kD2h];
    return KVX_OK;
}

int location(Policy *p, int64_t frame, int32_t *tier, int64_t *slot, cudaStream_t st) {
    if (frame < 0 || frame >= p->v.U) return KVX_EINVAL;
    location_kernel<<<1, 1, 0, st>>>(p->v, frame, p->scratch);
    long long r[3];
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpyAsync(r, p->scratch, sizeof(r), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return KVX_ECUDA;
    const bool on_dev = r[0] >= 0;
    if (tier) *tier = on_dev ? 0 : 1;
    if (slot) *slot = on_dev ? r[1] : r[2];
    return KVX_OK;
}

int error(Policy *p, int32_t *err, bool clear, cudaStream_t st) {
    long long c[kCtlN];
    int rc = read_ctl(p, c, st);
    if (rc != KVX_OK) return rc;
    *err = (int32_t)c[kErr];
    if (clear && c[kErr] && (cudaMemsetAsync(p->v.ctl + kErr, 0, sizeof(long long), st) != cudaSuccess ||
                             cudaStreamSynchronize(st) != cudaSuccess))
        return KVX_ECUDA;
    return KVX_OK;
}

}  // namespace kvx_tier_dev
