// tier.cpp -- kvx_tier: device frame pool + pinned host arena under the
// reference's LRU policy (include/kvx_tier.h).
//
// Policy (cache/kv_cache.cpp:86-148, KVManager): one recency list over the
// resident frames.  A hit moves the frame to the front; a miss first evicts
// the back when `capacity` frames are resident, then inserts at the front.
// The list is intrusive (prev/next arrays indexed by frame id), so a step of
// n accesses costs O(n) however large the universe is.
//
// Slots.  Residency (which frames) is the policy's; placement (which slot)
// is ours and never changes a decision:
//   * a load takes a device slot freed in an EARLIER step (or a spare one),
//     so this step's loads never wait for this step's write-backs;
//   * a victim's device slot becomes free for the next step;
//   * a victim accessed again later in the same step keeps its slot and
//     bytes: its write-back is cancelled, the policy still counts the
//     eviction and the miss;
//   * host slots alike: a write-back takes a host slot freed earlier, a
//     load frees its host slot for the next step.
//
// Copies.  Per step one gather/scatter launch per direction
// (kvx_migrate_frames) on two streams, so loads (H2D) and write-backs (D2H)
// use both directions of the host link at once.  The only writers are the
// copies; ordering (step s):
//   D2H_s waits H2D_{s-1}: it may write host slots H2D_{s-1} read;
//   H2D_s waits D2H_{s-1}: it may write device slots D2H_{s-1} read, and
//         it may read host slots D2H_{s-1} wrote;
//   H2D_s waits the reads marked for step s-L-2 (L = lookahead, the steps
//         that may be planned ahead of the reads): a device slot it writes
//         was freed by a victim of step s-L-1 or earlier (free device slots
//         are a FIFO, and a slot freed at step j is taken no earlier than
//         step j+L+1), and that victim was last read before the step that
//         evicted it (a step is shorter than the capacity), so at step s-L-2
//         or earlier; reads are marked in step order.
// Completion and read events are rings of L+2 steps; planning step s needs
// the reads of step s-L-2 marked (L = 0: the previous step's plan is all
// that is needed, as a step's reads are marked before the next plan).
// Pinned list staging is double-buffered by step parity; before reusing a
// parity the host waits for the copies of step s-2.
//
// Disk tier (host_frames > 0): RAM is a FIFO of arrivals (ram_prev/next).
// A write-back that finds RAM full first spills the oldest RAM frame to
// the spill file (after waiting for the copy that wrote its slot if it was
// one of the last two steps'), which frees its slot at once.  A miss on a
// disk frame is read into a host slot (after waiting for a load of the last
// two steps that read the slot, if any) and then loaded like a RAM frame.
// The step's file writes and then reads run on 8 host threads before its
// copies are issued.
//
// Device policy (device_policy = 1): the same decisions, with the recency
// order, the free slots and the copy lists held and updated by kernels
// (csrc/kvx_tier_dev.cu) on the store's plan stream s_pol.  A step's copy
// launches read their lists and counts from device memory (lists double-
// buffered by parity, as the staging above); the copies wait for the plan's
// event and are otherwise ordered exactly as above.  Nothing per step runs
// on the host but the launches.
#include "kvx_tier.h"

#include <cuda_runtime.h>

#include "../csrc/kvx_tier_policy.h"
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

extern "C" int kvx_migrate_frames(void *dev_base, int32_t dev_capacity, void *host_base,
                                  int32_t host_capacity, const int32_t *dev_frames,
                                  const int32_t *host_frames, int32_t num_frames, size_t frame_bytes,
                                  int32_t direction, int32_t ctas, int32_t *error_flag, void *stream);

namespace {

struct Copy {
    int32_t dev, host, frame;
    bool cancelled;
};

// FIFO of free slots with O(1) push/pop (ring over a fixed array).
struct SlotQueue {
    std::vector<int32_t> ring;
    size_t head = 0, count = 0;
    void init(size_t cap) { ring.assign(cap ? cap : 1, -1); head = count = 0; }
    bool empty() const { return count == 0; }
    void push(int32_t s) { ring[(head + count++) % ring.size()] = s; }
    void push_front(int32_t s) {
        head = (head + ring.size() - 1) % ring.size();
        ring[head] = s;
        ++count;
    }
    int32_t pop() {
        const int32_t s = ring[head];
        head = (head + 1) % ring.size();
        --count;
        return s;
    }
};

}  // namespace

struct kvx_tier {
    kvx_tier_config cfg{};
    int64_t dev_slots = 0, host_slots = 0;
    bool bookkeeping = false;
    std::mutex mu;

    // per frame
    std::vector<int32_t> dslot, hslot, prev, next, victim_idx;
    std::vector<int64_t> last_step;
    int32_t head = -1, tail = -1;
    int64_t resident = 0;
    SlotQueue dev_free, host_free;
    std::vector<int32_t> freed_dev, freed_host;
    std::vector<int64_t> reclaimed;  // per device slot: step in which a victim kept it
    std::vector<Copy> d2h;
    std::vector<int32_t> h2d_dev, h2d_host;
    int64_t step = 0;
    kvx_tier_stats totals{};

    // disk tier
    bool disk = false;
    int fd = -1;
    int64_t host_cap = 0, in_ram = 0;
    std::vector<int32_t> ram_prev, ram_next;  // RAM arrival order (head newest)
    int32_t ram_head = -1, ram_tail = -1;
    std::vector<int64_t> slot_step;           // per host slot: step whose write-back filled it
    std::vector<int64_t> slot_load_step;      // per host slot: step whose load read it last
    bool h2d_prev_synced = false;             // this step waited for the previous step's loads
    struct DiskIo {
        int32_t slot, frame;
    };
    std::vector<DiskIo> spills, reads;        // this step's file writes, then reads

    // device side
    uint8_t *dev_base = nullptr, *host_base = nullptr;
    cudaStream_t s_h2d = nullptr, s_d2h = nullptr;
    int ring = 2;                                    // lookahead + 2
    std::vector<cudaEvent_t> ev_h2d, ev_read;        // per step s at [s % ring]
    std::vector<int64_t> h2d_step, read_step;        // the step each holds (-1: none)
    cudaEvent_t ev_d2h[2] = {};                      // per step parity
    int64_t marked = 0;                              // steps whose reads are marked
    std::vector<int64_t> freed_at;                   // per device slot: step that freed it
    int32_t *stage[2] = {};   // pinned: [4][spare] (h2d dev, h2d host, d2h dev, d2h host)
    int32_t *lists[2] = {};   // device copies of the same
    int32_t *err = nullptr;   // device error flag

    // device policy (config device_policy): the bookkeeping above lives on
    // the device instead, in `pol`, and runs on s_pol
    kvx_tier_dev::Policy *pol = nullptr;
    cudaStream_t s_pol = nullptr;
    cudaEvent_t ev_pol = nullptr, ev_caller = nullptr;
    int32_t *d_frames = nullptr, *d_slot = nullptr, *d_evict = nullptr;  // host-array steps
    uint8_t *d_hit = nullptr;
};

namespace {

void unlink(kvx_tier *t, int32_t f) {
    const int32_t p = t->prev[f], n = t->next[f];
    if (p >= 0) t->next[p] = n; else t->head = n;
    if (n >= 0) t->prev[n] = p; else t->tail = p;
    t->prev[f] = t->next[f] = -1;
}

void push_front(kvx_tier *t, int32_t f) {
    t->prev[f] = -1;
    t->next[f] = t->head;
    if (t->head >= 0) t->prev[t->head] = f;
    t->head = f;
    if (t->tail < 0) t->tail = f;
}

void ram_unlink(kvx_tier *t, int32_t f) {
    const int32_t p = t->ram_prev[f], n = t->ram_next[f];
    if (p >= 0) t->ram_next[p] = n; else t->ram_head = n;
    if (n >= 0) t->ram_prev[n] = p; else t->ram_tail = p;
    t->ram_prev[f] = t->ram_next[f] = -1;
    --t->in_ram;
}

void ram_push(kvx_tier *t, int32_t f) {
    t->ram_prev[f] = -1;
    t->ram_next[f] = t->ram_head;
    if (t->ram_head >= 0) t->ram_prev[t->ram_head] = f;
    t->ram_head = f;
    if (t->ram_tail < 0) t->ram_tail = f;
    ++t->in_ram;
}

bool file_io(int fd, void *buf, size_t n, off_t off, bool write) {
    uint8_t *b = static_cast<uint8_t *>(buf);
    while (n) {
        const ssize_t r = write ? pwrite(fd, b, n, off) : pread(fd, b, n, off);
        if (r <= 0) return false;
        b += r;
        n -= (size_t)r;
        off += r;
    }
    return true;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? KVX_OK : KVX_ECUDA; }

// Wait until the write-back that filled host slot hs (if recent) is done.
int wait_slot_written(kvx_tier *t, int32_t hs) {
    const int64_t w = t->slot_step[hs];
    if (t->bookkeeping || w < 0 || w < t->step - 2) return KVX_OK;
    if (w == t->step) return KVX_ENOSPC;  // written by this very step: RAM tier too small
    return cuda_status(cudaEventSynchronize(t->ev_d2h[w & 1]));
}

// Move the oldest RAM frame to the spill file; its host slot is free again.
int spill_oldest(kvx_tier *t, kvx_tier_stats &st) {
    const int32_t f = t->ram_tail;
    if (f < 0) return KVX_ENOSPC;
    const int32_t hs = t->hslot[f];
    const int rc = wait_slot_written(t, hs);
    if (rc != KVX_OK) return rc;
    t->spills.push_back({hs, f});  // written before any later use of the slot (run_disk_io)
    ram_unlink(t, f);
    t->hslot[f] = -1;
    t->slot_step[hs] = -1;
    t->host_free.push_front(hs);
    ++st.frames_disk_write;
    return KVX_OK;
}

// The step's file traffic, 8 host threads per phase: every spill write, then
// every read (a read may land in a slot a spill of this step vacated).
int run_disk_io(kvx_tier *t) {
    if (t->bookkeeping) {
        t->spills.clear();
        t->reads.clear();
        return KVX_OK;
    }
    std::atomic<bool> ok{true};
    auto phase = [&](const std::vector<kvx_tier::DiskIo> &ios, bool write) {
        if (ios.empty()) return;
        const size_t nt = std::min<size_t>(8, (ios.size() + 7) / 8);
        std::vector<std::thread> th;
        for (size_t w = 0; w < nt; ++w)
            th.emplace_back([&, w] {
                for (size_t i = w; i < ios.size(); i += nt)
                    if (!file_io(t->fd, t->host_base + (size_t)ios[i].slot * t->cfg.frame_bytes, t->cfg.frame_bytes,
                                 (off_t)ios[i].frame * (off_t)t->cfg.frame_bytes, write))
                        ok = false;
            });
        for (auto &x : th) x.join();
    };
    phase(t->spills, true);
    phase(t->reads, false);
    t->spills.clear();
    t->reads.clear();
    return ok ? KVX_OK : KVX_ECUDA;
}

// A free host slot, spilling the oldest RAM frame when there is none.
int take_host_slot(kvx_tier *t, kvx_tier_stats &st, int32_t &hs) {
    if (t->host_free.empty()) {
        if (!t->disk) return KVX_ENOSPC;
        const int rc = spill_oldest(t, st);
        if (rc != KVX_OK) return rc;
    }
    hs = t->host_free.pop();
    return KVX_OK;
}

void release(kvx_tier *t) {
    if (t->pol) {
        if (t->s_pol) cudaStreamSynchronize(t->s_pol);
        kvx_tier_dev::destroy(t->pol);
        t->pol = nullptr;
        if (t->s_pol) cudaStreamDestroy(t->s_pol);
        if (t->ev_pol) cudaEventDestroy(t->ev_pol);
        if (t->ev_caller) cudaEventDestroy(t->ev_caller);
        for (void *q : {(void *)t->d_frames, (void *)t->d_slot, (void *)t->d_evict, (void *)t->d_hit})
            if (q) cudaFree(q);
    }
    if (!t->bookkeeping) {
        if (t->s_h2d) cudaStreamSynchronize(t->s_h2d);
        if (t->s_d2h) cudaStreamSynchronize(t->s_d2h);
        for (cudaEvent_t e : t->ev_h2d)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : t->ev_read)
            if (e) cudaEventDestroy(e);
        for (int p = 0; p < 2; ++p) {
            if (t->ev_d2h[p]) cudaEventDestroy(t->ev_d2h[p]);
            if (t->stage[p]) cudaFreeHost(t->stage[p]);
            if (t->lists[p]) cudaFree(t->lists[p]);
        }
        if (t->s_h2d) cudaStreamDestroy(t->s_h2d);
        if (t->s_d2h) cudaStreamDestroy(t->s_d2h);
        if (t->dev_base) cudaFree(t->dev_base);
        if (t->host_base) cudaFreeHost(t->host_base);
        if (t->err) cudaFree(t->err);
    }
    if (t->fd >= 0) close(t->fd);
}

int setup_device(kvx_tier *t) {
    if (cudaSetDevice(t->cfg.device) != cudaSuccess) return KVX_ENODEV;
    const size_t fb = t->cfg.frame_bytes;
    if (cudaMalloc(&t->dev_base, (size_t)t->dev_slots * fb) != cudaSuccess) {
        cudaGetLastError();
        return KVX_ENOSPC;
    }
    if (cudaHostAlloc(&t->host_base, (size_t)t->host_slots * fb, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        cudaGetLastError();
        t->host_base = nullptr;
        return KVX_ENOSPC;
    }
    if (cudaStreamCreateWithFlags(&t->s_h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&t->s_d2h, cudaStreamNonBlocking) != cudaSuccess)
        return KVX_ECUDA;
    const size_t lb = 4 * (size_t)(t->cfg.spare ? t->cfg.spare : 1) * sizeof(int32_t);
    for (int r = 0; r < t->ring; ++r)
        if (cudaEventCreateWithFlags(&t->ev_h2d[r], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&t->ev_read[r], cudaEventDisableTiming) != cudaSuccess)
            return KVX_ECUDA;
    for (int p = 0; p < 2; ++p) {
        if (cudaEventCreateWithFlags(&t->ev_d2h[p], cudaEventDisableTiming) != cudaSuccess) return KVX_ECUDA;
        if (cudaHostAlloc(reinterpret_cast<void **>(&t->stage[p]), lb, cudaHostAllocPortable) != cudaSuccess ||
            cudaMalloc(&t->lists[p], lb) != cudaSuccess)
            return KVX_ENOSPC;
    }
    if (cudaMalloc(&t->err, sizeof(int32_t)) != cudaSuccess) return KVX_ENOSPC;
    return cuda_status(cudaMemset(t->err, 0, sizeof(int32_t)));
}

// Event helpers, by step number: completion of step s's loads, and the
// reads marked for step j.
bool loads_issued(const kvx_tier *t, int64_t s) { return s >= 0 && t->h2d_step[s % t->ring] == s; }

int wait_loads(kvx_tier *t, cudaStream_t st, int64_t s) {
    if (!loads_issued(t, s)) return KVX_OK;
    return cuda_status(cudaStreamWaitEvent(st, t->ev_h2d[s % t->ring], 0));
}

// The newest mark of j's ring slot is j's own or an older step's (a newer
// one would be at least `ring` steps later, which the plan contract rules
// out), so waiting for it covers every read marked up to j in that slot.
int wait_reads(kvx_tier *t, cudaStream_t st, int64_t j) {
    if (j < 0 || t->read_step[j % t->ring] < 0) return KVX_OK;
    return cuda_status(cudaStreamWaitEvent(st, t->ev_read[j % t->ring], 0));
}

int record_loads(kvx_tier *t, int64_t s) {
    if (cudaEventRecord(t->ev_h2d[s % t->ring], t->s_h2d) != cudaSuccess) return KVX_ECUDA;
    t->h2d_step[s % t->ring] = s;
    return KVX_OK;
}

// Planning step s needs the reads of step s-L-2 marked (lookahead L > 0).
int plan_allowed(const kvx_tier *t) {
    const int64_t L = t->cfg.lookahead;
    return (L > 0 && t->marked < t->step - L - 1) ? KVX_EBUSY : KVX_OK;
}

// Enqueue the copies of step s, just planned.
int issue(kvx_tier *t, int64_t s) {
    const int parity = (int)(s & 1);
    const int64_t sp = t->cfg.spare;
    int32_t *st = t->stage[parity], *dl = t->lists[parity];
    if (loads_issued(t, s - 2)) {  // the copies of step s-2 read this staging
        if (cudaEventSynchronize(t->ev_h2d[(s - 2) % t->ring]) != cudaSuccess ||
            cudaEventSynchronize(t->ev_d2h[parity]) != cudaSuccess)
            return KVX_ECUDA;
    }
    int32_t nd = 0;
    for (const Copy &c : t->d2h)
        if (!c.cancelled) {
            st[2 * sp + nd] = c.dev;
            st[3 * sp + nd] = c.host;
            ++nd;
        }
    const int32_t nh = (int32_t)t->h2d_dev.size();
    if (nh) {
        std::memcpy(st, t->h2d_dev.data(), nh * sizeof(int32_t));
        std::memcpy(st + sp, t->h2d_host.data(), nh * sizeof(int32_t));
    }
    const int load_ctas = t->cfg.load_ctas > 0 ? t->cfg.load_ctas : 16;
    const int store_ctas = t->cfg.store_ctas > 0 ? t->cfg.store_ctas : 4;
    const int32_t dcap = (int32_t)t->dev_slots, hcap = (int32_t)t->host_slots;
    // write-backs
    int rc = wait_loads(t, t->s_d2h, s - 1);
    if (rc != KVX_OK) return rc;
    if (nd) {
        if (cudaMemcpyAsync(dl + 2 * sp, st + 2 * sp, nd * sizeof(int32_t), cudaMemcpyHostToDevice, t->s_d2h) !=
                cudaSuccess ||
            cudaMemcpyAsync(dl + 3 * sp, st + 3 * sp, nd * sizeof(int32_t), cudaMemcpyHostToDevice, t->s_d2h) !=
                cudaSuccess)
            return KVX_ECUDA;
        rc = kvx_migrate_frames(t->dev_base, dcap, t->host_base, hcap, dl + 2 * sp, dl + 3 * sp, nd,
                                t->cfg.frame_bytes, 0, store_ctas, t->err, t->s_d2h);
        if (rc != KVX_OK) return rc;
    }
    if (cudaEventRecord(t->ev_d2h[parity], t->s_d2h) != cudaSuccess) return KVX_ECUDA;
    // loads: after the previous write-backs and the reads of step s-L-2
    if (loads_issued(t, s - 1) && cudaStreamWaitEvent(t->s_h2d, t->ev_d2h[parity ^ 1], 0) != cudaSuccess)
        return KVX_ECUDA;
    rc = wait_reads(t, t->s_h2d, s - t->cfg.lookahead - 2);
    if (rc != KVX_OK) return rc;
    if (nh) {
        if (cudaMemcpyAsync(dl, st, nh * sizeof(int32_t), cudaMemcpyHostToDevice, t->s_h2d) != cudaSuccess ||
            cudaMemcpyAsync(dl + sp, st + sp, nh * sizeof(int32_t), cudaMemcpyHostToDevice, t->s_h2d) !=
                cudaSuccess)
            return KVX_ECUDA;
        rc = kvx_migrate_frames(t->dev_base, dcap, t->host_base, hcap, dl, dl + sp, nh, t->cfg.frame_bytes, 1,
                                load_ctas, t->err, t->s_h2d);
        if (rc != KVX_OK) return rc;
    }
    return record_loads(t, s);
}

// The copies of step s planned on the device: the lists and their counts
// are device arrays (kvx_tier_dev::lists), the launches read the counts
// there; ordering as in issue().
int issue_dev(kvx_tier *t, int64_t s) {
    const int parity = (int)(s & 1);
    const int32_t *hd, *hh, *dd, *dh, *cnt;
    kvx_tier_dev::lists(t->pol, parity, &hd, &hh, &dd, &dh, &cnt);
    const int load_ctas = t->cfg.load_ctas > 0 ? t->cfg.load_ctas : 16;
    const int store_ctas = t->cfg.store_ctas > 0 ? t->cfg.store_ctas : 4;
    const int32_t dcap = (int32_t)t->dev_slots, hcap = (int32_t)t->host_slots, mx = (int32_t)t->cfg.max_step;
    // write-backs: after the plan, and after the previous step's loads (host slots)
    if (cudaStreamWaitEvent(t->s_d2h, t->ev_pol, 0) != cudaSuccess) return KVX_ECUDA;
    int rc = wait_loads(t, t->s_d2h, s - 1);
    if (rc != KVX_OK) return rc;
    rc = kvx_tier_dev::migrate_counted(t->dev_base, dcap, t->host_base, hcap, dd, dh, cnt + 1, mx,
                                       t->cfg.frame_bytes, 0, store_ctas, t->err, t->s_d2h);
    if (rc != KVX_OK) return rc;
    if (cudaEventRecord(t->ev_d2h[parity], t->s_d2h) != cudaSuccess) return KVX_ECUDA;
    // loads: after the plan, the previous write-backs and the reads of step s-L-2
    if (cudaStreamWaitEvent(t->s_h2d, t->ev_pol, 0) != cudaSuccess) return KVX_ECUDA;
    if (loads_issued(t, s - 1) && cudaStreamWaitEvent(t->s_h2d, t->ev_d2h[parity ^ 1], 0) != cudaSuccess)
        return KVX_ECUDA;
    rc = wait_reads(t, t->s_h2d, s - t->cfg.lookahead - 2);
    if (rc != KVX_OK) return rc;
    rc = kvx_tier_dev::migrate_counted(t->dev_base, dcap, t->host_base, hcap, hd, hh, cnt, mx, t->cfg.frame_bytes, 1,
                                       load_ctas, t->err, t->s_h2d);
    if (rc != KVX_OK) return rc;
    return record_loads(t, s);
}

// One step planned on the device (policy kernels on s_pol), then its
// copies.  With `wait_caller` the plan waits for the work queued on `caller`
// (which produced `frames`; a null handle is the legacy default stream);
// without, s_pol itself produced them.
int step_device_core(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot, int32_t *evicted,
                     uint8_t *hit, bool wait_caller, cudaStream_t caller) {
    const int64_t s = t->step;
    const int parity = (int)(s & 1);
    if (wait_caller && (cudaEventRecord(t->ev_caller, caller) != cudaSuccess ||
                        cudaStreamWaitEvent(t->s_pol, t->ev_caller, 0) != cudaSuccess))
        return KVX_ECUDA;
    // this parity's copy lists were read by the copies of step s-2
    if (loads_issued(t, s - 2) &&
        (cudaStreamWaitEvent(t->s_pol, t->ev_h2d[(s - 2) % t->ring], 0) != cudaSuccess ||
         cudaStreamWaitEvent(t->s_pol, t->ev_d2h[parity], 0) != cudaSuccess))
        return KVX_ECUDA;
    int rc = kvx_tier_dev::step(t->pol, parity, s, s - t->cfg.lookahead - 1, frames, n, dev_slot, hit, evicted,
                                t->s_pol);
    if (rc == KVX_OK && cudaEventRecord(t->ev_pol, t->s_pol) != cudaSuccess) rc = KVX_ECUDA;
    if (rc == KVX_OK) rc = issue_dev(t, s);
    ++t->step;
    return rc;
}

int setup_policy(kvx_tier *t, int64_t resident0) {
    const int64_t mx = t->cfg.max_step;
    int rc = kvx_tier_dev::create(&t->pol, t->cfg.universe, t->cfg.capacity, resident0, t->dev_slots, t->host_slots,
                                  t->host_cap, mx);
    if (rc != KVX_OK) return rc;
    if (cudaStreamCreateWithFlags(&t->s_pol, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->ev_pol, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->ev_caller, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&t->d_frames, mx * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&t->d_slot, mx * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&t->d_evict, mx * sizeof(int32_t)) != cudaSuccess || cudaMalloc(&t->d_hit, mx) != cudaSuccess)
        return KVX_ENOSPC;
    return KVX_OK;
}

}  // namespace

extern "C" KVX_API int kvx_tier_create(const kvx_tier_config *cfg, kvx_tier **out) {
    if (!cfg || !out) return KVX_EINVAL;
    *out = nullptr;
    if (cfg->frame_bytes == 0 || cfg->frame_bytes % 16 || cfg->universe <= 0 || cfg->capacity <= 0 ||
        cfg->spare < 0 || cfg->universe > INT32_MAX)
        return KVX_EINVAL;
    kvx_tier *t = new (std::nothrow) kvx_tier;
    if (!t) return KVX_ENOSPC;
    t->cfg = *cfg;
    t->bookkeeping = cfg->device < 0;
    if (cfg->lookahead < 0 || cfg->lookahead > 62) {
        delete t;
        return KVX_EINVAL;
    }
    t->ring = (int)cfg->lookahead + 2;
    t->ev_h2d.assign(t->ring, nullptr);
    t->ev_read.assign(t->ring, nullptr);
    t->h2d_step.assign(t->ring, -1);
    t->read_step.assign(t->ring, -1);
    const int64_t U = cfg->universe, C = cfg->capacity, S = cfg->spare;
    const int64_t resident0 = U < C ? U : C;
    t->disk = cfg->host_frames > 0 && cfg->host_frames < U - resident0;
    if (t->disk && (!cfg->spill_path || cfg->host_frames < 3 * S)) {
        delete t;
        return KVX_EINVAL;  // the RAM tier must outlast three steps' write-backs
    }
    t->host_cap = t->disk ? cfg->host_frames : U - resident0;
    t->dev_slots = C + S;
    t->host_slots = t->host_cap + S;
    if (t->dev_slots > INT32_MAX || t->host_slots > INT32_MAX) {
        delete t;
        return KVX_EINVAL;
    }
    if (cfg->device_policy) {  // bookkeeping on the device: RAM tier only, a bounded step
        if (cfg->device < 0 || cfg->host_frames > 0 || cfg->max_step <= 0 || cfg->max_step >= C || U <= C) {
            delete t;
            return KVX_EINVAL;
        }
        t->resident = resident0;
        int rc = setup_device(t);
        if (rc == KVX_OK) rc = setup_policy(t, resident0);
        if (rc != KVX_OK) {
            release(t);
            delete t;
            return rc;
        }
        *out = t;
        return KVX_OK;
    }
    try {
        t->dslot.assign(U, -1);
        t->hslot.assign(U, -1);
        t->prev.assign(U, -1);
        t->next.assign(U, -1);
        t->victim_idx.assign(U, -1);
        t->last_step.assign(U, -1);
        t->reclaimed.assign(t->dev_slots, -1);
        t->freed_at.assign(t->dev_slots, INT64_MIN / 2);  // never used: free for any step
        t->slot_step.assign(t->host_slots, -1);
        t->slot_load_step.assign(t->host_slots, -1);
        if (t->disk) {
            t->ram_prev.assign(U, -1);
            t->ram_next.assign(U, -1);
        }
        t->dev_free.init(t->dev_slots);
        t->host_free.init(t->host_slots);
    } catch (const std::bad_alloc &) {
        delete t;
        return KVX_ENOSPC;
    }
    for (int64_t f = 0; f < resident0; ++f) {  // loaded in id order: frame 0 ends at the back
        t->dslot[f] = (int32_t)f;
        push_front(t, (int32_t)f);
    }
    t->resident = resident0;
    for (int64_t f = resident0; f < resident0 + t->host_cap; ++f) {  // the rest start on disk
        t->hslot[f] = (int32_t)(f - resident0);
        if (t->disk) ram_push(t, (int32_t)f);
    }
    for (int64_t s = resident0; s < t->dev_slots; ++s) t->dev_free.push((int32_t)s);
    for (int64_t s = t->host_cap; s < t->host_slots; ++s) t->host_free.push((int32_t)s);
    if (t->disk && !t->bookkeeping) {
        t->fd = open(cfg->spill_path, O_RDWR | O_CREAT | O_TRUNC, 0600);
        if (t->fd < 0 || ftruncate(t->fd, (off_t)U * (off_t)cfg->frame_bytes) != 0) {
            release(t);
            delete t;
            return KVX_EINVAL;
        }
    }
    if (!t->bookkeeping) {
        const int rc = setup_device(t);
        if (rc != KVX_OK) {
            release(t);
            delete t;
            return rc;
        }
    }
    *out = t;
    return KVX_OK;
}

extern "C" KVX_API void kvx_tier_destroy(kvx_tier *t) {
    if (!t) return;
    release(t);
    delete t;
}

extern "C" KVX_API int kvx_tier_device_arena(kvx_tier *t, void **base, int64_t *slots) {
    if (!t) return KVX_EINVAL;
    if (base) *base = t->dev_base;
    if (slots) *slots = t->dev_slots;
    return KVX_OK;
}

extern "C" KVX_API int kvx_tier_host_arena(kvx_tier *t, void **base, int64_t *slots) {
    if (!t) return KVX_EINVAL;
    if (base) *base = t->host_base;
    if (slots) *slots = t->host_slots;
    return KVX_OK;
}

extern "C" KVX_API int kvx_tier_location(kvx_tier *t, int64_t frame, int32_t *tier, int64_t *slot) {
    if (!t || frame < 0 || frame >= t->cfg.universe) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    if (t->pol) {
        return kvx_tier_dev::location(t->pol, frame, tier, slot, t->s_pol);
    }
    const bool on_dev = t->dslot[frame] >= 0, in_ram = !on_dev && t->hslot[frame] >= 0;
    if (tier) *tier = on_dev ? 0 : in_ram ? 1 : 2;
    if (slot) *slot = on_dev ? t->dslot[frame] : in_ram ? t->hslot[frame] : frame;
    return KVX_OK;
}

extern "C" KVX_API int kvx_tier_step_device(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot,
                                            int32_t *evicted, uint8_t *hit, void *stream) {
    if (!t) return KVX_EINVAL;
    if (!t->pol) return KVX_EUNSUPPORTED;
    if (n < 0 || n > t->cfg.max_step || (n > 0 && (!frames || !dev_slot))) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    const int rc = plan_allowed(t);
    if (rc != KVX_OK) return rc;
    return step_device_core(t, frames, n, dev_slot, evicted, hit, true, static_cast<cudaStream_t>(stream));
}

namespace {
// kvx_tier_step (host arrays) on a store whose bookkeeping is on the device:
// through the device and back, waiting; per-step stats from the totals.
int step_host_via_device(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot, int32_t *evicted,
                         uint8_t *hit, kvx_tier_stats *stats) {
    if (n > t->cfg.max_step) return KVX_EINVAL;
    kvx_tier_stats before{}, after{};
    int32_t err = 0;
    int rc = plan_allowed(t);
    if (rc != KVX_OK) return rc;
    rc = kvx_tier_dev::totals(t->pol, &before, t->s_pol);
    if (rc == KVX_OK) rc = kvx_tier_dev::error(t->pol, &err, true, t->s_pol);
    if (rc != KVX_OK) return rc;
    if (n > 0 && cudaMemcpyAsync(t->d_frames, frames, n * sizeof(int32_t), cudaMemcpyHostToDevice, t->s_pol) !=
                     cudaSuccess)
        return KVX_ECUDA;
    rc = step_device_core(t, t->d_frames, n, t->d_slot, evicted ? t->d_evict : nullptr, hit ? t->d_hit : nullptr,
                          false, nullptr);
    if (rc != KVX_OK) return rc;
    if (n > 0 &&
        (cudaMemcpyAsync(dev_slot, t->d_slot, n * sizeof(int32_t), cudaMemcpyDeviceToHost, t->s_pol) != cudaSuccess ||
         (evicted && cudaMemcpyAsync(evicted, t->d_evict, n * sizeof(int32_t), cudaMemcpyDeviceToHost, t->s_pol) !=
                         cudaSuccess) ||
         (hit && cudaMemcpyAsync(hit, t->d_hit, n, cudaMemcpyDeviceToHost, t->s_pol) != cudaSuccess)))
        return KVX_ECUDA;
    if (cudaStreamSynchronize(t->s_pol) != cudaSuccess) return KVX_ECUDA;
    rc = kvx_tier_dev::error(t->pol, &err, true, t->s_pol);
    if (rc != KVX_OK) return rc;
    if (err) return (err & 2) ? KVX_ENOSPC : KVX_EINVAL;  // rejected on the device, nothing changed
    rc = kvx_tier_dev::totals(t->pol, &after, t->s_pol);
    if (rc != KVX_OK) return rc;
    kvx_tier_stats st{};
    st.accesses = after.accesses - before.accesses;
    st.hits = after.hits - before.hits;
    st.misses = after.misses - before.misses;
    st.evictions = after.evictions - before.evictions;
    st.reloads = after.reloads - before.reloads;
    st.frames_h2d = after.frames_h2d - before.frames_h2d;
    st.frames_d2h = after.frames_d2h - before.frames_d2h;
    t->totals = after;
    if (stats) *stats = st;
    return KVX_OK;
}
}  // namespace

extern "C" KVX_API int kvx_tier_step(kvx_tier *t, const int32_t *frames, int64_t n, int32_t *dev_slot,
                                     int32_t *evicted, uint8_t *hit, kvx_tier_stats *stats) {
    if (!t || n < 0 || (n > 0 && (!frames || !dev_slot))) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    if (t->pol) return step_host_via_device(t, frames, n, dev_slot, evicted, hit, stats);
    if (n >= t->cfg.capacity && t->cfg.universe > t->cfg.capacity) return KVX_EINVAL;
    const int rc0 = plan_allowed(t);
    if (rc0 != KVX_OK) return rc0;
    const int64_t s = t->step;
    // pre-pass: ids valid, and the distinct frames to load fit the free slots
    int64_t loads = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t f = frames[i];
        if (f < 0 || f >= t->cfg.universe) return KVX_EINVAL;
        if (t->dslot[f] < 0 && t->victim_idx[f] != -2) {
            t->victim_idx[f] = -2;  // counted
            ++loads;
        }
    }
    for (int64_t i = 0; i < n; ++i)
        if (t->victim_idx[frames[i]] == -2) t->victim_idx[frames[i]] = -1;
    if (loads > t->cfg.spare || (uint64_t)loads > t->dev_free.count ||
        (!t->disk && (uint64_t)loads > t->host_free.count))
        return KVX_ENOSPC;
    if (loads > 0) {  // the loads take the FIFO's first slots: all freed by step s-L-1 or earlier
        const auto &q = t->dev_free;
        if (t->freed_at[q.ring[(q.head + loads - 1) % q.ring.size()]] > s - t->cfg.lookahead - 1) return KVX_ENOSPC;
    }
    t->h2d_prev_synced = false;

    kvx_tier_stats st{};
    st.accesses = n;
    t->d2h.clear();
    t->h2d_dev.clear();
    t->h2d_host.clear();
    t->freed_dev.clear();
    t->freed_host.clear();
    for (int64_t i = 0; i < n; ++i) {
        const int32_t f = frames[i];
        if (evicted) evicted[i] = -1;
        if (t->dslot[f] >= 0) {  // hit
            if (hit) hit[i] = 1;
            ++st.hits;
            if (t->head != f) {
                unlink(t, f);
                push_front(t, f);
            }
        } else {
            if (hit) hit[i] = 0;
            ++st.misses;
            if (t->resident >= t->cfg.capacity) {  // evict the back first
                const int32_t v = t->tail;
                unlink(t, v);
                --t->resident;
                ++st.evictions;
                if (evicted) evicted[i] = v;
                int32_t hs = -1;
                if (t->disk) {  // RAM full: the oldest RAM frame goes to disk first
                    int rc = KVX_OK;
                    while (rc == KVX_OK && t->in_ram >= t->host_cap) rc = spill_oldest(t, st);
                    if (rc == KVX_OK) rc = take_host_slot(t, st, hs);
                    if (rc != KVX_OK) return rc;
                    t->slot_step[hs] = s;
                    ram_push(t, v);
                } else {
                    hs = t->host_free.pop();
                }
                t->victim_idx[v] = (int32_t)t->d2h.size();
                t->d2h.push_back(Copy{t->dslot[v], hs, v, false});
                t->freed_dev.push_back(t->dslot[v]);
                t->hslot[v] = hs;
                t->dslot[v] = -1;
            }
            if (t->victim_idx[f] >= 0) {  // evicted earlier in this step: keep slot and bytes
                Copy &c = t->d2h[t->victim_idx[f]];
                c.cancelled = true;
                ++st.reloads;
                t->dslot[f] = c.dev;
                t->reclaimed[c.dev] = s;
                if (t->disk) {
                    ram_unlink(t, f);
                    t->slot_step[c.host] = -1;
                }
                t->host_free.push_front(c.host);
                t->hslot[f] = -1;
                t->victim_idx[f] = -1;
            } else {
                if (t->disk) {
                    if (t->hslot[f] >= 0) {
                        ram_unlink(t, f);
                    } else {  // on disk: read it into a host slot, then load as from RAM
                        int32_t hs = -1;
                        int rc = take_host_slot(t, st, hs);
                        const int64_t w = t->slot_load_step[hs];
                        if (rc == KVX_OK && !t->bookkeeping && w >= 0 && w >= s - 2 &&
                            !(w == s - 1 && t->h2d_prev_synced)) {
                            // a load of one of the last two steps may still read this slot
                            // (older loads finished: issue() waited for step s-3's copies)
                            if (cudaEventSynchronize(t->ev_h2d[w % t->ring]) != cudaSuccess) rc = KVX_ECUDA;
                            if (w == s - 1) t->h2d_prev_synced = true;
                        }
                        if (rc != KVX_OK) return rc;
                        t->reads.push_back({hs, f});  // read before this step's loads are issued
                        t->hslot[f] = hs;
                        ++st.frames_disk_read;
                    }
                    t->slot_step[t->hslot[f]] = -1;
                }
                const int32_t ds = t->dev_free.pop();
                if (t->disk) t->slot_load_step[t->hslot[f]] = s;
                t->h2d_dev.push_back(ds);
                t->h2d_host.push_back(t->hslot[f]);
                t->freed_host.push_back(t->hslot[f]);
                t->hslot[f] = -1;
                t->dslot[f] = ds;
            }
            push_front(t, f);
            ++t->resident;
        }
        t->last_step[f] = s;
        dev_slot[i] = t->dslot[f];
    }
    for (const Copy &c : t->d2h) {
        t->victim_idx[c.frame] = -1;
        if (!c.cancelled) ++st.frames_d2h;
    }
    st.frames_h2d = (int64_t)t->h2d_dev.size();
    int rc = t->disk ? run_disk_io(t) : KVX_OK;
    if (rc == KVX_OK && !t->bookkeeping) rc = issue(t, s);
    // slots freed by this step serve later ones (device slots: from step s+L+1)
    for (int32_t d : t->freed_dev)
        if (t->reclaimed[d] != s) {
            t->dev_free.push(d);
            t->freed_at[d] = s;
        }
    for (int32_t h : t->freed_host) t->host_free.push(h);
    ++t->step;
    t->totals.accesses += st.accesses;
    t->totals.hits += st.hits;
    t->totals.misses += st.misses;
    t->totals.evictions += st.evictions;
    t->totals.reloads += st.reloads;
    t->totals.frames_h2d += st.frames_h2d;
    t->totals.frames_d2h += st.frames_d2h;
    t->totals.frames_disk_read += st.frames_disk_read;
    t->totals.frames_disk_write += st.frames_disk_write;
    if (stats) *stats = st;
    return rc;
}

extern "C" KVX_API int kvx_tier_plan_stream(kvx_tier *t, void **stream) {
    if (!t || !stream) return KVX_EINVAL;
    if (!t->pol) return KVX_EUNSUPPORTED;
    *stream = t->s_pol;
    return KVX_OK;
}

namespace {
// The step whose reads come next: the last one planned (lookahead 0), or
// the oldest one not yet marked.
int64_t read_cursor(const kvx_tier *t) { return t->cfg.lookahead > 0 ? t->marked : t->step - 1; }
}  // namespace

extern "C" KVX_API int kvx_tier_wait_resident(kvx_tier *t, void *stream) {
    if (!t) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    const int64_t j = read_cursor(t);
    if (t->bookkeeping || j < 0 || j >= t->step) return KVX_OK;
    return wait_loads(t, static_cast<cudaStream_t>(stream), j);
}

extern "C" KVX_API int kvx_tier_mark_read(kvx_tier *t, void *stream) {
    if (!t) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    const int64_t j = read_cursor(t);
    if (j < 0) return KVX_OK;
    if (j >= t->step) return KVX_EINVAL;  // every planned step is marked already
    if (!t->bookkeeping) {
        if (cudaEventRecord(t->ev_read[j % t->ring], static_cast<cudaStream_t>(stream)) != cudaSuccess)
            return KVX_ECUDA;
        t->read_step[j % t->ring] = j;
    }
    t->marked = j + 1;
    return KVX_OK;
}

extern "C" KVX_API int kvx_tier_sync(kvx_tier *t) {
    if (!t) return KVX_EINVAL;
    if (t->bookkeeping) return KVX_OK;
    if (t->pol) {  // the plan's stream, and a step the device rejected
        int32_t perr = 0;
        if (kvx_tier_dev::error(t->pol, &perr, true, t->s_pol) != KVX_OK) return KVX_ECUDA;  // reported once
        if (perr) return (perr & 2) ? KVX_ENOSPC : KVX_EINVAL;
    }
    if (cudaStreamSynchronize(t->s_h2d) != cudaSuccess || cudaStreamSynchronize(t->s_d2h) != cudaSuccess)
        return KVX_ECUDA;
    int32_t e = 0;
    if (cudaMemcpy(&e, t->err, sizeof(e), cudaMemcpyDeviceToHost) != cudaSuccess) return KVX_ECUDA;
    return e ? KVX_EINVAL : KVX_OK;
}

extern "C" KVX_API int kvx_tier_totals(kvx_tier *t, kvx_tier_stats *stats) {
    if (!t || !stats) return KVX_EINVAL;
    std::lock_guard<std::mutex> lk(t->mu);
    if (t->pol) {
        return kvx_tier_dev::totals(t->pol, stats, t->s_pol);
    }
    *stats = t->totals;
    return KVX_OK;
}

namespace {

int frame_io(kvx_tier *t, int64_t frame, void *buf, bool to_store) {
    if (!t || !buf || frame < 0 || frame >= t->cfg.universe || t->bookkeeping) return KVX_EINVAL;
    int rc = kvx_tier_sync(t);
    if (rc != KVX_OK) return rc;
    std::lock_guard<std::mutex> lk(t->mu);
    const size_t fb = t->cfg.frame_bytes;
    if (t->pol) {  // where the device's bookkeeping says the frame is
        int32_t tier = 0;
        int64_t slot = 0;
        rc = kvx_tier_dev::location(t->pol, frame, &tier, &slot, t->s_pol);
        if (rc != KVX_OK) return rc;
        if (tier == 0) {
            uint8_t *d = t->dev_base + (size_t)slot * fb;
            return cuda_status(to_store ? cudaMemcpy(d, buf, fb, cudaMemcpyHostToDevice)
                                        : cudaMemcpy(buf, d, fb, cudaMemcpyDeviceToHost));
        }
        uint8_t *h = t->host_base + (size_t)slot * fb;
        if (to_store) std::memcpy(h, buf, fb); else std::memcpy(buf, h, fb);
        return KVX_OK;
    }
    if (t->dslot[frame] >= 0) {
        uint8_t *d = t->dev_base + (size_t)t->dslot[frame] * fb;
        return cuda_status(to_store ? cudaMemcpy(d, buf, fb, cudaMemcpyHostToDevice)
                                    : cudaMemcpy(buf, d, fb, cudaMemcpyDeviceToHost));
    }
    if (t->hslot[frame] >= 0) {
        uint8_t *h = t->host_base + (size_t)t->hslot[frame] * fb;
        if (to_store) std::memcpy(h, buf, fb); else std::memcpy(buf, h, fb);
        return KVX_OK;
    }
    return file_io(t->fd, buf, fb, (off_t)frame * (off_t)fb, to_store) ? KVX_OK : KVX_ECUDA;
}

}  // namespace

extern "C" KVX_API int kvx_tier_write_frame(kvx_tier *t, int64_t frame, const void *buf) {
    return frame_io(t, frame, const_cast<void *>(buf), true);
}

extern "C" KVX_API int kvx_tier_read_frame(kvx_tier *t, int64_t frame, void *buf) {
    return frame_io(t, frame, buf, false);
}
