// kvx_evict.cu -- device-side eviction bookkeeping.
//
//  * kvx_lru_select: arg-min over access stamps.  Replaces
//    LRUEvictionPolicy::selectPageToEvict
//    (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23) and
//    KVCacheGPU::findLRUPage (native-engine/cpp/KVCacheGPU.cpp:54-66): the
//    strictly smallest stamp wins, the lowest index on ties, and a stamp of
//    UINT64_MAX (the reference's initial minToken) is never chosen.
//    One cluster of 8 CTAs x 1024 threads scans the stamps; each thread
//    keeps its first minimum in index order, then a (stamp, index)
//    lexicographic reduction over warps, CTAs and -- through distributed
//    shared memory -- the cluster.  One launch, no workspace, deterministic.
//  * kvx_evict_select / kvx_evict_select_composite: the other policies of
//    native-engine/cpp/AdvancedEvictionPolicy.cpp (TokenWeighted :35-64,
//    AttentionBased :69-105, Predictive :119-152) and the weighted
//    CompositeEvictionManager (:238-263), scored exactly as the reference's
//    selectPageToEvict scores them: with currentToken = 0, so a page's token
//    age is 0 - lastAccessToken modulo 2^64.  The reference's pow / log of
//    those ages are evaluated in double and rounded to float; with wrapped
//    ages they are 0 / 1 and one shared value in practice.  Highest score
//    strictly above -1 wins, the lowest index on ties (+0 and -0 tie), NaN
//    scores never.  Same cluster scan: a score becomes a rank (smaller is
//    better) so both reductions are one (rank, index) minimum.
#include <cooperative_groups.h>

#include "kvx_common.cuh"

namespace kvx {
namespace {

// native-engine/include/AdvancedEvictionPolicy.h:19-27, same layout.
struct EvictMetrics {
    uint64_t last_access_token;
    float total_attention, average_attention, access_frequency;
    uint32_t pad0;
    uint64_t creation_time, page_size;
    int32_t page_id;
    uint32_t pad1;
};
static_assert(sizeof(EvictMetrics) == 48, "EvictionMetrics layout");

constexpr int kMaxPolicies = 8;
struct PolicySet {
    int32_t n;
    int32_t type[kMaxPolicies];
    float weight[kMaxPolicies];
};

// calculateScore(m, 0) of one policy (AdvancedEvictionPolicy.cpp:29-31, 60-64,
// 95-105, 142-152).
__device__ __forceinline__ float policy_score(int type, const EvictMetrics &m, float decay, float pred) {
    const float age = __ull2float_rn(0ull - m.last_access_token);
    switch (type) {
    case 0: return age;
    case 1: return __fsub_rn(1.0f, (float)pow((double)decay, (double)age));
    case 2: {
        const float recency = (float)log((double)__fadd_rn(age, 1.0f));
        return __fmul_rn(__fsub_rn(1.0f, m.average_attention), recency);
    }
    default: return pred < 0.f ? 1000.0f : __fsub_rn(0.0f, pred);
    }
}

constexpr int kSelCtas = 8;        // one portable cluster
constexpr int kSelThreads = 1024;

// Rank of a candidate, smaller is better; UINT64_MAX never wins.
struct StampRank {  // LRU over raw stamps: the stamp itself, the index out
    const uint64_t *stamps;
    __device__ uint64_t rank(size_t i) const { return __ldg(stamps + i); }
    __device__ int32_t result(long long i) const { return (int32_t)i; }
};

struct PolicyRank {  // selectPageToEvict over EvictionMetrics, the page id out
    const EvictMetrics *pages;
    PolicySet ps;
    float decay;
    const float *predicted;
    bool lru;
    __device__ uint64_t rank(size_t i) const {
        const EvictMetrics &m = pages[i];
        if (lru) return m.last_access_token;
        const float pred = predicted ? predicted[i] : -1.0f;
        float sc;
        if (ps.n == 1) {
            sc = policy_score(ps.type[0], m, decay, pred);
        } else {
            sc = 0.0f;
            for (int p = 0; p < ps.n; ++p)
                sc = __fadd_rn(sc, __fmul_rn(ps.weight[p], policy_score(ps.type[p], m, decay, pred)));
        }
        if (!(sc > -1.0f)) return UINT64_MAX;  // best starts at -1, strict '>': NaN never
        // larger score -> smaller rank; +0 and -0 tie
        const uint32_t u = __float_as_uint(sc == 0.0f ? 0.0f : sc);
        const uint32_t key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        return (uint64_t)(0xFFFFFFFFu - key);
    }
    __device__ int32_t result(long long i) const { return pages[i].page_id; }
};

__device__ __forceinline__ void min_rank(uint64_t &best, long long &bi, uint64_t v, long long i) {
    if (i >= 0 && v != UINT64_MAX && (bi < 0 || v < best || (v == best && i < bi))) {
        best = v;
        bi = i;
    }
}

__device__ __forceinline__ void warp_min_rank(uint64_t &best, long long &bi) {
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const uint64_t ov = __shfl_xor_sync(0xffffffffu, best, off);
        const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
        min_rank(best, bi, ov, oi);
    }
}

template <typename Src>
__global__ void __cluster_dims__(kSelCtas, 1, 1) __launch_bounds__(kSelThreads)
select_kernel(Src src, size_t n, int32_t *out) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned cr = cluster.block_rank();
    uint64_t best = UINT64_MAX;
    long long bi = -1;
    // each thread visits its indices in increasing order: the first minimum stays
    for (size_t i = (size_t)cr * kSelThreads + threadIdx.x; i < n; i += (size_t)kSelCtas * kSelThreads) {
        const uint64_t r = src.rank(i);
        if (r < best) {
            best = r;
            bi = (long long)i;
        }
    }
    warp_min_rank(best, bi);
    __shared__ uint64_t sv[32];
    __shared__ long long si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        best = sv[lane];
        bi = si[lane];
        warp_min_rank(best, bi);
        if (lane == 0) {
            sv[0] = best;
            si[0] = bi;
        }
    }
    cluster.sync();  // every CTA's (rank, index) is in its shared memory
    if (cr == 0 && warp == 0) {
        best = UINT64_MAX;
        bi = -1;
        if (lane < kSelCtas) {
            best = *cluster.map_shared_rank(&sv[0], lane);
            bi = *cluster.map_shared_rank(&si[0], lane);
        }
        warp_min_rank(best, bi);
        if (lane == 0) *out = bi >= 0 ? src.result(bi) : -1;
    }
    cluster.sync();  // keep the other CTAs' shared memory until it was read
}

template <typename Src> int launch_select(const Src &src, size_t n, int32_t *out, void *stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) return cudaMemsetAsync(out, 0xff, sizeof(int32_t), st) == cudaSuccess ? KVX_OK : KVX_ECUDA;
    select_kernel<Src><<<kSelCtas, kSelThreads, 0, st>>>(src, n, out);
    return launch_status();
}

int launch_policy_select(const void *pages, size_t n, const PolicySet &ps, float decay, const float *predicted,
                         bool lru, int32_t *page_id, void *stream) {
    if (!page_id || (n && !pages) || n > 0x7fffffffull) return KVX_EINVAL;
    if (reinterpret_cast<uintptr_t>(pages) & 7) return KVX_EINVAL;
    return launch_select(PolicyRank{static_cast<const EvictMetrics *>(pages), ps, decay, predicted, lru}, n, page_id,
                         stream);
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_evict_select(int32_t policy, const kvx_evict_metrics *pages, size_t n, float decay,
                                        const float *predicted, int32_t *page_id, void *stream) {
    if (policy < KVX_EVICT_LRU || policy > KVX_EVICT_PREDICTIVE) return KVX_EINVAL;
    PolicySet ps{};
    ps.n = 1;
    ps.type[0] = policy;
    ps.weight[0] = 1.0f;
    return launch_policy_select(pages, n, ps, decay, predicted, policy == KVX_EVICT_LRU, page_id, stream);
}

extern "C" KVX_API int kvx_evict_select_composite(const int32_t *policies, const float *weights,
                                                  int32_t num_policies, const kvx_evict_metrics *pages, size_t n,
                                                  float decay, const float *predicted, int32_t *page_id,
                                                  void *stream) {
    if (!policies || !weights || num_policies < 1 || num_policies > kMaxPolicies) return KVX_EINVAL;
    if (num_policies == 1) return kvx_evict_select(policies[0], pages, n, decay, predicted, page_id, stream);
    PolicySet ps{};
    ps.n = num_policies;
    for (int p = 0; p < num_policies; ++p) {
        if (policies[p] < KVX_EVICT_LRU || policies[p] > KVX_EVICT_PREDICTIVE) return KVX_EINVAL;
        ps.type[p] = policies[p];
        ps.weight[p] = weights[p];
    }
    return launch_policy_select(pages, n, ps, decay, predicted, false, page_id, stream);
}

extern "C" KVX_API int kvx_lru_select(const uint64_t *stamps, size_t n, int32_t *victim,
                                      void *stream) {
    if (!victim || (n && !stamps)) return KVX_EINVAL;
    if (n > 0x7fffffffull) return KVX_EINVAL;
    if (reinterpret_cast<uintptr_t>(stamps) & 15) return KVX_EINVAL;
    return launch_select(StampRank{stamps}, n, victim, stream);
}
