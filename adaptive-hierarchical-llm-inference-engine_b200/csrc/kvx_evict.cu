// kvx_evict.cu -- device-side eviction bookkeeping.
//
//  * kvx_lru_select: arg-min over access stamps.  Replaces
//    LRUEvictionPolicy::selectPageToEvict
//    (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23) and
//    KVCacheGPU::findLRUPage (native-engine/cpp/KVCacheGPU.cpp:54-66): the
//    strictly smallest stamp wins, the lowest index on ties, and a stamp of
//    UINT64_MAX (the reference's initial minToken) is never chosen.
//    One CTA of 1024 threads reads the stamps with 16-byte loads; each thread
//    keeps its first minimum in index order, then a (stamp, index)
//    lexicographic tree reduction.  No workspace, deterministic.
//  * kvx_evict_select / kvx_evict_select_composite: the other policies of
//    native-engine/cpp/AdvancedEvictionPolicy.cpp (TokenWeighted :35-64,
//    AttentionBased :69-105, Predictive :119-152) and the weighted
//    CompositeEvictionManager (:238-263), scored exactly as the reference's
//    selectPageToEvict scores them: with currentToken = 0, so a page's token
//    age is 0 - lastAccessToken modulo 2^64.  The reference's pow / log of
//    those ages are evaluated in double and rounded to float; with wrapped
//    ages they are 0 / 1 and one shared value in practice.  Highest score
//    strictly above -1 wins, the lowest index on ties (+0 and -0 tie), NaN
//    scores never.  Same single-CTA scan and tree reduction as above.
#include "kvx_common.cuh"

namespace kvx {
namespace {

__device__ __forceinline__ void take(uint64_t &best, long long &bi, uint64_t v, long long i) {
    if (v < best || (v == best && v != UINT64_MAX && i < bi)) {
        best = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024)
lru_select_kernel(const uint64_t *__restrict__ stamps, size_t n, int32_t *victim) {
    uint64_t best = UINT64_MAX;
    long long bi = -1;
    const size_t pairs = n / 2;
    for (size_t i = threadIdx.x; i < pairs; i += blockDim.x) {
        const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2 *>(stamps) + i);
        take(best, bi, v.x, (long long)(2 * i));
        take(best, bi, v.y, (long long)(2 * i + 1));
    }
    if ((n & 1) && threadIdx.x == 0) take(best, bi, stamps[n - 1], (long long)(n - 1));
    // warp then block reduction on (stamp, index)
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const uint64_t ov = __shfl_xor_sync(0xffffffffu, best, off);
        const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi >= 0 && (bi < 0 || ov < best || (ov == best && oi < bi))) {
            best = ov;
            bi = oi;
        }
    }
    __shared__ uint64_t sv[32];
    __shared__ long long si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : UINT64_MAX;
        bi = lane < nw ? si[lane] : -1;
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const uint64_t ov = __shfl_xor_sync(0xffffffffu, best, off);
            const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi >= 0 && (bi < 0 || ov < best || (ov == best && oi < bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) *victim = (int32_t)bi;
    }
}

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

__device__ __forceinline__ bool better(float s, long long i, float best, long long bi) {
    return i >= 0 && (bi < 0 || s > best || (s == best && i < bi));
}

// One CTA.  lru: selectPageToEvict of LRU (smallest lastAccessToken below
// UINT64_MAX); otherwise the (weighted) scores of `ps`.
__global__ void __launch_bounds__(1024)
policy_select_kernel(const EvictMetrics *__restrict__ pages, size_t n, PolicySet ps, float decay,
                     const float *__restrict__ predicted, bool lru, int32_t *page_id) {
    float best = -1.0f;
    uint64_t bmin = UINT64_MAX;
    long long bi = -1;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
        const EvictMetrics m = pages[i];
        if (lru) {
            if (m.last_access_token < bmin) {
                bmin = m.last_access_token;
                bi = (long long)i;
            }
            continue;
        }
        const float pred = predicted ? predicted[i] : -1.0f;
        float sc;
        if (ps.n == 1) {
            sc = policy_score(ps.type[0], m, decay, pred);
        } else {
            sc = 0.0f;
            for (int p = 0; p < ps.n; ++p)
                sc = __fadd_rn(sc, __fmul_rn(ps.weight[p], policy_score(ps.type[p], m, decay, pred)));
        }
        if (sc > best) {
            best = sc;
            bi = (long long)i;
        }
    }
    // (score, index) reduction; LRU compares negated order through bmin
    auto reduce = [&](float &b, uint64_t &bm, long long &i0) {
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, b, off);
            const uint64_t om = __shfl_xor_sync(0xffffffffu, bm, off);
            const long long oi = __shfl_xor_sync(0xffffffffu, i0, off);
            const bool take = lru ? (oi >= 0 && (i0 < 0 || om < bm || (om == bm && oi < i0)))
                                  : better(ob, oi, b, i0);
            if (take) {
                b = ob;
                bm = om;
                i0 = oi;
            }
        }
    };
    reduce(best, bmin, bi);
    __shared__ float sb[32];
    __shared__ uint64_t sm[32];
    __shared__ long long si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sb[warp] = best;
        sm[warp] = bmin;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sb[lane] : -1.0f;
        bmin = lane < nw ? sm[lane] : UINT64_MAX;
        bi = lane < nw ? si[lane] : -1;
        reduce(best, bmin, bi);
        if (lane == 0) *page_id = bi >= 0 ? pages[bi].page_id : -1;
    }
}

int launch_policy_select(const void *pages, size_t n, const PolicySet &ps, float decay, const float *predicted,
                         bool lru, int32_t *page_id, void *stream) {
    if (!page_id || (n && !pages) || n > 0x7fffffffull) return KVX_EINVAL;
    if (reinterpret_cast<uintptr_t>(pages) & 7) return KVX_EINVAL;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) return cudaMemsetAsync(page_id, 0xff, sizeof(int32_t), st) == cudaSuccess ? KVX_OK : KVX_ECUDA;
    policy_select_kernel<<<1, 1024, 0, st>>>(static_cast<const EvictMetrics *>(pages), n, ps, decay, predicted, lru,
                                             page_id);
    return launch_status();
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
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) {
        return cudaMemsetAsync(victim, 0xff, sizeof(int32_t), st) == cudaSuccess ? KVX_OK : KVX_ECUDA;
    }
    lru_select_kernel<<<1, 1024, 0, st>>>(stamps, n, victim);
    return launch_status();
}
