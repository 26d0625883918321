// kvx_decode_params.cuh -- parameters shared by the paged decode kernels
// (SIMT path in kvx_decode.cu, tensor-core path in kvx_decode_tc.cu).
#pragma once
#include <math_constants.h>

#include "kvx_common.cuh"

namespace kvx {

struct DecodeParams {
    const uint8_t *pool;
    const float *stats;
    const int32_t *block_table;
    const int32_t *seq_lens;
    const void *q;
    void *out;
    float *part_o;   // [batch][hq][max_splits][128]
    float *part_ml;  // [batch][hq][max_splits][2]
    int32_t *counters;  // [batch][hkv][nhg], zero between launches
    const int32_t *positions;  // fused append: token position per sequence (else null)
    const uint8_t *new_k, *new_v;  // fused append rows [batch][hkv][128]
    int32_t *error_flag;
    // attention mass (tensor-core path only; null = off): per (sequence,
    // q-head, logical page) the running max and the page's sum of
    // exp2(score - max) [batch][hq][max_pages][2]; per (sequence, q-head)
    // the final max and sum [batch][hq][2]
    float *attn_pm, *attn_ml;
    // launch completion signal (null = off): done[0] counts finished CTAs
    // (left at zero), done[1] receives `epoch` once every CTA has finished
    uint32_t *done;
    uint32_t epoch;
    int num_pages, hkv, hq, max_pages, max_splits, chunk, group, nhg;
    float scale_log2;
};

// Programmatic dependent launch (launches with
// cudaLaunchAttributeProgrammaticStreamSerialization): let the next grid on
// the stream be scheduled once every CTA of this one got here, and wait for
// the previous grid's completion (a no-op without such a launch).
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Completion signal of a whole launch, called by every CTA after its last
// global write: the CTA's writes are released (barrier, then a GPU-scope
// fence by thread 0) before it counts itself in done[0]; the CTA that counts
// last resets done[0] and stores `epoch` to done[1] with release semantics,
// so whoever observes done[1] >= epoch (a stream memory wait on another
// stream) sees every output of the launch.  Each CTA first waits for the
// previous grid on the stream, whose last CTA resets the same counter:
// launches that share `done` must be ordered on one stream.
__device__ __forceinline__ void grid_done_signal(uint32_t *done, uint32_t epoch) {
    grid_dependency_wait();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
        __threadfence();
        if (atomicAdd(done, 1u) == total - 1) {
            atomicExch(done, 0u);
            __threadfence();
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(done + 1), "r"(epoch) : "memory");
        }
    }
}

// Flash-decoding combine of one output element: the splits' (m, l) pairs
// at part_ml[(base + c) * 2] and partial sums part_o[(base + c) * 128 + d],
// c < nsplit, folded in split order; returns O and sets the row's max M and
// sum L.  Loads go out in groups of 8: a long sequence has up to
// max_pages / 4 splits, walked by one thread per (row, dim), so they must
// not wait one by one.
__device__ __forceinline__ float fold_splits(const float *part_ml, const float *part_o, size_t base, int nsplit,
                                             int d, float &M, float &L) {
    const float2 *ml = reinterpret_cast<const float2 *>(part_ml) + base;
    const float *po = part_o + base * 128 + d;
    M = -CUDART_INF_F;
    int c = 0;
    for (; c + 8 <= nsplit; c += 8) {
        float mv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mv[u] = __ldcg(&ml[c + u].x);
#pragma unroll
        for (int u = 0; u < 8; ++u) M = fmaxf(M, mv[u]);
    }
    for (; c < nsplit; ++c) M = fmaxf(M, __ldcg(&ml[c].x));
    float O = 0.f;
    L = 0.f;
    auto fold = [&](float2 m_l, float o) {
        const float w = m_l.x == -CUDART_INF_F ? 0.f : exp2f(m_l.x - M);
        L += w * m_l.y;
        O += w * o;
    };
    c = 0;
    for (; c + 8 <= nsplit; c += 8) {
        float2 mlv[8];
        float ov[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            mlv[u] = __ldcg(ml + c + u);
            ov[u] = __ldcg(po + (size_t)(c + u) * 128);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) fold(mlv[u], ov[u]);
    }
    for (; c < nsplit; ++c) fold(__ldcg(ml + c), __ldcg(po + (size_t)c * 128));
    return O;
}

// Tensor-core path for fp16 and int8 pools (kvx_decode_tc.cu).  Returns a
// kvx_status; KVX_EUNSUPPORTED when the geometry has no tensor-core kernel.
int launch_decode_tc(DecodeParams &p, int kv_dtype, int io_dtype, int batch, cudaStream_t st);

}  // namespace kvx
