// kvx_dense.cu -- dense (unpaged) softmax and attention for the
// runtime::gpu::cuda_softmax / cuda_attention drop-ins.
//
// Replaces softmax_row_kernel + the two cuBLAS SGEMMs of the reference's
// runtime/gpu/cuda_executor.cu:149-311 and the 1-thread-per-row softmax of
// native-engine/cuda/softmax.cu.  Semantics follow TensorOps
// (runtime/tensor_ops.cpp:155-219): row softmax with the sum==0 -> 1e-6
// guard; attention = softmax(Q K^T * scale) V, scale 1/sqrt(dim) by default
// (the reference's cuda_attention leaves the scale out; TensorOps and
// native-engine/cuda/attention.cu apply it).
//  * softmax: one CTA per row, block reductions of max and sum.
//  * attention, head_dim 128: 8 query rows per CTA over K / V tiles staged
//    in shared memory (attention_dense128_kernel); other head dims (<= 1024):
//    one CTA of 4 warps per query row, each warp every 4th key, lanes split
//    the head dimension, online softmax per warp, warps merged through
//    shared memory.  Neither materialises the seq x seq score matrix.
#include <math_constants.h>

#include "kvx_common.cuh"

namespace kvx {
namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(256) softmax_rows_kernel(const float *__restrict__ in,
                                                           float *__restrict__ out, long long cols) {
    __shared__ float red[8];
    const float *row = in + (size_t)blockIdx.x * cols;
    float *orow = out + (size_t)blockIdx.x * cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = -CUDART_INF_F;
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, row[c]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[lane < 8 ? lane : 0];
    m = warp_max(m);
    __syncthreads();
    float s = 0.f;
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) s += expf(row[c] - m);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = lane < 8 ? red[lane] : 0.f;
    s = warp_sum(s);
    if (s == 0.f) s = 1e-6f;
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) orow[c] = expf(row[c] - m) / s;
}

constexpr int kMaxDimPerLane = 32;  // head dim <= 1024

__global__ void __launch_bounds__(128) attention_dense_kernel(const float *__restrict__ Q,
                                                              const float *__restrict__ K,
                                                              const float *__restrict__ V,
                                                              float *__restrict__ out, int seq_k,
                                                              int dim, float scale) {
    __shared__ float s_m[4], s_l[4];
    extern __shared__ float s_acc[];  // [4][dim]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *q = Q + (size_t)blockIdx.x * dim;
    const int per = (dim + 31) / 32;
    float qr[kMaxDimPerLane], acc[kMaxDimPerLane];
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) {
        const int d = lane + 32 * i;
        qr[i] = (i < per && d < dim) ? q[d] : 0.f;
        acc[i] = 0.f;
    }
    float m = -CUDART_INF_F, l = 0.f;
    for (int j = warp; j < seq_k; j += 4) {
        const float *k = K + (size_t)j * dim;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxDimPerLane; ++i) {
            const int d = lane + 32 * i;
            if (i < per && d < dim) dot = fmaf(qr[i], k[d], dot);
        }
        const float sc = warp_sum(dot) * scale;
        const float mn = fmaxf(m, sc);
        const float a = expf(m - mn), p = expf(sc - mn);
        l = l * a + p;
        m = mn;
        const float *v = V + (size_t)j * dim;
#pragma unroll
        for (int i = 0; i < kMaxDimPerLane; ++i) {
            const int d = lane + 32 * i;
            if (i < per && d < dim) acc[i] = fmaf(p, v[d], acc[i] * a);
        }
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) {
        const int d = lane + 32 * i;
        if (i < per && d < dim) s_acc[warp * dim + d] = acc[i];
    }
    __syncthreads();
    float M = -CUDART_INF_F;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f;
    for (int w = 0; w < 4; ++w) L += s_m[w] == -CUDART_INF_F ? 0.f : s_l[w] * expf(s_m[w] - M);
    if (L == 0.f) L = 1e-6f;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < 4; ++w)
            if (s_m[w] != -CUDART_INF_F) o += s_acc[w * dim + d] * expf(s_m[w] - M);
        out[(size_t)blockIdx.x * dim + d] = o / L;
    }
}

// head_dim 128: a CTA of 8 warps takes 8 query rows (one per warp) and
// streams K and V through shared memory in tiles of 32 keys, so each key is
// read from L2 once per 8 queries instead of once per query.  In a tile,
// lane j scores key j (K rows padded to 129 floats: the 32 lanes reading
// one column hit 32 banks), the warp takes the tile's max, rescales once,
// and P.V runs with p_j broadcast from lane j and lane d holding dims
// d, d + 32, d + 64, d + 96.  Same order of operations per key as the
// general kernel up to the per-tile max.
constexpr int kDQ = 8, kDK = 32, kDD = 128, kDPad = kDD + 1;

__global__ void __launch_bounds__(256) attention_dense128_kernel(const float *__restrict__ Q,
                                                                 const float *__restrict__ K,
                                                                 const float *__restrict__ V,
                                                                 float *__restrict__ out, int seq_q, int seq_k,
                                                                 float scale) {
    __shared__ float sk[kDK * kDPad];
    __shared__ __align__(16) float sv[kDK * kDD];
    __shared__ __align__(16) float sq[kDQ * kDD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kDQ + warp;
    for (int i = threadIdx.x; i < kDQ * kDD; i += blockDim.x) {
        const int r = blockIdx.x * kDQ + i / kDD;
        sq[i] = r < seq_q ? Q[(size_t)r * kDD + i % kDD] : 0.f;
    }
    float m = -CUDART_INF_F, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    const float *q = sq + warp * kDD;
    for (int k0 = 0; k0 < seq_k; k0 += kDK) {
        const int nk = min(kDK, seq_k - k0);
        __syncthreads();  // the previous tile is consumed (and sq written, first time)
        for (int i = threadIdx.x; i < kDK * kDD / 4; i += blockDim.x) {
            const int j = i / (kDD / 4), d4 = i % (kDD / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (j < nk) {
                kv = __ldg(reinterpret_cast<const float4 *>(K + (size_t)(k0 + j) * kDD) + d4);
                vv = __ldg(reinterpret_cast<const float4 *>(V + (size_t)(k0 + j) * kDD) + d4);
            }
            float *kr = sk + j * kDPad + 4 * d4;
            kr[0] = kv.x, kr[1] = kv.y, kr[2] = kv.z, kr[3] = kv.w;
            reinterpret_cast<float4 *>(sv + j * kDD)[d4] = vv;
        }
        __syncthreads();
        float dot = 0.f;
        const float *kr = sk + lane * kDPad;
#pragma unroll 8
        for (int d = 0; d < kDD; d += 4) {
            const float4 qv = *reinterpret_cast<const float4 *>(q + d);
            dot = fmaf(qv.x, kr[d], dot);
            dot = fmaf(qv.y, kr[d + 1], dot);
            dot = fmaf(qv.z, kr[d + 2], dot);
            dot = fmaf(qv.w, kr[d + 3], dot);
        }
        const float sc = lane < nk ? dot * scale : -CUDART_INF_F;
        const float mn = fmaxf(m, warp_max(sc));
        const float a = expf(m - mn);
        const float p = lane < nk ? expf(sc - mn) : 0.f;
        l = l * a + warp_sum(p);
        m = mn;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] *= a;
        for (int j = 0; j < nk; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            const float *vr = sv + j * kDD + lane;
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[c] = fmaf(pj, vr[32 * c], acc[c]);
        }
    }
    if (row < seq_q) {
        const float L = l == 0.f ? 1e-6f : l;
#pragma unroll
        for (int c = 0; c < 4; ++c) out[(size_t)row * kDD + lane + 32 * c] = acc[c] / L;
    }
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_softmax_rows(const float *in, float *out, int64_t rows, int64_t cols,
                                        void *stream) {
    if (!in || !out || rows < 0 || cols <= 0 || rows > 0x7fffffff) return KVX_EINVAL;
    if (rows == 0) return KVX_OK;
    softmax_rows_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, cols);
    return launch_status();
}

extern "C" KVX_API int kvx_attention_dense(const float *Q, const float *K, const float *V, float *out,
                                           int64_t seq_q, int64_t seq_k, int32_t dim, float scale,
                                           void *stream) {
    if (!Q || !K || !V || !out || seq_q < 0 || seq_k <= 0 || dim <= 0) return KVX_EINVAL;
    if (dim > 32 * kMaxDimPerLane || seq_q > 0x7fffffff || seq_k > 0x7fffffff) return KVX_EUNSUPPORTED;
    if (seq_q == 0) return KVX_OK;
    const float s = scale > 0.f ? scale : 1.0f / sqrtf((float)dim);
    const bool aligned = !((reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V)) & 15);
    if (dim == kDD && aligned) {
        attention_dense128_kernel<<<(unsigned)((seq_q + kDQ - 1) / kDQ), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            Q, K, V, out, (int)seq_q, (int)seq_k, s);
        return launch_status();
    }
    attention_dense_kernel<<<(unsigned)seq_q, 128, 4 * dim * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
        Q, K, V, out, (int)seq_k, dim, s);
    return launch_status();
}
