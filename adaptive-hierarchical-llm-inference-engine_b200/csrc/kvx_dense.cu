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
#include <cuda.h>
#include <cooperative_groups.h>
#include <math_constants.h>

#include <mutex>

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

// ---------------------------------------------------------------------------
// head_dim 128 on the tensor cores (attention_tc128_kernel).
//
// mma.sync m16n8k8 with tf32 operands and fp32 accumulation, each product
// split three ways for fp32-grade accuracy over fp32's whole range
// ("3xTF32"): x = big + small with big = tf32(x), small = tf32(x - big),
// and a.b ~ big_a.big_b + big_a.small_b + small_a.big_b (the dropped
// small.small term and small's own rounding are ~2^-21 relative).
//  * A CTA owns 16 query rows (the mma's M) and half of the keys: the two
//    CTAs of a cluster split the keys and merge through distributed shared
//    memory, so 1,024 queries make 128 CTAs.
//  * K and V stream through shared memory in tiles of 64 keys (TMA, four
//    64 x 32 boxes each with 128-byte swizzle, so every fragment load below
//    is bank-conflict free) in a ring of three buffers: one producer warp
//    fills a buffer ("full" mbarrier) once all eight consumer warps have
//    released it ("empty" mbarrier, one arrival per warp), so the consumer
//    warps never meet at a block barrier inside the loop and drift apart
//    (one warp's softmax overlaps another's mmas).  Consumer warp w takes
//    keys 8w .. 8w+7 of each tile: S = Q K^T (16 k-steps), online softmax in
//    the log2 domain, O += P V (16 n-tiles); it issues the S mmas of tile
//    t+1 before the softmax and P V of tile t, so its own mma chains overlap
//    its softmax.
//  * P feeds the P.V mma straight from the S accumulators: a thread holds
//    keys 2t, 2t+1 of its rows, which the A fragment wants at k positions
//    t, t+4, so the P.V k order is permuted (position t <-> key 2t,
//    position t+4 <-> key 2t+1) and V rows are read in the same order.
//  * The 8 warps' (max, sum, O) merge through shared memory, then the
//    cluster's two CTAs through DSMEM; rank 0 writes the rows.
constexpr int kTcRows = 16, kTcKeys = 64, kTcWarpsD = 8, kTcOPad = 136;
constexpr int kTcTileFloats = kTcKeys * 128;               // one K or V tile: 4 swizzled boxes of 64 x 32
constexpr int kTcQWords = 16 * 32 * 8;                      // Q A-fragments: big [k-step][lane][4], then small

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t &big, uint32_t &small) {
    big = to_tf32(x);
    small = to_tf32(x - __uint_as_float(big));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// c += A.B with A = (ab + as), B = (bb + bs), three tf32 mmas
__device__ __forceinline__ void mma3(float (&c)[4], const uint32_t (&ab)[4], const uint32_t (&as)[4],
                                     uint32_t bb0, uint32_t bb1, uint32_t bs0, uint32_t bs1) {
    mma_tf32(c, as[0], as[1], as[2], as[3], bb0, bb1);
    mma_tf32(c, ab[0], ab[1], ab[2], ab[3], bs0, bs1);
    mma_tf32(c, ab[0], ab[1], ab[2], ab[3], bb0, bb1);
}

__device__ __forceinline__ void tma_load_2d_f(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Float index of (row r, dim d) in a tile of four 64 x 32 boxes loaded with
// 128-byte swizzle: box d / 32, row r, 16-byte chunk ((d / 4) % 8) XOR
// (r % 8).  The K and V fragment reads below hit 32 distinct banks.
__device__ __forceinline__ int swz_f(int r, int d) {
    return (d >> 5) * (kTcKeys * 32) + r * 32 + ((((d >> 2) & 7) ^ (r & 7)) << 2) + (d & 3);
}

constexpr int kTcStagesD = 3;
constexpr int kTcThreadsD = (kTcWarpsD + 1) * 32;  // 8 consumer warps + the producer
constexpr int kTcSmem = 1024 /* alignment */ + (2 * kTcStagesD * kTcTileFloats + kTcQWords) * 4 +
                       2 * kTcWarpsD * kTcRows * 4 + 2 * kTcRows * 4 + 2 * kTcStagesD * 8 + 16;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreadsD, 1)
attention_tc128_kernel(const float *__restrict__ Q, float *__restrict__ out, int seq_q, int seq_k,
                        float scale_log2, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) float dsm_raw[];
    float *dsm = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    float *kt = dsm;                                  // [3][4 boxes][64][32]
    float *vt = kt + kTcStagesD * kTcTileFloats;        // [3][4 boxes][64][32]
    uint4 *qfb = reinterpret_cast<uint4 *>(vt + kTcStagesD * kTcTileFloats);  // [16][32]
    uint4 *qfs = qfb + 16 * 32;                                              // [16][32]
    float *wm = reinterpret_cast<float *>(qfs + 16 * 32);                    // [8][16] warp maxima
    float *wl = wm + kTcWarpsD * kTcRows;                                     // [8][16] warp sums
    uint64_t *full = reinterpret_cast<uint64_t *>(wl + kTcWarpsD * kTcRows + 2 * kTcRows);
    uint64_t *empty = full + kTcStagesD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int rank = (int)cluster.block_rank();
    const int row0 = (blockIdx.x >> 1) * kTcRows;
    const int half = ((seq_k + 1) / 2 + kTcKeys - 1) / kTcKeys * kTcKeys;
    const int kbeg = rank * half, kend = min(seq_k, kbeg + half);
    const int ntiles = kend > kbeg ? (kend - kbeg + kTcKeys - 1) / kTcKeys : 0;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kTcStagesD; ++b) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], kTcWarpsD);
        }
        fence_barrier_init();
    }
    // Q as ready A fragments (all threads): lane ln's {a0..a3} of k-step ks
    for (int i = threadIdx.x; i < 16 * 32; i += blockDim.x) {
        const int ks = i >> 5, ln = i & 31, gg = ln >> 2, tt = ln & 3;
        uint32_t b[4], sm[4];
        const int rr[4] = {gg, gg + 8, gg, gg + 8}, dd[4] = {8 * ks + tt, 8 * ks + tt, 8 * ks + tt + 4, 8 * ks + tt + 4};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float x = row0 + rr[e] < seq_q ? Q[(size_t)(row0 + rr[e]) * 128 + dd[e]] : 0.f;
            split_tf32(x, b[e], sm[e]);
        }
        qfb[i] = make_uint4(b[0], b[1], b[2], b[3]);
        qfs[i] = make_uint4(sm[0], sm[1], sm[2], sm[3]);
    }
    __syncthreads();  // barriers initialised, Q fragments visible

    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;  // rows g, g + 8

    if (warp == kTcWarpsD) {  // ---- producer (the whole warp waits, lane 0 issues: it stays converged)
        for (int it = 0; it < ntiles; ++it) {
            const int b = it % kTcStagesD;
            if (it >= kTcStagesD)  // the consumers released tile it - 3
                (void)mbar_wait_bounded(&empty[b], ((it / kTcStagesD) - 1) & 1, nullptr);
            if (lane == 0) {
                const int key0 = kbeg + it * kTcKeys;
                float *kd = kt + b * kTcTileFloats, *vd = vt + b * kTcTileFloats;
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&full[b], 2u * kTcTileFloats * 4u);
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    tma_load_2d_f(kd + x * kTcKeys * 32, &tmk, 32 * x, key0, &full[b]);
                    tma_load_2d_f(vd + x * kTcKeys * 32, &tmv, 32 * x, key0, &full[b]);
                }
            }
            __syncwarp();
        }
    } else if (ntiles > 0) {  // ---- consumer warp: keys 8w .. 8w+7 of every tile
        const int kr = 8 * warp;
        // S = Q K^T over this warp's 8 keys of one tile: six independent
        // accumulator chains (product kind x k-step parity)
        auto qk = [&](const float *kd, float (&sacc)[4]) {
            float acc[6][4];
#pragma unroll
            for (int c = 0; c < 6; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 16; ++ks) {
                const int d0 = 8 * ks + t;
                const uint4 fb = qfb[ks * 32 + lane], fs = qfs[ks * 32 + lane];
                uint32_t bb0, bs0, bb1, bs1;
                split_tf32(kd[swz_f(kr + g, d0)], bb0, bs0);
                split_tf32(kd[swz_f(kr + g, d0 + 4)], bb1, bs1);
                const int p = ks & 1;
                mma_tf32(acc[p], fs.x, fs.y, fs.z, fs.w, bb0, bb1);
                mma_tf32(acc[2 + p], fb.x, fb.y, fb.z, fb.w, bs0, bs1);
                mma_tf32(acc[4 + p], fb.x, fb.y, fb.z, fb.w, bb0, bb1);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e)
                sacc[e] = ((acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e])) + (acc[4][e] + acc[5][e]);
        };
        float scur[4], snext[4] = {0.f, 0.f, 0.f, 0.f};
        (void)mbar_wait_bounded(&full[0], 0, nullptr);
        qk(kt, scur);
        for (int it = 0; it < ntiles; ++it) {
            const int b = it % kTcStagesD;
            if (it + 1 < ntiles) {  // the next tile's scores first: independent of this tile's softmax
                const int nb = (it + 1) % kTcStagesD;
                (void)mbar_wait_bounded(&full[nb], ((it + 1) / kTcStagesD) & 1, nullptr);
                qk(kt + nb * kTcTileFloats, snext);
            }
            const float *vd = vt + b * kTcTileFloats;
            // online softmax (log2 domain) of rows g (keys 2t, 2t+1) and g + 8
            const int kidx = kbeg + it * kTcKeys + 8 * warp + 2 * t;
            const float s00 = kidx < kend ? scur[0] * scale_log2 : -CUDART_INF_F;
            const float s01 = kidx + 1 < kend ? scur[1] * scale_log2 : -CUDART_INF_F;
            const float s10 = kidx < kend ? scur[2] * scale_log2 : -CUDART_INF_F;
            const float s11 = kidx + 1 < kend ? scur[3] * scale_log2 : -CUDART_INF_F;
            float mx0 = fmaxf(s00, s01), mx1 = fmaxf(s10, s11);
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            const float a0 = n0 == -CUDART_INF_F ? 1.f : exp2f(m0 - n0);
            const float a1 = n1 == -CUDART_INF_F ? 1.f : exp2f(m1 - n1);
            const float p00 = n0 == -CUDART_INF_F ? 0.f : exp2f(s00 - n0);
            const float p01 = n0 == -CUDART_INF_F ? 0.f : exp2f(s01 - n0);
            const float p10 = n1 == -CUDART_INF_F ? 0.f : exp2f(s10 - n1);
            const float p11 = n1 == -CUDART_INF_F ? 0.f : exp2f(s11 - n1);
            m0 = n0;
            m1 = n1;
            l0 = l0 * a0 + (p00 + p01);
            l1 = l1 * a1 + (p10 + p11);
            uint32_t pb[4], ps[4];
            split_tf32(p00, pb[0], ps[0]);
            split_tf32(p10, pb[1], ps[1]);
            split_tf32(p01, pb[2], ps[2]);
            split_tf32(p11, pb[3], ps[3]);
            // O = O * alpha + P V (alpha is 1 unless a running max moved;
            // scaling unconditionally keeps the loop body one basic block)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                o[j][0] *= a0;
                o[j][1] *= a0;
                o[j][2] *= a1;
                o[j][3] *= a1;
                uint32_t bb0, bs0, bb1, bs1;
                split_tf32(vd[swz_f(kr + 2 * t, 8 * j + g)], bb0, bs0);
                split_tf32(vd[swz_f(kr + 2 * t + 1, 8 * j + g)], bb1, bs1);
                mma3(o[j], pb, ps, bb0, bb1, bs0, bs1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[b]);  // this warp is done with tile it's buffer
#pragma unroll
            for (int e = 0; e < 4; ++e) scur[e] = snext[e];
        }
    }
    __syncthreads();  // every warp is done with the ring: it holds the partials now

    // ---- merge the 8 consumer warps, then the cluster's two CTAs
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (warp < kTcWarpsD) {
        if (t == 0) {
            wm[warp * kTcRows + g] = m0;
            wm[warp * kTcRows + g + 8] = m1;
            wl[warp * kTcRows + g] = l0;
            wl[warp * kTcRows + g + 8] = l1;
        }
        float *po = dsm + warp * kTcRows * kTcOPad;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            *reinterpret_cast<float2 *>(po + g * kTcOPad + 8 * j + 2 * t) = make_float2(o[j][0], o[j][1]);
            *reinterpret_cast<float2 *>(po + (g + 8) * kTcOPad + 8 * j + 2 * t) = make_float2(o[j][2], o[j][3]);
        }
    }
    __syncthreads();
    float *co = dsm + kTcWarpsD * kTcRows * kTcOPad;  // [16][128]
    float *cml = co + kTcRows * 128;                  // [16][2]
    if (threadIdx.x < kTcRows) {
        const int r = threadIdx.x;
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < kTcWarpsD; ++w) M = fmaxf(M, wm[w * kTcRows + r]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarpsD; ++w) {
            const float mw = wm[w * kTcRows + r];
            const float sw = mw == -CUDART_INF_F ? 0.f : exp2f(mw - M);
            L += sw * wl[w * kTcRows + r];
            wm[w * kTcRows + r] = sw;
        }
        cml[2 * r] = M;
        cml[2 * r + 1] = L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kTcRows * 128; i += blockDim.x) {
        const int r = i >> 7, d = i & 127;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarpsD; ++w) acc += wm[w * kTcRows + r] * dsm[(w * kTcRows + r) * kTcOPad + d];
        co[i] = acc;
    }
    cluster.sync();
    if (rank == 0) {
        const float *ro = cluster.map_shared_rank(co, 1);
        const float *rml = cluster.map_shared_rank(cml, 1);
        for (int i = threadIdx.x; i < kTcRows * 128; i += blockDim.x) {
            const int r = i >> 7;
            if (row0 + r >= seq_q) continue;
            const float Ma = cml[2 * r], La = cml[2 * r + 1], Mb = rml[2 * r], Lb = rml[2 * r + 1];
            const float M = fmaxf(Ma, Mb);
            const float wa = Ma == -CUDART_INF_F ? 0.f : exp2f(Ma - M);
            const float wb = Mb == -CUDART_INF_F ? 0.f : exp2f(Mb - M);
            float L = wa * La + wb * Lb;
            if (L == 0.f) L = 1e-6f;  // TensorOps::softmax's guard
            out[(size_t)(row0 + r) * 128 + (i & 127)] = (wa * co[i] + wb * ro[i]) / L;
        }
    }
    cluster.sync();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda): rows of 128 fp32, boxes of 64 rows x 32 floats, 128-byte
// swizzle, zero fill past the last row.
using EncodeTiledFnD = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool make_rows_map(CUtensorMap *tm, const float *base, long long rows) {
    static EncodeTiledFnD fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFnD>(f);
    });
    if (!fn || rows <= 0 || rows > (1ll << 31)) return false;
    cuuint64_t gdim[2] = {128, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {128 * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)kTcKeys};
    cuuint32_t estride[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), gdim, gstride, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
    if (dim == kDD && aligned && !((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(out)) & 15) &&
        seq_q <= (int64_t)0x3fffffff) {
        static std::atomic<bool> attr_done[kMaxDevices];
        CUtensorMap tmk, tmv;
        if (make_rows_map(&tmk, K, seq_k) && make_rows_map(&tmv, V, seq_k)) {
            const unsigned tiles = (unsigned)((seq_q + kTcRows - 1) / kTcRows);
            if (ensure_smem_attr(attr_done, attention_tc128_kernel, kTcSmem) != KVX_OK) return KVX_ECUDA;
            attention_tc128_kernel<<<2 * tiles, kTcThreadsD, kTcSmem, static_cast<cudaStream_t>(stream)>>>(
                Q, out, (int)seq_q, (int)seq_k, s * 1.4426950408889634f, tmk, tmv);
            return launch_status();
        }
    }
    if (dim == kDD && aligned) {
        attention_dense128_kernel<<<(unsigned)((seq_q + kDQ - 1) / kDQ), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            Q, K, V, out, (int)seq_q, (int)seq_k, s);
        return launch_status();
    }
    attention_dense_kernel<<<(unsigned)seq_q, 128, 4 * dim * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
        Q, K, V, out, (int)seq_k, dim, s);
    return launch_status();
}
