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
//  * attention, head_dim 128 with 16-byte aligned rows: the 5th-generation
//    tensor cores (attention_umma_kernel, tcgen05.mma kind::tf32 with
//    3xTF32 products) over 128 query rows x 64 keys per CTA, then
//    combine_splits_kernel over the key tiles.  Head dim 128 with only K / V
//    aligned: 8 query rows per CTA over K / V tiles staged in shared memory
//    (attention_dense128_kernel, fp32 CUDA cores).  Other head dims
//    (<= 1024): one CTA of 4 warps per query row, each warp every 4th key,
//    lanes split the head dimension, online softmax per warp, warps merged
//    through shared memory.  None materialises the seq x seq score matrix.
#include <cuda.h>
#include <math_constants.h>

#include <algorithm>
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
// head_dim 128 on the 5th-generation tensor cores (attention_umma_kernel).
//
// tcgen05.mma kind::tf32 (one thread issues, accumulators in tensor memory),
// 3xTF32 products for fp32-grade accuracy: every operand element x enters
// as big = x itself, of which the tensor core reads the top 19 bits (x with
// the low 13 mantissa bits cleared), and small = x - that truncation
// (exact); a.b ~ big.big + big.small + small.big.  A CTA owns 128 query
// rows (the MMA's M, one tensor-memory lane per row) and a range of 64-key
// tiles; per tile:
//  * TMA brings the raw fp32 Q (4 boxes of 128 rows x 32 floats), K and V
//    (4 boxes of 64 keys x 32 floats each), 128-byte swizzle: the K-major
//    canonical layout of the MMA's shared-memory descriptors.  Rows past
//    the ends read as zero.  The raw Q and K are the big operands;
//  * the CTA's 256 threads write Q small and K small at the same swizzled
//    offsets of their own regions;
//  * S = Q K^T: 16 k-steps x 2 MMAs (M 128, K 8): Q big against K big over
//    K small (N 128, the two boxes adjacent in shared memory) into
//    tensor-memory columns 0-127, Q small against K big (N 64) into 0-63;
//    S = columns 0-63 + columns 64-127;
//  * once S is complete each thread writes 32 keys of one dim of V, big and
//    small, into the transposed (128 dims x 64 keys, K-major) V tiles over
//    Q big; the two warpgroups load 32 columns each of their row of S
//    (tcgen05.ld: the warps of either group reach all 128 lanes), agree on
//    the row's max and sum in the log2 domain through shared memory and
//    write their half of P big / small into the K-major P tiles over Q
//    small.  (V as stored is an MN-major B operand; in the 128-byte swizzle
//    layout that kind::tf32 MMA wrote zeros on B200 whatever its leading /
//    stride offsets.)
//  * O = P V: 8 k-steps x 3 MMAs (M 128, N 128, K 8) into columns 128-255;
//    each warpgroup loads 64 columns of its rows of O and folds them into
//    registers (running max and sum of the row over the CTA's tiles).
// At the end the registers go through a swizzled staging tile (over V) and
// leave as 4 TMA tensor stores: the output rows when the CTA has all the
// keys, else the CTA's partial with (max, sum) per row beside it.
// combine_splits_kernel folds the splits' partials of every row.
constexpr int kURows = 128, kUKeys = 64;
constexpr int kUQBox = kURows * 128, kUKBox = kUKeys * 128;  // bytes of one Q / K (V) box
constexpr int kUVtBox = 128 * 128;                             // 128 dims x 32 keys of the transposed V
// Q big, Q small (64 KB each), K big / small (boxes interleaved) and raw V (32 KB each), barriers
constexpr int kUSmem = 1024 + 224 * 1024 + 64;  // 4 mbarriers + the tensor-memory address
static_assert(kUSmem <= 227 * 1024, "tcgen05 attention exceeds the shared memory of a CTA");

struct UmmaMaps {
    CUtensorMap q, k, v, part_o;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3fff) | ((uint64_t)((lbo >> 4) & 0x3fff) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46) /* sm100 descriptor */ |
           (2ull << 61) /* 128-byte swizzle */;
}

// c_format F32, a/b TF32, A K-major, B K- or MN-major, N, M = 128
__host__ __device__ constexpr uint32_t umma_idesc(int n, bool b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kURows >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tm_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
                 : "r"(taddr));
}

__device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}

__device__ __forceinline__ void umma_tma(uint32_t dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

// 2^x on the special-function unit (ex2.approx.ftz: 2^-inf = +0)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Tiled bulk tensor store shared -> global (completion through bulk groups).
__device__ __forceinline__ void umma_tma_store(const CUtensorMap *tm, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}

__global__ void __launch_bounds__(256, 1)
attention_umma_kernel(float2 *__restrict__ part_ml, int rows_pad, int seq_k, int tiles_per_split,
                      float scale_log2, const __grid_constant__ UmmaMaps maps) {
    extern __shared__ __align__(16) uint8_t usm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(usm_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_addr(sm);
    // K: box x (32 dims) of K big at k_base + 16 KB x, of K small 8 KB further:
    // one 128-row B operand of K big over K small per box
    const uint32_t q_big = base, q_small = base + 64 * 1024, k_base = base + 128 * 1024;
    const uint32_t v_raw = base + 192 * 1024;
    const uint32_t v_big = base, v_small = base + 32 * 1024;            // over Q big, once S is done
    const uint32_t p_big = base + 64 * 1024, p_small = base + 96 * 1024;  // over Q small
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 224 * 1024);      // K load, V load, MMAs, Q load
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 4);
    float *red = reinterpret_cast<float *>(sm + 136 * 1024);  // over K small's box 0, once S is done: max, sum
    const int warp = threadIdx.x >> 5, wg = threadIdx.x >> 7, row = threadIdx.x & 127;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;  // this warp's tensor-memory lanes
    const int row0 = blockIdx.x * kURows;
    const int tiles = (seq_k + kUKeys - 1) / kUKeys;
    const int t_begin = blockIdx.y * tiles_per_split, t_end = min(tiles, t_begin + tiles_per_split);
    // the combine (a dependent launch) may start its CTAs now; it waits for
    // this grid's completion before reading a partial
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // raw K (bars[0]) and V (bars[1]) of key tile t, raw Q (bars[3]): each
    // issued as soon as its region is free (the next tile's K once S is
    // done, its V once the transposed V and P are written, Q once O is done)
    auto load_k = [&](int t) {
        mbar_arrive_expect_tx(&bars[0], 4 * kUKBox);
        for (int x = 0; x < 4; ++x) umma_tma(k_base + x * 2 * kUKBox, &maps.k, 32 * x, t * kUKeys, &bars[0]);
    };
    auto load_v = [&](int t) {
        mbar_arrive_expect_tx(&bars[1], 4 * kUKBox);
        for (int x = 0; x < 4; ++x) umma_tma(v_raw + x * kUKBox, &maps.v, 32 * x, t * kUKeys, &bars[1]);
    };
    auto load_q = [&]() {
        mbar_arrive_expect_tx(&bars[3], 4 * kUQBox);
        for (int x = 0; x < 4; ++x) umma_tma(q_big + x * kUQBox, &maps.q, 32 * x, row0, &bars[3]);
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
        if (t_begin < t_end) {  // in flight during the tensor-memory allocation
            load_q();
            load_k(t_begin);
            load_v(t_begin);
        }
    }
    if (warp == 0) {  // 256 tensor-memory columns: S in two halves at 0-127, O at 128-255
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_addr(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot, t_s = tmem, t_o = tmem + 128;

    auto split16 = [](uint32_t raw, uint32_t dst_small) {
        float4 v;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "r"(raw));
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst_small), "f"(v.x - tf32_trunc(v.x)),
                     "f"(v.y - tf32_trunc(v.y)), "f"(v.z - tf32_trunc(v.z)), "f"(v.w - tf32_trunc(v.w))
                     : "memory");
    };

    // this thread's 64 columns (64 wg ..) of its row of the split's O, with
    // the running max and sum over the split's key tiles
    float acc[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    float M = -CUDART_INF_F, L = 0.f;

    for (int t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const int key0 = t * kUKeys;
        const uint32_t ph = it & 1;  // bars[0, 1, 3]: one phase per tile; bars[2]: two (S, then O)
        const bool more = t + 1 < t_end;

        // Q small and K small at the raw copies' offsets in their own regions
        (void)mbar_wait_bounded(&bars[3], ph, nullptr);
        (void)mbar_wait_bounded(&bars[0], ph, nullptr);
#pragma unroll 4
        for (int i = threadIdx.x; i < 4 * kUQBox / 16; i += 256) split16(q_big + 16 * i, q_small + 16 * i);
#pragma unroll 4
        for (int i = threadIdx.x; i < 4 * kUKBox / 16; i += 256) {  // box i / 512, 16-byte chunk i % 512
            const uint32_t src = k_base + (i >> 9) * 2 * kUKBox + (i & 511) * 16;
            split16(src, src + kUKBox);
        }
        fence_proxy_async_smem();  // the split's generic stores before the tensor core's reads
        tc_fence_before();
        __syncthreads();

        if (threadIdx.x == 0) {
            tc_fence_after();
            // S = Q K^T: k-step k reads 8 dims = 32 bytes of box k / 4.  Q big
            // against K big over K small (N 128: Qb.Kb into columns 0-63,
            // Qb.Ks into 64-127), then Q small against K big into 0-63; S is
            // the sum of the two column halves.
            constexpr uint32_t idesc128 = umma_idesc(2 * kUKeys, false), idesc64 = umma_idesc(kUKeys, false);
            for (int k = 0; k < 16; ++k) {
                const uint32_t ao = (k >> 2) * kUQBox + (k & 3) * 32, bo = (k >> 2) * 2 * kUKBox + (k & 3) * 32;
                const uint64_t ab = umma_desc(q_big + ao, 16, 1024), as = umma_desc(q_small + ao, 16, 1024);
                const uint64_t bk = umma_desc(k_base + bo, 16, 1024);
                umma_tf32(t_s, ab, bk, idesc128, k > 0);
                umma_tf32(t_s, as, bk, idesc64, 1);
            }
            umma_commit(&bars[2]);
        }
        (void)mbar_wait_bounded(&bars[2], 0, nullptr);  // S complete, Q and K free
        if (threadIdx.x == 0 && more) load_k(t + 1);
        __syncwarp();  // warp 0's thread 0 issued the MMAs: reconverge before the aligned loads
        tc_fence_after();

        // V^T big / small, this thread's dim d = row, keys 32 wg .. 32 wg + 31:
        // key j of raw V sits in box d / 32, row j, 16-byte chunk
        // ((d % 32) / 4) ^ (j % 8); the transposed element (d, j) in box j / 32,
        // row d, chunk ((j % 32) / 4) ^ (d % 8).
        (void)mbar_wait_bounded(&bars[1], ph, nullptr);
        {
            const int d = row;
            const uint32_t src = v_raw + (d >> 5) * kUKBox + (d & 3) * 4;
#pragma unroll 4
            for (int c = 8 * wg; c < 8 * wg + 8; ++c) {  // keys 4c .. 4c+3
                float x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * c + e;
                    asm volatile("ld.shared.f32 %0, [%1];"
                                 : "=f"(x[e])
                                 : "r"(src + j * 128 + ((((d & 31) >> 2) ^ (j & 7)) << 4)));
                }
                const uint32_t off = (c >> 3) * kUVtBox + d * 128 + (((c & 7) ^ (d & 7)) << 4);
                asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(v_big + off), "f"(x[0]), "f"(x[1]),
                             "f"(x[2]), "f"(x[3])
                             : "memory");
                asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(v_small + off),
                             "f"(x[0] - tf32_trunc(x[0])), "f"(x[1] - tf32_trunc(x[1])), "f"(x[2] - tf32_trunc(x[2])),
                             "f"(x[3] - tf32_trunc(x[3]))
                             : "memory");
            }
        }
        // this warpgroup's 32 keys of the thread's row of S (sum of the halves)
        uint32_t r[32], r2[32];
        tm_ld32(t_s + 32 * wg + lane_base, r);
        tm_ld32(t_s + 64 + 32 * wg + lane_base, r2);
        tm_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(r2[j]));
        const int nk = min(kUKeys, seq_k - key0) - 32 * wg;
        float m = -CUDART_INF_F;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float s = j < nk ? __uint_as_float(r[j]) * scale_log2 : -CUDART_INF_F;
            r[j] = __float_as_uint(s);
            m = fmaxf(m, s);
        }
        red[wg * 128 + row] = m;
        __syncthreads();
        m = fmaxf(red[row], red[128 + row]);  // finite: key key0 is valid
        float l = 0.f;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {  // keys 32 wg + 4cc .. +3: box wg, 16-byte chunk cc
            float p4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                p4[e] = ex2_approx(__uint_as_float(r[4 * cc + e]) - m);  // masked keys: -inf - m
                l += p4[e];
            }
            const uint32_t off = wg * kUQBox + row * 128 + (((cc ^ (row & 7))) << 4);
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(p_big + off), "f"(p4[0]), "f"(p4[1]),
                         "f"(p4[2]), "f"(p4[3])
                         : "memory");
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(p_small + off),
                         "f"(p4[0] - tf32_trunc(p4[0])), "f"(p4[1] - tf32_trunc(p4[1])),
                         "f"(p4[2] - tf32_trunc(p4[2])), "f"(p4[3] - tf32_trunc(p4[3]))
                         : "memory");
        }
        red[256 + wg * 128 + row] = l;
        fence_proxy_async_smem();  // P's generic stores before the tensor core's reads
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x == 0) {
            tc_fence_after();
            // O = P V: k-step k reads 8 keys (32 bytes of box k / 4) of P and of
            // the transposed V
            constexpr uint32_t idesc = umma_idesc(128, false);
            for (int k = 0; k < 8; ++k) {
                const uint32_t ao = (k >> 2) * kUQBox + (k & 3) * 32, vo = (k >> 2) * kUVtBox + (k & 3) * 32;
                const uint64_t ab = umma_desc(p_big + ao, 16, 1024), as = umma_desc(p_small + ao, 16, 1024);
                const uint64_t bb = umma_desc(v_big + vo, 16, 1024), bs = umma_desc(v_small + vo, 16, 1024);
                umma_tf32(t_o, ab, bb, idesc, k > 0);
                umma_tf32(t_o, ab, bs, idesc, 1);
                umma_tf32(t_o, as, bb, idesc, 1);
            }
            umma_commit(&bars[2]);
            if (more) load_v(t + 1);  // every thread is past its reads of the raw V
        }
        (void)mbar_wait_bounded(&bars[2], 1, nullptr);
        if (threadIdx.x == 0 && more) load_q();  // the MMAs are done with Q's space (transposed V, P)
        __syncwarp();
        tc_fence_after();
        // fold the tile into the running (M, L, acc) of the thread's row
        {
            const float mn = fmaxf(M, m);
            const float a = ex2_approx(M - mn), w = ex2_approx(m - mn);  // M = -inf on the first tile: a = 0
            L = L * a + (red[256 + row] + red[384 + row]) * w;
            M = mn;
            uint32_t o[64];
            tm_ld64(t_o + 64 * wg + lane_base, o);
            tm_wait_ld();
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] = acc[j] * a + __uint_as_float(o[j]) * w;
        }
        // every thread's reads of this tile's red and tensor memory are done
        // before the next tile's split and MMAs
        tc_fence_before();
        __syncthreads();
    }

    // the split's result into staging boxes 2 wg, 2 wg + 1 (32 columns x 128
    // rows each, 128-byte swizzle) over V: O itself with (M, L) beside it
    // when the keys are split over several CTAs, else O / L, the output rows
    const bool direct = gridDim.y == 1;
    const float inv = direct ? 1.f / L : 1.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const uint32_t off = (2 * wg + (c >> 3)) * kUVtBox + row * 128 + (((c & 7) ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(base + off), "f"(acc[4 * c] * inv),
                     "f"(acc[4 * c + 1] * inv), "f"(acc[4 * c + 2] * inv), "f"(acc[4 * c + 3] * inv)
                     : "memory");
    }
    const int prow0 = direct ? row0 : blockIdx.y * rows_pad + row0;
    if (!direct && wg == 0) part_ml[(size_t)prow0 + row] = make_float2(M, L);
    fence_proxy_async_smem();  // the staging stores before the bulk copy's reads
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // rows past the output's end (direct) are not written by the copy
        for (int x = 0; x < 4; ++x) umma_tma_store(&maps.part_o, 32 * x, prow0, base + x * kUVtBox);
        bulk_commit();
        bulk_wait_read_all();  // the staging tile stays until the copy has read it
    }
    __syncwarp();  // thread 0 rejoins its warp before the aligned dealloc
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
}

// out[row] = sum_t exp2(m_t - M) O_t / sum_t exp2(m_t - M) L_t over the key
// splits t; one warp per row, a float4 of dims per lane.  Splits go in
// batches of 16 with a running max: a batch's (max, sum) pairs (lane j holds
// split j's) and its 16 partial rows are all loaded before any is used, so a
// batch costs one memory round trip.  Launched as a programmatic dependent
// of the attention grid: it waits for that grid's completion first.
__global__ void combine_splits_kernel(const float *__restrict__ part_o, const float2 *__restrict__ part_ml,
                                      float *__restrict__ out, int seq_q, int rows_pad, int nsplit) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= seq_q) return;
    float M = -CUDART_INF_F, L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t0 = 0; t0 < nsplit; t0 += 16) {
        const int cnt = min(16, nsplit - t0);
        float2 ml = make_float2(-CUDART_INF_F, 0.f);
        if (lane < cnt) ml = part_ml[(size_t)(t0 + lane) * rows_pad + row];
        // all 16 loads issued here (volatile: not sunk to their uses); tiles
        // past the batch re-read its first tile and get weight 0
        float4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const float *src = part_o + ((size_t)(t0 + (u < cnt ? u : 0)) * rows_pad + row) * 128 + 4 * lane;
            asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(v[u].x), "=f"(v[u].y), "=f"(v[u].z), "=f"(v[u].w)
                         : "l"(src));
        }
        float mb = ml.x;
#pragma unroll
        for (int o = 16; o; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        const float Mn = fmaxf(M, mb);  // finite: every tile has a valid key
        const float a = M == -CUDART_INF_F ? 0.f : exp2f(M - Mn);
        const float w = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - Mn);
        float lb = w * ml.y;
#pragma unroll
        for (int o = 16; o; o >>= 1) lb += __shfl_xor_sync(0xffffffffu, lb, o);
        L = L * a + lb;
        acc = make_float4(acc.x * a, acc.y * a, acc.z * a, acc.w * a);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const float wu = __shfl_sync(0xffffffffu, w, u);
            acc.x += wu * v[u].x, acc.y += wu * v[u].y, acc.z += wu * v[u].z, acc.w += wu * v[u].w;
        }
        M = Mn;
    }
    if (L == 0.f) L = 1e-6f;  // TensorOps::softmax's guard
    reinterpret_cast<float4 *>(out + (size_t)row * 128)[lane] =
        make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
using EncodeTiledFnD = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// fp32 rows of `cols` floats (a multiple of 32), boxes of box_rows rows x 32
// floats, 128-byte swizzle, zero fill past the last row.
bool make_map_f32(CUtensorMap *tm, const float *base, long long rows, int box_rows, long long cols = 128) {
    static EncodeTiledFnD fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFnD>(f);
    });
    if (!fn || rows <= 0 || rows > (1ll << 31) || cols <= 0 || cols % 32 || cols > (1ll << 31)) return false;
    cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), gdim, gstride, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The library's stream-ordered scratch pool on device `dev` (made once, kept
// for the process): freed blocks stay in the pool (release threshold at its
// maximum), so a call after the first allocates no device memory.  A pool
// of its own leaves the device's default pool as the application set it.
cudaMemPool_t scratch_pool(int dev) {
    static std::mutex mu;
    static cudaMemPool_t pools[kMaxDevices] = {};
    std::lock_guard<std::mutex> lk(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t p = nullptr;
        if (cudaMemPoolCreate(&p, &props) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        uint64_t keep = ~0ull;
        cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
        pools[dev] = p;
    }
    return pools[dev];
}

// The tcgen05 path.  Key tiles split over CTAs only as far as the row tiles
// leave SMs idle (one CTA per SM: floor(SMs / row tiles) splits, at most one
// per tile); each CTA folds its tiles in registers.  One split: the CTAs
// write the output rows themselves.  Several: their partials go to
// stream-ordered scratch (scratch_pool; at most about SMs x 128 rows of
// partials, whatever the sequence lengths), the combine folds them, the
// scratch is released in stream order.
int attention_umma(const float *Q, const float *K, const float *V, float *out, int seq_q, int seq_k, float s,
                   cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KVX_ECUDA;
    static std::atomic<bool> attr_done[kMaxDevices];
    if (ensure_smem_attr(attr_done, attention_umma_kernel, kUSmem) != KVX_OK) return KVX_ECUDA;
    const long long row_tiles = ((long long)seq_q + kURows - 1) / kURows, rows_pad = row_tiles * kURows;
    const long long tiles = ((long long)seq_k + kUKeys - 1) / kUKeys;
    if (row_tiles > 0x7fffffffLL) return KVX_EUNSUPPORTED;
    long long nsplit = std::min<long long>(tiles, std::max<long long>(1, sm_count() / row_tiles));
    const long long per = (tiles + nsplit - 1) / nsplit;
    nsplit = (tiles + per - 1) / per;
    const float scale_log2 = s * 1.4426950408889634f;
    UmmaMaps maps;
    if (!(make_map_f32(&maps.q, Q, seq_q, kURows) && make_map_f32(&maps.k, K, seq_k, kUKeys) &&
          make_map_f32(&maps.v, V, seq_k, kUKeys)))
        return KVX_ECUDA;
    const dim3 grid((unsigned)row_tiles, (unsigned)nsplit);
    if (nsplit == 1) {
        if (!make_map_f32(&maps.part_o, out, seq_q, kURows)) return KVX_ECUDA;
        attention_umma_kernel<<<grid, 256, kUSmem, st>>>(nullptr, (int)rows_pad, seq_k, (int)per, scale_log2, maps);
        return launch_status();
    }
    cudaMemPool_t pool = scratch_pool(dev);
    if (!pool) return KVX_ECUDA;
    const size_t pb = (size_t)nsplit * rows_pad * 512, mb = (size_t)nsplit * rows_pad * 8;
    uint8_t *w = nullptr;
    if (cudaMallocFromPoolAsync(reinterpret_cast<void **>(&w), pb + mb, pool, st) != cudaSuccess) {
        cudaGetLastError();
        return KVX_ENOSPC;
    }
    float *po = reinterpret_cast<float *>(w);
    float2 *pml = reinterpret_cast<float2 *>(w + pb);
    int rc = make_map_f32(&maps.part_o, po, nsplit * rows_pad, kURows) ? KVX_OK : KVX_ECUDA;
    if (rc == KVX_OK) {
        attention_umma_kernel<<<grid, 256, kUSmem, st>>>(pml, (int)rows_pad, seq_k, (int)per, scale_log2, maps);
        rc = launch_status();
    }
    if (rc == KVX_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((seq_q * 32LL + 255) / 256));
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, combine_splits_kernel, (const float *)po, (const float2 *)pml, out, seq_q,
                               (int)rows_pad, (int)nsplit) != cudaSuccess) {
            cudaGetLastError();
            rc = KVX_ECUDA;
        }
    }
    if (cudaFreeAsync(w, st) != cudaSuccess && rc == KVX_OK) rc = KVX_ECUDA;
    return rc;
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
        return attention_umma(Q, K, V, out, (int)seq_q, (int)seq_k, s, static_cast<cudaStream_t>(stream));
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
