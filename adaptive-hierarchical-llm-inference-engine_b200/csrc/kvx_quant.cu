// kvx_quant.cu -- the reference's KV codecs as vectorised sm_100a kernels.
//
//  * int8 per-block quantisation, bit-exact with KVCompressionEngine::
//    compressToINT8 / decompressINT8
//    (native-engine/cpp/KVCompressionEngine.cpp:83-122).  One warp per block
//    (2048 elements = one (page, K|V, head) block at 16 x 128), 16-byte
//    loads, the block held in registers between the min/max pass and the
//    quantise pass, 16-byte code stores.
//  * NF4 (uniform 4-bit) per-block quantisation, bit-exact with
//    compressToNF4 / decompressNF4 (KVCompressionEngine.cpp:124-180): the
//    same pipeline with 15 levels and two codes per byte (high nibble
//    first).
//  * the truncating fp32<->fp16 converter of the disk tier, bit-exact with
//    float_to_half / half_to_float (compression/kv_compress.cpp:6-46), and
//    the engine's own exponent-wrapping FP16 codec (compressToFP16 /
//    decompressFP16, KVCompressionEngine.cpp:36-80).
//
// Bit-exactness notes.  The reference is plain x86-64 SSE fp32 without FMA,
// so every step here uses the explicitly rounded intrinsics (__fsub_rn,
// __fdiv_rn, __fmul_rn, __fadd_rn) that the compiler cannot contract.
//  - min/max: the reference keeps the FIRST element that compares smallest
//    (largest) in index order; only +0/-0 compare equal with different bits,
//    so the reduction carries (value, index) and breaks ties on the index.
//    A NaN first element makes min and max NaN; later NaNs are never taken.
//  - (int32_t)std::round(x): roundf, then x86 cvttss2si, which yields
//    INT32_MIN for NaN and out-of-range values (clamped to code -128).
#include <cuda_fp16.h>
#include <math_constants.h>

#include <map>
#include <mutex>
#include <utility>

#include "kvx_common.cuh"

namespace kvx {
namespace {

__device__ __forceinline__ int32_t cvt_trunc_i32_x86(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT32_MIN;
    return (int32_t)r;
}

// x86 SSE NaN rules for a binary op r = a op b: a NaN operand is returned
// quieted (the first one if both are NaN); an invalid operation on non-NaN
// operands (0*inf, inf-inf, 0/0) returns the default NaN 0xFFC00000.  The
// GPU returns the canonical 0x7FFFFFFF instead, so NaN results are rebuilt.
__device__ __forceinline__ float x86_nan(float r, float a, float b) {
    if (r == r) return r;
    if (a != a) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (b != b) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xFFC00000u);
}

// clamp((int)std::round((x - mn) / scale), 0, kLevels) with the reference's
// rounding and x86 conversion.
template <int kLevels>
__device__ __forceinline__ int32_t quant_level(float x, float mn, float scale) {
    const float normalized = __fdiv_rn(__fsub_rn(x, mn), scale);
    int32_t q = cvt_trunc_i32_x86(roundf(normalized));
    return q < 0 ? 0 : (q > kLevels ? kLevels : q);
}

__device__ __forceinline__ int8_t quant_one(float x, float mn, float scale) {
    return (int8_t)(quant_level<255>(x, mn, scale) - 128);
}

// (value, index) candidates in index order; strict comparisons keep the
// first occurrence, exactly as std::min / std::max over a forward loop.
struct MinMax {
    float mn, mx;
    int imn, imx;
};

__device__ __forceinline__ void mm_take(MinMax &a, float v, int i) {
    if (v != v) return;  // NaN never replaces (first element handled apart)
    if (v < a.mn || (v == a.mn && i < a.imn)) { a.mn = v; a.imn = i; }
    if (a.mx < v || (v == a.mx && i < a.imx)) { a.mx = v; a.imx = i; }
}

__device__ __forceinline__ MinMax mm_warp_reduce(MinMax a) {
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const float mn = __shfl_xor_sync(0xffffffffu, a.mn, off);
        const int imn = __shfl_xor_sync(0xffffffffu, a.imn, off);
        const float mx = __shfl_xor_sync(0xffffffffu, a.mx, off);
        const int imx = __shfl_xor_sync(0xffffffffu, a.imx, off);
        if (mn < a.mn || (mn == a.mn && imn < a.imn)) { a.mn = mn; a.imn = imn; }
        if (a.mx < mx || (mx == a.mx && imx < a.imx)) { a.mx = mx; a.imx = imx; }
    }
    return a;
}

template <typename T> __device__ __forceinline__ float ld_elem(const T *p, size_t i);
template <> __device__ __forceinline__ float ld_elem<float>(const float *p, size_t i) { return p[i]; }
// fp16 -> fp32 widening, exact; NaNs keep their payload with the quiet bit
// set (as x86 F16C / gcc's _Float16 conversion does).
template <> __device__ __forceinline__ float ld_elem<__half>(const __half *p, size_t i) {
    const uint16_t h = __half_as_ushort(p[i]);
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu))
        return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7FC00000u | ((uint32_t)(h & 0x3FFu) << 13));
    return __half2float(p[i]);
}

// Finish stats from the reduced min/max; writes stats[4] from lane 0.
template <int kLevels>
__device__ __forceinline__ void finish_stats(MinMax r, float first, float *stats, int lane,
                                             float &mn, float &scale) {
    if (first != first) {  // NaN first element: the reference keeps NaN
        r.mn = first;
        r.mx = first;
    }
    mn = r.mn;
    const float range = x86_nan(__fsub_rn(r.mx, r.mn), r.mx, r.mn);
    float sc = x86_nan(__fdiv_rn(range, (float)kLevels), range, (float)kLevels);
    if (sc == 0.0f) sc = 1.0f;
    scale = sc;
    if (lane == 0) *reinterpret_cast<float4 *>(stats) = make_float4(r.mn, r.mx, sc, r.mn);
}

// Plain widening for the shortcut (a NaN only has to stay NaN there).
template <typename T> __device__ __forceinline__ float ld_raw(const T *p, int i);
template <> __device__ __forceinline__ float ld_raw<float>(const float *p, int i) { return p[i]; }
template <> __device__ __forceinline__ float ld_raw<__half>(const __half *p, int i) { return __half2float(p[i]); }

// Distance from a half-integer below which the reciprocal shortcut defers to
// the exact division.  For a finite block every quotient is <= 255 * (1 +
// 2^-23); t = RN(RN(x - mn) * RN(1/scale)) is then within 255 * 2^-23 <
// 3.1e-5 of (x - mn) / scale and RN((x - mn) / scale) within 2^-17 < 7.7e-6
// of it, so when |t - rint(t)| <= 0.5 - 4e-5 both round to rint(t).
constexpr float kTieLimit = 0.5f - 4.0e-5f;
constexpr float kTwo23 = 8388608.0f;  // t + 2^23: rint(t) in the low mantissa bits

__device__ __forceinline__ float max_nan(float a, float b) {  // NaN wins
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Fast path: 2048-element blocks, 16-byte vectors, block kept in registers.
// min / max first by value alone (fp16 pairs for fp16 input), NaN-skipping;
// only when a result is +-0 -- the one tie whose bits differ -- does a
// second pass pick the first such element in index order.  Codes come from
// the reciprocal shortcut above; a lane holding a near-tie or a NaN then
// rewrites those codes with the exact division (quant_one).
template <typename T, int kLevels>
__global__ void __launch_bounds__(256)
compress_2048_kernel(const T *__restrict__ src, uint8_t *__restrict__ codes,
                     float *__restrict__ stats, size_t num_blocks) {
    constexpr bool kNf4 = kLevels == 15;
    constexpr int kCodeBytes = kNf4 ? 1024 : 2048;  // code bytes per block
    constexpr int kBlock = 2048;
    constexpr int kPerVec = 16 / sizeof(T);             // elements per 16-byte load
    constexpr int kVecs = kBlock / kPerVec / 32;        // loads per lane
    const int lane = threadIdx.x & 31;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t b = blockIdx.x * (size_t)(blockDim.x >> 5) + (threadIdx.x >> 5); b < num_blocks;
         b += warps) {
        const T *in = src + b * kBlock;
        uint4 w[kVecs];
#pragma unroll
        for (int j = 0; j < kVecs; ++j)
            w[j] = __ldcs(reinterpret_cast<const uint4 *>(in) + j * 32 + lane);
        float mn, mx;
        if constexpr (sizeof(T) == 2) {
            __half2 lo = reinterpret_cast<const __half2 *>(&w[0])[0], hi = lo;
#pragma unroll
            for (int j = 0; j < kVecs; ++j) {
                const __half2 *h = reinterpret_cast<const __half2 *>(&w[j]);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    lo = __hmin2(lo, h[k]);
                    hi = __hmax2(hi, h[k]);
                }
            }
            mn = fminf(__low2float(lo), __high2float(lo));
            mx = fmaxf(__low2float(hi), __high2float(hi));
        } else {
            mn = CUDART_INF_F;
            mx = -CUDART_INF_F;
#pragma unroll
            for (int j = 0; j < kVecs; ++j) {
                const float *e = reinterpret_cast<const float *>(&w[j]);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    mn = fminf(mn, e[k]);
                    mx = fmaxf(mx, e[k]);
                }
            }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        }
        const float first = ld_elem<T>(in, 0);
        MinMax a{mn, mx, 0, 0};
        if (mn != mn) {  // every element NaN: the reference keeps in[0]
            a.mn = a.mx = first;
        } else if (mn == 0.f || mx == 0.f) {  // +-0 ties: first in index order
            MinMax z{CUDART_INF_F, -CUDART_INF_F, 1 << 30, 1 << 30};
#pragma unroll 1
            for (int i = lane; i < kBlock; i += 32) mm_take(z, ld_elem<T>(in, i), i);
            a = mm_warp_reduce(z);
        }
        float mnv, scale;
        finish_stats<kLevels>(a, first, stats + 4 * b, lane, mnv, scale);
        const float rcp = __frcp_rn(scale);
        uint8_t *out = codes + b * kCodeBytes;
        if (isfinite(scale) && isfinite(rcp)) {  // warp-uniform; mn, mx finite too
            uint32_t bad = 0;  // vectors holding a near-tie or a NaN
#pragma unroll
            for (int j = 0; j < kVecs; ++j) {
                const T *e = reinterpret_cast<const T *>(&w[j]);
                uint32_t word[kPerVec / 4];
                float worst = 0.f;
#pragma unroll
                for (int k4 = 0; k4 < kPerVec / 4; ++k4) {
                    uint32_t u[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float t = __fmul_rn(__fsub_rn(ld_raw<T>(e, 4 * k4 + k), mnv), rcp);
                        const float s = __fadd_rn(t, kTwo23);
                        worst = max_nan(worst, fabsf(__fsub_rn(t, __fsub_rn(s, kTwo23))));
                        u[k] = __float_as_uint(s);
                    }
                    if constexpr (kNf4)  // 2 bytes: (q0 << 4 | q1), (q2 << 4 | q3)
                        word[k4] = ((u[0] & 0xFu) << 4) | (u[1] & 0xFu) | ((u[2] & 0xFu) << 12) |
                                   ((u[3] & 0xFu) << 8);
                    else
                        word[k4] = __byte_perm(__byte_perm(u[0], u[1], 0x0040),
                                               __byte_perm(u[2], u[3], 0x0040), 0x5410) ^ 0x80808080u;
                }
                if (!(worst <= kTieLimit)) bad |= 1u << j;
                if constexpr (kNf4) {
                    if constexpr (kPerVec == 8)
                        __stcs(reinterpret_cast<uint32_t *>(out) + j * 32 + lane, word[0] | (word[1] << 16));
                    else
                        __stcs(reinterpret_cast<unsigned short *>(out) + j * 32 + lane, (unsigned short)word[0]);
                } else {
                    if constexpr (kPerVec == 8)
                        __stcs(reinterpret_cast<uint2 *>(out) + j * 32 + lane, make_uint2(word[0], word[1]));
                    else
                        __stcs(reinterpret_cast<uint32_t *>(out) + j * 32 + lane, word[0]);
                }
            }
            // rare: redo the flagged vectors' codes with the exact division
            // (x re-read from global, no indexed register array)
#pragma unroll 1
            while (bad) {
                const int j = __ffs(bad) - 1;
                bad &= bad - 1;
                {
                    const int base = (j * 32 + lane) * kPerVec;
                    if constexpr (kNf4) {  // redo the lane's bytes exactly (two codes each)
#pragma unroll 1
                        for (int k = 0; k < kPerVec; k += 2)
                            out[(base + k) / 2] = (uint8_t)((quant_level<15>(ld_elem<T>(in, base + k), mnv, scale) << 4) |
                                                            quant_level<15>(ld_elem<T>(in, base + k + 1), mnv, scale));
                    } else {
#pragma unroll 1
                        for (int k = 0; k < kPerVec; ++k) {
                            const float x = ld_elem<T>(in, base + k);
                            const float t = __fmul_rn(__fsub_rn(x, mnv), rcp);
                            if (!(fabsf(__fsub_rn(t, rintf(t))) <= kTieLimit))
                                out[base + k] = (uint8_t)quant_one(x, mnv, scale);
                        }
                    }
                }
            }
        } else {  // inf / NaN range or denormal scale: exact division throughout
            if constexpr (kNf4) {
#pragma unroll 1
                for (int i = lane; i < kBlock / 2; i += 32)
                    out[i] = (uint8_t)((quant_level<15>(ld_elem<T>(in, 2 * i), mnv, scale) << 4) |
                                       quant_level<15>(ld_elem<T>(in, 2 * i + 1), mnv, scale));
            } else {
#pragma unroll 1
                for (int i = lane; i < kBlock; i += 32) out[i] = (uint8_t)quant_one(ld_elem<T>(in, i), mnv, scale);
            }
        }
    }
}

// Generic path: any block size, one warp per block, two passes over global.
template <typename T, int kLevels>
__global__ void __launch_bounds__(256)
compress_generic_kernel(const T *__restrict__ src, uint8_t *__restrict__ codes,
                        float *__restrict__ stats, size_t num_blocks, int block_elems) {
    const int lane = threadIdx.x & 31;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t b = blockIdx.x * (size_t)(blockDim.x >> 5) + (threadIdx.x >> 5); b < num_blocks;
         b += warps) {
        const T *in = src + b * (size_t)block_elems;
        MinMax a{CUDART_INF_F, -CUDART_INF_F, 1 << 30, 1 << 30};
        for (int i = lane; i < block_elems; i += 32) mm_take(a, ld_elem<T>(in, i), i);
        const float first = ld_elem<T>(in, 0);
        a = mm_warp_reduce(a);
        if (a.imn == (1 << 30)) a.mn = first;
        if (a.imx == (1 << 30)) a.mx = first;
        float mn, scale;
        finish_stats<kLevels>(a, first, stats + 4 * b, lane, mn, scale);
        if constexpr (kLevels == 15) {  // two codes per byte, high nibble first; odd tail -> 0
            const int nb = (block_elems + 1) / 2;
            uint8_t *out = codes + b * (size_t)nb;
            for (int i = lane; i < nb; i += 32) {
                const int32_t q1 = quant_level<15>(ld_elem<T>(in, 2 * i), mn, scale);
                const int32_t q2 = 2 * i + 1 < block_elems ? quant_level<15>(ld_elem<T>(in, 2 * i + 1), mn, scale) : 0;
                out[i] = (uint8_t)((q1 << 4) | q2);
            }
        } else {
            uint8_t *out = codes + b * (size_t)block_elems;
            for (int i = lane; i < block_elems; i += 32) out[i] = (uint8_t)quant_one(ld_elem<T>(in, i), mn, scale);
        }
    }
}

__device__ __forceinline__ float dequant_one(int8_t c, float zp, float scale) {
    const float q = (float)((int32_t)c + 128);
    const float m = x86_nan(__fmul_rn(q, scale), q, scale);
    return x86_nan(__fadd_rn(zp, m), zp, m);
}

// fp32 value of byte k of w, exactly: the bytes {b, 0, 0, 0x4B} are the
// float 2^23 + b, and subtracting 2^23 is exact (no conversion instruction).
__device__ __forceinline__ float byte_value(uint32_t w, int k) {
    return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)k)), 8388608.0f);
}

template <typename T> __device__ __forceinline__ void store16(T *dst, const float (&v)[16]);
template <> __device__ __forceinline__ void store16<float>(float *dst, const float (&v)[16]) {
    float4 *o = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int k = 0; k < 4; ++k) __stcs(o + k, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
}
template <> __device__ __forceinline__ void store16<__half>(__half *dst, const float (&v)[16]) {
    uint32_t u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        u[k] = *reinterpret_cast<const uint32_t *>(&h);
    }
    __stcs(reinterpret_cast<uint4 *>(dst), make_uint4(u[0], u[1], u[2], u[3]));
    __stcs(reinterpret_cast<uint4 *>(dst) + 1, make_uint4(u[4], u[5], u[6], u[7]));
}

// The same 16 values into a shared-memory image of the block.
template <typename T> __device__ __forceinline__ void store16_shared(T *dst, const float (&v)[16]);
template <> __device__ __forceinline__ void store16_shared<float>(float *dst, const float (&v)[16]) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
        reinterpret_cast<float4 *>(dst)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}
template <> __device__ __forceinline__ void store16_shared<__half>(__half *dst, const float (&v)[16]) {
    uint32_t u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        u[k] = *reinterpret_cast<const uint32_t *>(&h);
    }
    reinterpret_cast<uint4 *>(dst)[0] = make_uint4(u[0], u[1], u[2], u[3]);
    reinterpret_cast<uint4 *>(dst)[1] = make_uint4(u[4], u[5], u[6], u[7]);
}

// Decoders write a block's output (4 KiB fp16 / 8 KiB fp32) into a
// per-warp shared-memory image and send it with one bulk copy: one TMA
// operation per block instead of 256 16-byte stores, which had the store
// queue throttling the warps.  32 KiB of images per CTA.
template <typename T> constexpr int kDqWarps = sizeof(T) == 2 ? 8 : 4;

// Warp per 2048-element block: stats read once, 16 codes per lane-load.
// Finite scale and zero point (every block the quantiser writes from finite
// data): zp + u * scale with u taken from the code byte exactly; otherwise
// the x86 NaN rebuild, element by element, in a loop kept out of line.
template <typename T>
__global__ void __launch_bounds__(kDqWarps<T> * 32)
decompress_2048_kernel(const int8_t *__restrict__ codes, const float *__restrict__ stats,
                       T *__restrict__ dst, size_t num_blocks) {
    __shared__ __align__(128) T image[kDqWarps<T>][2048];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T *img = image[warp];
    bool sent = false;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t b = blockIdx.x * (size_t)(blockDim.x >> 5) + warp; b < num_blocks; b += warps) {
        const float4 st = __ldg(reinterpret_cast<const float4 *>(stats) + b);
        const float scale = st.z, zp = st.w;
        const uint4 *src = reinterpret_cast<const uint4 *>(codes + b * 2048);
        uint4 w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = __ldcs(src + j * 32 + lane);
        if (isfinite(scale) && isfinite(zp)) {  // warp-uniform
            if (sent) {  // the previous block's copy has read the image
                if (lane == 0) bulk_wait_read_all();
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // 4 x 16 codes per lane
                const uint32_t u[4] = {w[j].x ^ 0x80808080u, w[j].y ^ 0x80808080u, w[j].z ^ 0x80808080u,
                                       w[j].w ^ 0x80808080u};  // c + 128
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = __fadd_rn(zp, __fmul_rn(byte_value(u[k >> 2], k & 3), scale));
                store16_shared<T>(img + (j * 32 + lane) * 16, v);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_s2g(dst + (size_t)b * 2048, img, 2048 * sizeof(T));
                bulk_commit();
            }
            sent = true;
        } else {  // rare: codes re-read from global, no indexed register array
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                const int8_t *c = codes + b * 2048 + (size_t)(j * 32 + lane) * 16;
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = dequant_one(c[k], zp, scale);
                store16<T>(dst + (size_t)b * 2048 + (size_t)(j * 32 + lane) * 16, v);
            }
        }
    }
    if (sent && lane == 0) bulk_wait_all();  // the images stay until the copies are done
}

// Any block size or alignment: one thread per element.
template <typename T>
__global__ void decompress_scalar_kernel(const int8_t *__restrict__ codes, const float *__restrict__ stats,
                                         T *__restrict__ dst, size_t num_blocks, int block_elems) {
    const size_t n = num_blocks * (size_t)block_elems;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const size_t b = e / (size_t)block_elems;
        const float v = dequant_one(codes[e], stats[4 * b + 3], stats[4 * b + 2]);
        if constexpr (sizeof(T) == 4)
            dst[e] = v;
        else
            dst[e] = __float2half_rn(v);
    }
}

// One thread per 4 codes; block_elems % 4 == 0.
template <typename T>
__global__ void __launch_bounds__(256)
decompress_kernel(const int8_t *__restrict__ codes, const float *__restrict__ stats,
                  T *__restrict__ dst, size_t num_blocks, int block_elems) {
    const size_t quads = num_blocks * (size_t)(block_elems / 4);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t e0 = i * 4;
        const size_t b = e0 / block_elems;
        const float4 st = __ldg(reinterpret_cast<const float4 *>(stats) + b);
        const uint32_t w = __ldcs(reinterpret_cast<const uint32_t *>(codes) + i);
        const int8_t *c = reinterpret_cast<const int8_t *>(&w);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = dequant_one(c[k], st.w, st.z);
        if constexpr (sizeof(T) == 4) {
            __stcs(reinterpret_cast<float4 *>(dst) + i, make_float4(v[0], v[1], v[2], v[3]));
        } else {
            __half2 a = __floats2half2_rn(v[0], v[1]), bb = __floats2half2_rn(v[2], v[3]);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t *>(&a);
            u.y = *reinterpret_cast<uint32_t *>(&bb);
            __stcs(reinterpret_cast<uint2 *>(dst) + i, u);
        }
    }
}

// ---- compression/kv_compress.cpp:6-46 ------------------------------------
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t mant = x & 0x007FFFFFu;
    const int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e > -15) return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | (mant >> 13));
    return (uint16_t)sign;
}

__device__ __forceinline__ float f16_trunc_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h & 0x7C00u) >> 10;
    const uint32_t mant = (uint32_t)h & 0x03FFu;
    uint32_t x;
    if (e == 0) x = sign;
    else if (e == 0x1F) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e - 15 + 127) << 23) | (mant << 13);
    return __uint_as_float(x);
}

// `vec`: both arrays 16 / 8-byte aligned, so four elements move per access;
// otherwise every element is handled on its own.
__global__ void __launch_bounds__(256)
encode_trunc_kernel(const float *__restrict__ src, uint16_t *__restrict__ dst, size_t n, bool vec) {
    const size_t quads = vec ? n / 4 : 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads; i += stride) {
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(src) + i);
        uint2 o;
        o.x = (uint32_t)f32_to_f16_trunc(v.x) | ((uint32_t)f32_to_f16_trunc(v.y) << 16);
        o.y = (uint32_t)f32_to_f16_trunc(v.z) | ((uint32_t)f32_to_f16_trunc(v.w) << 16);
        __stcs(reinterpret_cast<uint2 *>(dst) + i, o);
    }
    for (size_t i = quads * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = f32_to_f16_trunc(src[i]);
}

__global__ void __launch_bounds__(256)
decode_trunc_kernel(const uint16_t *__restrict__ src, float *__restrict__ dst, size_t n, bool vec) {
    const size_t quads = vec ? n / 4 : 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads; i += stride) {
        const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(src) + i);
        __stcs(reinterpret_cast<float4 *>(dst) + i,
               make_float4(f16_trunc_to_f32((uint16_t)v.x), f16_trunc_to_f32((uint16_t)(v.x >> 16)),
                           f16_trunc_to_f32((uint16_t)v.y), f16_trunc_to_f32((uint16_t)(v.y >> 16))));
    }
    for (size_t i = quads * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = f16_trunc_to_f32(src[i]);
}

__device__ __forceinline__ float dequant_level(uint32_t q, float zp, float scale) {
    const float qf = (float)q;
    const float m = x86_nan(__fmul_rn(qf, scale), qf, scale);
    return x86_nan(__fadd_rn(zp, m), zp, m);
}

template <typename T> __device__ __forceinline__ void st_out(T *p, float v);
template <> __device__ __forceinline__ void st_out<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void st_out<__half>(__half *p, float v) { *p = __float2half_rn(v); }

// NF4 decode, warp per 2048-element block: 1024 code bytes as two 16-byte
// loads per lane, 64 values out per lane.
template <typename T>
__global__ void __launch_bounds__(kDqWarps<T> * 32)
decompress_nf4_2048_kernel(const uint8_t *__restrict__ codes, const float *__restrict__ stats,
                           T *__restrict__ dst, size_t num_blocks) {
    __shared__ __align__(128) T image[kDqWarps<T>][2048];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T *img = image[warp];
    bool sent = false;
    const size_t warps = (size_t)gridDim.x * (blockDim.x >> 5);
    for (size_t b = blockIdx.x * (size_t)(blockDim.x >> 5) + warp; b < num_blocks; b += warps) {
        const float4 st = __ldg(reinterpret_cast<const float4 *>(stats) + b);
        const float scale = st.z, zp = st.w;
        const uint4 *src = reinterpret_cast<const uint4 *>(codes + b * 1024);
        uint4 w[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) w[j] = __ldcs(src + j * 32 + lane);
        if (isfinite(scale) && isfinite(zp)) {  // warp-uniform
            if (sent) {  // the previous block's copy has read the image
                if (lane == 0) bulk_wait_read_all();
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {  // 16 bytes = 32 codes per lane, high nibble first
                const uint32_t ww[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
                T *out = img + (j * 32 + lane) * 32;
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // bytes 8h .. 8h + 7 -> elements 16h .. 16h + 15
                    float v[16];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t word = ww[2 * h + (k >> 2)];
                        const uint32_t hi = (word >> 4) & 0x0F0F0F0Fu, lo = word & 0x0F0F0F0Fu;
                        v[2 * k] = __fadd_rn(zp, __fmul_rn(byte_value(hi, k & 3), scale));
                        v[2 * k + 1] = __fadd_rn(zp, __fmul_rn(byte_value(lo, k & 3), scale));
                    }
                    store16_shared<T>(out + 16 * h, v);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_s2g(dst + (size_t)b * 2048, img, 2048 * sizeof(T));
                bulk_commit();
            }
            sent = true;
        } else {  // rare: codes re-read from global, no indexed register array
#pragma unroll 1
            for (int i = 0; i < 4; ++i) {  // 8 bytes -> 16 values per step
                const int j = i >> 1, h = i & 1;
                const uint8_t *c = codes + b * 1024 + (size_t)(j * 32 + lane) * 16 + 8 * h;
                float v[16];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    v[2 * k] = dequant_level(c[k] >> 4, zp, scale);
                    v[2 * k + 1] = dequant_level(c[k] & 0xFu, zp, scale);
                }
                store16<T>(dst + (size_t)b * 2048 + (size_t)(j * 32 + lane) * 32 + 16 * h, v);
            }
        }
    }
    if (sent && lane == 0) bulk_wait_all();  // the images stay until the copies are done
}

// NF4 decode, any block size: one thread per element.
template <typename T>
__global__ void decompress_nf4_kernel(const uint8_t *__restrict__ codes, const float *__restrict__ stats,
                                      T *__restrict__ dst, size_t num_blocks, int block_elems) {
    const size_t n = num_blocks * (size_t)block_elems;
    const size_t cb = (size_t)(block_elems + 1) / 2;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += stride) {
        const size_t b = e / (size_t)block_elems, i = e % (size_t)block_elems;
        const uint32_t byte = codes[b * cb + i / 2];
        const uint32_t q = (i & 1) ? (byte & 0xFu) : (byte >> 4);
        st_out<T>(dst + e, dequant_level(q, stats[4 * b + 3], stats[4 * b + 2]));
    }
}

// compressToFP16 (KVCompressionEngine.cpp:36-61): Inf/NaN -> +-Inf, zero
// exponent -> +-0, else exponent rebiased modulo 32, mantissa truncated.
__device__ __forceinline__ uint32_t fp16_wrap_enc(float f) {
    const uint32_t bits = __float_as_uint(f);
    const uint32_t sign = bits >> 31, e = (bits >> 23) & 0xFFu, m = bits & 0x7FFFFFu;
    if (e == 0xFFu) return (sign << 15) | 0x7C00u;
    if (e == 0u) return sign << 15;
    return (sign << 15) | ((((int32_t)e - 127 + 15) & 0x1F) << 10) | ((m >> 13) & 0x3FFu);
}

// decompressFP16 (KVCompressionEngine.cpp:63-80): exponent rebiased modulo
// 256 with no special cases.
__device__ __forceinline__ float fp16_wrap_dec(uint32_t h) {
    const uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    return __uint_as_float((sign << 31) | (((e + 112u) & 0xFFu) << 23) | (m << 13));
}

__global__ void fp16_wrap_encode_kernel(const float *__restrict__ src, uint16_t *__restrict__ dst, size_t n,
                                        bool vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t quads = vec ? n / 4 : 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads; i += stride) {
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(src) + i);
        __stcs(reinterpret_cast<uint2 *>(dst) + i,
               make_uint2(fp16_wrap_enc(v.x) | (fp16_wrap_enc(v.y) << 16), fp16_wrap_enc(v.z) | (fp16_wrap_enc(v.w) << 16)));
    }
    for (size_t i = quads * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = (uint16_t)fp16_wrap_enc(src[i]);
}

__global__ void fp16_wrap_decode_kernel(const uint16_t *__restrict__ src, float *__restrict__ dst, size_t n,
                                        bool vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t quads = vec ? n / 4 : 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads; i += stride) {
        const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(src) + i);
        __stcs(reinterpret_cast<float4 *>(dst) + i,
               make_float4(fp16_wrap_dec(v.x & 0xFFFFu), fp16_wrap_dec(v.x >> 16), fp16_wrap_dec(v.y & 0xFFFFu),
                           fp16_wrap_dec(v.y >> 16)));
    }
    for (size_t i = quads * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = fp16_wrap_dec(src[i]);
}

// fp16 -> fp32 decoders over whole tiles of 2048 elements: one CTA per tile,
// each thread one 16-byte load of 8 halves; the 8 KiB of floats go out as
// one bulk copy from a shared-memory image (as the block decoders do).
struct TruncDec {
    __device__ static float dec(uint32_t h) { return f16_trunc_to_f32((uint16_t)h); }
};
struct WrapDec {
    __device__ static float dec(uint32_t h) { return fp16_wrap_dec(h); }
};

template <typename Op>
__global__ void __launch_bounds__(256) f16_decode_tile_kernel(const uint16_t *__restrict__ src, float *__restrict__ dst) {
    __shared__ __align__(128) float img[2048];
    const size_t t = blockIdx.x;
    const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(src + t * 2048) + threadIdx.x);
    float4 *o = reinterpret_cast<float4 *>(img) + 2 * threadIdx.x;
    o[0] = make_float4(Op::dec(v.x & 0xFFFFu), Op::dec(v.x >> 16), Op::dec(v.y & 0xFFFFu), Op::dec(v.y >> 16));
    o[1] = make_float4(Op::dec(v.z & 0xFFFFu), Op::dec(v.z >> 16), Op::dec(v.w & 0xFFFFu), Op::dec(v.w >> 16));
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
        bulk_s2g(dst + t * 2048, img, 2048 * sizeof(float));
        bulk_commit();
        bulk_wait_all();
    }
}

// CTAs that fit on the current GPU at once for `kernel` at 256 threads (its
// occupancy times the SM count), cached per kernel and device.
int resident_ctas(const void *kernel) {
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({kernel, dev});
    if (it != cache.end()) return it->second;
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
    cudaGetLastError();  // leave no error from the queries for launch_status()
    return cache[{kernel, dev}] = sms * per_sm;
}

// Grid for a grid-stride kernel: `work` items, `per_block` per CTA, capped
// at `waves` times the CTAs that fit at once (0: no cap, one CTA per
// `per_block` items).  The SMs' shares of HBM bandwidth differ, so CTAs
// handed out dynamically balance better than equal static shares: the
// decoders run uncapped, the encoders (heavier per CTA) at 16 waves, the
// element-wise converters at 8.
template <typename K> unsigned grid_for(K kernel, size_t work, int per_block, int waves) {
    size_t b = (work + per_block - 1) / per_block;
    const size_t cap = waves > 0 ? (size_t)waves * resident_ctas(reinterpret_cast<const void *>(kernel)) : b;
    if (b > cap) b = cap;
    if (b > 0x7FFFFFFFu) b = 0x7FFFFFFFu;
    return (unsigned)(b ? b : 1);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_compress_int8(const void *src, int32_t src_dtype, int8_t *codes,
                                         float *stats, size_t num_blocks, int32_t block_elems,
                                         void *stream) {
    if (!src || !codes || !stats || block_elems <= 0) return KVX_EINVAL;
    if (src_dtype != KVX_F16 && src_dtype != KVX_F32) return KVX_EINVAL;
    if (!aligned16(stats)) return KVX_EINVAL;
    if (num_blocks == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool fast = block_elems == 2048 && aligned16(src) && aligned16(codes);
    uint8_t *c = reinterpret_cast<uint8_t *>(codes);
    if (src_dtype == KVX_F16) {
        if (fast)
            compress_2048_kernel<__half, 255><<<grid_for(compress_2048_kernel<__half, 255>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const __half *>(src), c, stats, num_blocks);
        else
            compress_generic_kernel<__half, 255><<<grid_for(compress_generic_kernel<__half, 255>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const __half *>(src), c, stats, num_blocks, block_elems);
    } else {
        if (fast)
            compress_2048_kernel<float, 255><<<grid_for(compress_2048_kernel<float, 255>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const float *>(src), c, stats, num_blocks);
        else
            compress_generic_kernel<float, 255><<<grid_for(compress_generic_kernel<float, 255>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const float *>(src), c, stats, num_blocks, block_elems);
    }
    return launch_status();
}

extern "C" KVX_API int kvx_compress_nf4(const void *src, int32_t src_dtype, uint8_t *codes, float *stats,
                                        size_t num_blocks, int32_t block_elems, void *stream) {
    if (!src || !codes || !stats || block_elems <= 0) return KVX_EINVAL;
    if (src_dtype != KVX_F16 && src_dtype != KVX_F32) return KVX_EINVAL;
    if (!aligned16(stats)) return KVX_EINVAL;
    if (num_blocks == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool fast = block_elems == 2048 && aligned16(src) && aligned16(codes);
    if (src_dtype == KVX_F16) {
        if (fast)
            compress_2048_kernel<__half, 15><<<grid_for(compress_2048_kernel<__half, 15>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const __half *>(src), codes, stats, num_blocks);
        else
            compress_generic_kernel<__half, 15><<<grid_for(compress_generic_kernel<__half, 15>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const __half *>(src), codes, stats, num_blocks, block_elems);
    } else {
        if (fast)
            compress_2048_kernel<float, 15><<<grid_for(compress_2048_kernel<float, 15>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const float *>(src), codes, stats, num_blocks);
        else
            compress_generic_kernel<float, 15><<<grid_for(compress_generic_kernel<float, 15>, num_blocks, 8, 16), 256, 0, st>>>(static_cast<const float *>(src), codes, stats, num_blocks, block_elems);
    }
    return launch_status();
}

extern "C" KVX_API int kvx_decompress_nf4(const uint8_t *codes, const float *stats, void *dst, int32_t dst_dtype,
                                          size_t num_blocks, int32_t block_elems, void *stream) {
    if (!codes || !stats || !dst || block_elems <= 0) return KVX_EINVAL;
    if (dst_dtype != KVX_F16 && dst_dtype != KVX_F32) return KVX_EINVAL;
    const size_t esz = dst_dtype == KVX_F32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(stats) & 3) || (reinterpret_cast<uintptr_t>(dst) & (esz - 1))) return KVX_EINVAL;
    if (num_blocks == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (block_elems == 2048 && aligned16(codes) && aligned16(dst) && aligned16(stats)) {
        if (dst_dtype == KVX_F32)
            decompress_nf4_2048_kernel<float><<<(unsigned)((num_blocks + kDqWarps<float> - 1) / kDqWarps<float>),
                                                kDqWarps<float> * 32, 0, st>>>(codes, stats, static_cast<float *>(dst), num_blocks);
        else
            decompress_nf4_2048_kernel<__half><<<(unsigned)((num_blocks + kDqWarps<__half> - 1) / kDqWarps<__half>),
                                                 kDqWarps<__half> * 32, 0, st>>>(codes, stats, static_cast<__half *>(dst), num_blocks);
        return launch_status();
    }
    if (dst_dtype == KVX_F32)
        decompress_nf4_kernel<float><<<grid_for(decompress_nf4_kernel<float>, num_blocks * (size_t)block_elems, 256, 8), 256, 0, st>>>(codes, stats, static_cast<float *>(dst), num_blocks, block_elems);
    else
        decompress_nf4_kernel<__half><<<grid_for(decompress_nf4_kernel<__half>, num_blocks * (size_t)block_elems, 256, 8), 256, 0, st>>>(codes, stats, static_cast<__half *>(dst), num_blocks, block_elems);
    return launch_status();
}

extern "C" KVX_API int kvx_fp16_wrap_encode(const float *src, uint16_t *dst, size_t n, void *stream) {
    if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(dst) & 1))
        return KVX_EINVAL;
    if (n == 0) return KVX_OK;
    const bool vec = aligned16(src) && !(reinterpret_cast<uintptr_t>(dst) & 7);
    fp16_wrap_encode_kernel<<<grid_for(fp16_wrap_encode_kernel, vec ? n / 4 + 1 : n, 256, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        src, dst, n, vec);
    return launch_status();
}

extern "C" KVX_API int kvx_fp16_wrap_decode(const uint16_t *src, float *dst, size_t n, void *stream) {
    if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 1) || (reinterpret_cast<uintptr_t>(dst) & 3))
        return KVX_EINVAL;
    if (n == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    size_t done = 0;
    if (aligned16(src) && aligned16(dst) && n >= 2048) {
        done = n / 2048 * 2048;
        f16_decode_tile_kernel<WrapDec><<<(unsigned)(n / 2048), 256, 0, st>>>(src, dst);
        if (done == n) return launch_status();
    }
    src += done, dst += done, n -= done;
    const bool vec = !(reinterpret_cast<uintptr_t>(src) & 7) && aligned16(dst);
    fp16_wrap_decode_kernel<<<grid_for(fp16_wrap_decode_kernel, vec ? n / 4 + 1 : n, 256, 8), 256, 0, st>>>(
        src, dst, n, vec);
    return launch_status();
}

extern "C" KVX_API int kvx_decompress_int8(const int8_t *codes, const float *stats, void *dst,
                                           int32_t dst_dtype, size_t num_blocks,
                                           int32_t block_elems, void *stream) {
    if (!codes || !stats || !dst || block_elems <= 0) return KVX_EINVAL;
    if (dst_dtype != KVX_F16 && dst_dtype != KVX_F32) return KVX_EINVAL;
    const uintptr_t esz = dst_dtype == KVX_F32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(stats) & 3) || (reinterpret_cast<uintptr_t>(dst) & (esz - 1)))
        return KVX_EINVAL;
    if (num_blocks == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (block_elems % 4 || !aligned16(stats) || (reinterpret_cast<uintptr_t>(codes) & 3) || !aligned16(dst)) {
        if (dst_dtype == KVX_F32)
            decompress_scalar_kernel<float><<<grid_for(decompress_scalar_kernel<float>, num_blocks * (size_t)block_elems, 256, 8), 256, 0, st>>>(codes, stats, static_cast<float *>(dst), num_blocks, block_elems);
        else
            decompress_scalar_kernel<__half><<<grid_for(decompress_scalar_kernel<__half>, num_blocks * (size_t)block_elems, 256, 8), 256, 0, st>>>(codes, stats, static_cast<__half *>(dst), num_blocks, block_elems);
        return launch_status();
    }
    if (block_elems == 2048 && aligned16(codes)) {
        if (dst_dtype == KVX_F32)
            decompress_2048_kernel<float><<<(unsigned)((num_blocks + kDqWarps<float> - 1) / kDqWarps<float>),
                                            kDqWarps<float> * 32, 0, st>>>(codes, stats, static_cast<float *>(dst), num_blocks);
        else
            decompress_2048_kernel<__half><<<(unsigned)((num_blocks + kDqWarps<__half> - 1) / kDqWarps<__half>),
                                             kDqWarps<__half> * 32, 0, st>>>(codes, stats, static_cast<__half *>(dst), num_blocks);
        return launch_status();
    }
    if (dst_dtype == KVX_F32)
        decompress_kernel<float><<<grid_for(decompress_kernel<float>, num_blocks * (size_t)(block_elems / 4), 256, 8), 256, 0, st>>>(codes, stats, static_cast<float *>(dst), num_blocks, block_elems);
    else
        decompress_kernel<__half><<<grid_for(decompress_kernel<__half>, num_blocks * (size_t)(block_elems / 4), 256, 8), 256, 0, st>>>(codes, stats, static_cast<__half *>(dst), num_blocks, block_elems);
    return launch_status();
}

extern "C" KVX_API int kvx_f32_to_f16_trunc(const float *src, uint16_t *dst, size_t n, void *stream) {
    if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(dst) & 1))
        return KVX_EINVAL;
    if (n == 0) return KVX_OK;
    const bool vec = aligned16(src) && !(reinterpret_cast<uintptr_t>(dst) & 7);
    encode_trunc_kernel<<<grid_for(encode_trunc_kernel, vec ? n / 4 + 1 : n, 256, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        src, dst, n, vec);
    return launch_status();
}

extern "C" KVX_API int kvx_f16_trunc_to_f32(const uint16_t *src, float *dst, size_t n, void *stream) {
    if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 1) || (reinterpret_cast<uintptr_t>(dst) & 3))
        return KVX_EINVAL;
    if (n == 0) return KVX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    size_t done = 0;
    if (aligned16(src) && aligned16(dst) && n >= 2048) {
        done = n / 2048 * 2048;
        f16_decode_tile_kernel<TruncDec><<<(unsigned)(n / 2048), 256, 0, st>>>(src, dst);
        if (done == n) return launch_status();
    }
    src += done, dst += done, n -= done;
    const bool vec = !(reinterpret_cast<uintptr_t>(src) & 7) && aligned16(dst);
    decode_trunc_kernel<<<grid_for(decode_trunc_kernel, vec ? n / 4 + 1 : n, 256, 8), 256, 0, st>>>(
        src, dst, n, vec);
    return launch_status();
}
