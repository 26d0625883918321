// kvx_decode_tc.cu -- tensor-core paged GQA decode for fp16 pools (sm_100a).
//
// Same contract and CTA decomposition as the SIMT kernel in kvx_decode.cu
// (grid = split x kv-head x sequence, 4 warps per CTA, pages round-robin
// over warps, flash-decoding partials folded by the last CTA), with the math
// moved to the tensor cores so the kernel is bound by HBM, not by issue:
//
//  * staging: per (page, head) the K and V blocks (16 tokens x 128 dims) are
//    fetched as four 2 KiB TMA tensor tiles (cp.async.bulk.tensor.2d, box
//    64 dims x 16 tokens, 128-byte swizzle) into a per-warp 2-stage ring,
//    completing on an mbarrier (bounded wait).  The swizzle makes every
//    ldmatrix below bank-conflict free although page rows are 256 B apart.
//  * S = Q K^T: mma.sync m16n8k16 (fp16 in, fp32 accumulate) with the GQA
//    group as M (q-heads, padded to 16), tokens as N (two n-tiles per page)
//    and head_dim as K (8 k-steps).  Q lives in registers as A fragments.
//  * online softmax on the S fragments in the log2 domain (fp32).
//  * O += P V: the S accumulators, rounded to fp16, are the A fragments of
//    the next mma (no shared-memory round trip); V is read with
//    ldmatrix.trans; O is 16 n-tiles of fp32 accumulators per warp.
//
// Instruction count per (page, head): 8 + 8 ldmatrix.x4, 32 mma, ~40 for
// softmax and rescale -- against ~1100 for the SIMT kernel.
//
// int8 pools (codes of the reference's KVCompressionEngine scheme, one
// {min, max, scale, zero_point} per (page, K|V, head) block) run the same
// kernel with kI8: a stage is two (page, head)s, each two 2 KiB code blocks
// (TMA box 128 x 16 bytes, 128-byte swizzle) plus two 16-byte stats rows
// (bulk copies), two stages per warp.  Codes become fp16 in registers: x = c ^ 0x80 is the
// unsigned code u = c + 128, and the bytes {u, 0x64} are the fp16 1024 + u
// (byte permutes, no conversion instruction).  With k = zp + scale * u:
//   q.k = scale * (q . (1024 + u)) + (zp - 1024 * scale) * sum(q)
// per page, so the mma runs on 1024 + u directly; for V the softmax weights
// are multiplied by the page's scale before rounding to fp16 (P' = p * sv)
// and the zero point enters through one scalar per row,
//   sum_t p_t v_t = P' . (1024 + u) + sum_t (zp * p_t - 1024 * P'_t),
// with P'_t the rounded values the mma used, so the 1024 terms cancel.
// The head dimension is permuted so fragments come straight from shared
// memory: for QK, k-step kc of lane (g, r) takes bytes 32r + 4kc .. +3 of
// its token row (Q loaded in the same order); for PV, ldmatrix.trans of the
// codes as 16-bit pairs hands lane (g, r) dims 2g, 2g+1 of tokens 2r, 2r+1,
// so n-tile 2c + par column g is dim 16c + 2g + par.
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>

#include <mutex>

#include "kvx_decode_params.cuh"

namespace kvx {
namespace {

constexpr int kTcWarps = 4;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kBox = 2048;          // 16 tokens x 64 dims x fp16 (or 128 int8), 128B-swizzled
constexpr int kQloBytes = 8 * 32 * 16;  // q lo A fragments, 8 k-steps x 32 lanes x 4 regs (group > 8)
constexpr int kBtCache = 64;            // block-table entries staged per warp
constexpr int kCombineFloats = 4096;    // split weights kept in the ring for the combine

// Per-warp staging ring of 2 stages.  fp16: a stage is one page, K dims 0-63
// | K 64-127 | V 0-63 | V 64-127.  int8: a stage is two pages, K codes | V
// codes | K codes | V codes, their four stats rows kept apart.
template <bool kI8> struct TcCfg {
    static constexpr int kStages = 2;
    static constexpr int kStage = 4 * kBox;
    static constexpr int kPages = kI8 ? 2 : 1;      // pages per stage
    static constexpr int kRing = kStages * kStage;  // >= 16 KiB: parks O at the end
    static constexpr int kStatBytes = 0;  // int8 stats travel in registers (lanes 0-3), one stage ahead
    static constexpr int kSmem = 1024 /* alignment slack */ + kTcWarps * kRing + kTcWarps * kStages * 8 +
                                 kStatBytes + 2 * kTcWarps * 16 * 4 + 16 + kQloBytes + kTcWarps * kBtCache * 4;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Same mma when only rows 0-7 of the tile matter (GQA group <= 8): the
// accumulator rows 8-15 enter as zero and their results are discarded, so
// they occupy no long-lived registers.
__device__ __forceinline__ void mma16816_lo(float &c0, float &c1, const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
    float d2 __attribute__((unused)), d3 __attribute__((unused));  // rows 8-15, discarded
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%12};"
        : "=f"(c0), "=f"(c1), "=f"(d2), "=f"(d3)
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(0.f));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Byte offset of 16-byte chunk `c` (0..7) of `row` inside a 128B-swizzled
// box whose rows are 128 bytes: the TMA unit XORs the chunk index with the
// row index modulo 8.
__device__ __forceinline__ uint32_t swz(int row, int c) {
    return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4));
}

// One staged (page, head) tile pair: S = Q K^T (two n-tiles of 8 tokens),
// online softmax in the log2 domain, O += P V.  `sbase` is the shared
// address of the stage (K lo | K hi | V lo | V hi, 128B-swizzled); `tok`
// the absolute index of token 2*tq of the page; tokens >= T are masked.
//
// q enters as fp16 hi + lo (q - hi rounded again), so that scores keep
// fp32-like accuracy against keys with outlier channels: with a GQA group
// <= 8 the lo parts are rows 8-15 of the A tile (padding otherwise) and S
// adds rows g and g + 8; with a larger group the lo fragments come from
// shared memory (`qlo`, CTA-wide) and take a second mma per k-step.
template <bool kBig>
__device__ __forceinline__ void tc_page(uint32_t sbase, const uint32_t (&qa)[8][4], uint32_t qlo,
                                        float (&o)[16][4], float &m0, float &m1, float &l0, float &l1,
                                        int tok, int T, float scale_log2, int lane, float &psum0, float &psum1) {
    const int lrow = lane & 7, lmat = lane >> 3;
    // ---- S = Q K^T for tokens 0-7 (n-tile 0) and 8-15 (n-tile 1)
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {  // k-steps 2kp, 2kp+1 = chunks 4kp..4kp+3
        uint32_t l0a[4], l1a[4];
        if constexpr (kBig) {
            const uint4 x = lds128(qlo + ((2 * kp) * 32 + lane) * 16);
            const uint4 y = lds128(qlo + ((2 * kp + 1) * 32 + lane) * 16);
            l0a[0] = x.x, l0a[1] = x.y, l0a[2] = x.z, l0a[3] = x.w;
            l1a[0] = y.x, l1a[1] = y.y, l1a[2] = y.z, l1a[3] = y.w;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int chunk = 4 * kp + lmat;
            const uint32_t addr = sbase + (chunk >> 3) * kBox + swz(8 * j + lrow, chunk & 7);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(addr, b0, b1, b2, b3);
            mma16816(sc[j], qa[2 * kp], b0, b1);
            mma16816(sc[j], qa[2 * kp + 1], b2, b3);
            if constexpr (kBig) {
                mma16816(sc[j], l0a, b0, b1);
                mma16816(sc[j], l1a, b2, b3);
            }
        }
    }
    if constexpr (!kBig) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            sc[j][0] += sc[j][2];
            sc[j][1] += sc[j][3];
        }
    }
    // ---- online softmax (log2 domain)
    float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const bool valid = tok + 8 * j + e < T;
            sc[j][e] = valid ? sc[j][e] * scale_log2 : -CUDART_INF_F;
            mx0 = fmaxf(mx0, sc[j][e]);
            if constexpr (kBig) {
                sc[j][2 + e] = valid ? sc[j][2 + e] * scale_log2 : -CUDART_INF_F;
                mx1 = fmaxf(mx1, sc[j][2 + e]);
            }
        }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    const float mn0 = fmaxf(m0, mx0);
    const float a0 = exp2f(m0 - mn0);
    m0 = mn0;
    float a1 = 1.f;
    if constexpr (kBig) {
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn1 = fmaxf(m1, mx1);
        a1 = exp2f(m1 - mn1);
        m1 = mn1;
    }
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            sc[j][e] = exp2f(sc[j][e] - m0);
            ps0 += sc[j][e];
            if constexpr (kBig) {
                sc[j][2 + e] = exp2f(sc[j][2 + e] - m1);
                ps1 += sc[j][2 + e];
            }
        }
    l0 = l0 * a0 + ps0;
    if constexpr (kBig) l1 = l1 * a1 + ps1;
    psum0 = ps0;
    psum1 = ps1;
    uint32_t pa[4];
    pa[0] = pack_h2(sc[0][0], sc[0][1]);
    pa[2] = pack_h2(sc[1][0], sc[1][1]);
    if constexpr (kBig) {
        pa[1] = pack_h2(sc[0][2], sc[0][3]);
        pa[3] = pack_h2(sc[1][2], sc[1][3]);
    } else {
        pa[1] = pa[3] = 0u;
    }
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {  // a running max moved
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= a0;
            o[n][1] *= a0;
            if constexpr (kBig) {
                o[n][2] *= a1;
                o[n][3] *= a1;
            }
        }
    }
    // ---- O += P V
#pragma unroll
    for (int np = 0; np < 8; ++np) {
        const int chunk = 2 * np + (lmat >> 1);
        const int vrow = (lmat & 1) * 8 + lrow;
        const uint32_t addr = sbase + 2 * kBox + (chunk >> 3) * kBox + swz(vrow, chunk & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        if constexpr (kBig) {
            mma16816(o[2 * np], pa, b0, b1);
            mma16816(o[2 * np + 1], pa, b2, b3);
        } else {
            mma16816_lo(o[2 * np][0], o[2 * np][1], pa, b0, b1);
            mma16816_lo(o[2 * np + 1][0], o[2 * np + 1][1], pa, b2, b3);
        }
    }
}

// fp16 pair {1024 + byte lo, 1024 + byte hi} of two bytes of x.
__device__ __forceinline__ uint32_t u8x2_to_h2(uint32_t x, uint32_t sel) { return __byte_perm(x, 0x64u, sel); }

// One staged pair of int8 (page, head)s: K codes of page a at base, V at
// base + kBox, page b's at base + 2 kBox / 3 kBox (128-byte rows,
// 128B-swizzled); st = their stats rows {min, max, scale, zero_point} in the
// order K a, V a, K b, V b; va / vb: the page is there (a missing page is
// masked to weight 0, whatever its staged bytes).  qs0 / qs1 = sum of the q
// fed to the mma for rows g / g + 8; z0 / z1 the zero-point scalars of rows
// g / g + 8 (partial over this lane's tokens).  Two pages per call give four
// independent QK accumulation chains and one softmax update per 32 tokens.
//
// The weights multiply v - zp = scale * u, which in a block with outliers
// can be far larger than v itself, so one fp16 rounding of P' would cost up
// to 2^-11 of the block's range.  P' is therefore carried as fp16 hi + lo,
// like q: with a GQA group <= 8 the lo parts ride in rows 8-15 of the m16
// tile, which are padding otherwise (S and O add rows g and g + 8); with a
// larger group the lo parts take a second mma into the same accumulators
// (q lo fragments from shared memory, `qlo`).
template <bool kBig>
__device__ __forceinline__ void tc_pair_i8(uint32_t base, float2 st, bool va, bool vb,
                                           const uint32_t (&qa)[8][4], uint32_t qlo, float qs0, float qs1,
                                           float (&o)[16][4], float &m0, float &m1, float &l0, float &l1,
                                           float &z0, float &z1, int tok_a, int tok_b, int T,
                                           float scale_log2, int lane, float (&psum)[2][2]) {
    const int g = lane >> 2, r = lane & 3;
    // {scale, zero_point} of K a, V a, K b, V b sit in lanes 0-3
    float2 ska, sva, skb, svb;
    ska.x = __shfl_sync(0xffffffffu, st.x, 0), ska.y = __shfl_sync(0xffffffffu, st.y, 0);
    sva.x = __shfl_sync(0xffffffffu, st.x, 1), sva.y = __shfl_sync(0xffffffffu, st.y, 1);
    skb.x = __shfl_sync(0xffffffffu, st.x, 2), skb.y = __shfl_sync(0xffffffffu, st.y, 2);
    svb.x = __shfl_sync(0xffffffffu, st.x, 3), svb.y = __shfl_sync(0xffffffffu, st.y, 3);
    // ---- S = scale * Q (1024 + u) + (zp - 1024 scale) sum(q); tile t = 2 page + j
    float sc[4][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // chunk 2r + half holds k-steps 4 half .. 4 half + 3
        uint4 kw[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) kw[t] = lds128(base + (t >> 1) * 2 * kBox + swz(8 * (t & 1) + g, 2 * r + half));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const int kc = 4 * half + kk;
            uint32_t la[4];
            if constexpr (kBig) {
                const uint4 x = lds128(qlo + (kc * 32 + lane) * 16);
                la[0] = x.x, la[1] = x.y, la[2] = x.z, la[3] = x.w;
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t w = (kk == 0 ? kw[t].x : kk == 1 ? kw[t].y : kk == 2 ? kw[t].z : kw[t].w) ^ 0x80808080u;
                const uint32_t b0 = u8x2_to_h2(w, 0x4140), b1 = u8x2_to_h2(w, 0x4342);
                mma16816(sc[t], qa[kc], b0, b1);
                if constexpr (kBig) mma16816(sc[t], la, b0, b1);
            }
        }
    }
    if constexpr (!kBig) {  // q hi (rows 0-7) + q lo (rows 8-15)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            sc[t][0] += sc[t][2];
            sc[t][1] += sc[t][3];
        }
    }
    // ---- online softmax (log2 domain) over the 32 tokens
    const float ks[2] = {ska.x * scale_log2, skb.x * scale_log2};
    const float ko[2] = {fmaf(-1024.f, ska.x, ska.y) * scale_log2, fmaf(-1024.f, skb.x, skb.y) * scale_log2};
    const bool have[2] = {va, vb};
    const int tok[2] = {tok_a, tok_b};
    float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int pg = t >> 1, j = t & 1;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const bool valid = have[pg] && tok[pg] + 8 * j + e < T;
            sc[t][e] = valid ? fmaf(sc[t][e], ks[pg], ko[pg] * qs0) : -CUDART_INF_F;
            mx0 = fmaxf(mx0, sc[t][e]);
            if constexpr (kBig) {
                sc[t][2 + e] = valid ? fmaf(sc[t][2 + e], ks[pg], ko[pg] * qs1) : -CUDART_INF_F;
                mx1 = fmaxf(mx1, sc[t][2 + e]);
            }
        }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    const float mn0 = fmaxf(m0, mx0);
    const float a0 = exp2f(m0 - mn0);
    m0 = mn0;
    float a1 = 1.f;
    if constexpr (kBig) {
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn1 = fmaxf(m1, mx1);
        a1 = exp2f(m1 - mn1);
        m1 = mn1;
    }
    float ps0[2] = {0.f, 0.f}, ps1[2] = {0.f, 0.f};
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            sc[t][e] = exp2f(sc[t][e] - m0);
            ps0[t >> 1] += sc[t][e];
            if constexpr (kBig) {
                sc[t][2 + e] = exp2f(sc[t][2 + e] - m1);
                ps1[t >> 1] += sc[t][2 + e];
            }
        }
    l0 = l0 * a0 + (ps0[0] + ps0[1]);
    if constexpr (kBig) l1 = l1 * a1 + (ps1[0] + ps1[1]);
    psum[0][0] = ps0[0], psum[0][1] = ps1[0], psum[1][0] = ps0[1], psum[1][1] = ps1[1];
    // P' = p * scale_v as fp16 hi + lo (masked tokens stay exactly 0).  hi +
    // lo equals P' to 2^-22 relative, so the zero-point scalar may use the
    // unrounded sum: (zp - 1024 scale_v) * sum(p), off by < 2.5e-4 * scale_v
    // of the output.
    const float svs[2] = {sva.x, svb.x};
    auto split = [](float x, float y, uint32_t &hi, uint32_t &lo) {
        hi = pack_h2(x, y);
        const float2 h = h2_to_f2(hi);
        lo = pack_h2(x - h.x, y - h.y);
    };
    uint32_t pa[2][4], pl[2][4];
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
        auto wv = [&](float pv) { return pv == 0.f ? 0.f : pv * svs[pg]; };
        split(wv(sc[2 * pg][0]), wv(sc[2 * pg][1]), pa[pg][0], pl[pg][0]);
        split(wv(sc[2 * pg + 1][0]), wv(sc[2 * pg + 1][1]), pa[pg][2], pl[pg][2]);
        if constexpr (kBig) {
            split(wv(sc[2 * pg][2]), wv(sc[2 * pg][3]), pa[pg][1], pl[pg][1]);
            split(wv(sc[2 * pg + 1][2]), wv(sc[2 * pg + 1][3]), pa[pg][3], pl[pg][3]);
        } else {  // rows 8-15: the lo parts
            pa[pg][1] = pl[pg][0];
            pa[pg][3] = pl[pg][2];
        }
    }
    const float voa = va ? fmaf(-1024.f, sva.x, sva.y) : 0.f, vob = vb ? fmaf(-1024.f, svb.x, svb.y) : 0.f;
    z0 = fmaf(z0, a0, fmaf(voa, ps0[0], vob * ps0[1]));
    if constexpr (kBig) z1 = fmaf(z1, a1, fmaf(voa, ps1[0], vob * ps1[1]));
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {  // a running max moved
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= a0;
            o[n][1] *= a0;
            o[n][2] *= kBig ? a1 : a0;
            o[n][3] *= kBig ? a1 : a0;
        }
    }
    // ---- O += P' (1024 + u).  ldmatrix.trans over the V codes as 16-bit
    // pairs gives lane (g, r) the bytes {V[2r][2g], V[2r][2g+1], V[2r+1][2g],
    // V[2r+1][2g+1]} of a 16-dim chunk (tokens 8-15 in the next matrix):
    // bytes 0,2 are B rows k, k+1 of n-tile column "dim 2g", bytes 1,3 of
    // "dim 2g+1".  n-tile 2c + par, column g = dim 16c + 2g + par.
    const int lrow = lane & 7, lmat = lane >> 3;
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
        if (!have[pg]) continue;  // warp-uniform
        const uint32_t vbase = base + pg * 2 * kBox + kBox;
#pragma unroll
        for (int cp = 0; cp < 4; ++cp) {  // chunks 2cp, 2cp+1
            const int chunk = 2 * cp + (lmat >> 1);
            const int vrow = (lmat & 1) * 8 + lrow;
            uint32_t v0, v1, v2, v3;  // (tok 0-7, chunk 2cp) (8-15, 2cp) (0-7, 2cp+1) (8-15, 2cp+1)
            ldsm_x4_t(vbase + swz(vrow, chunk), v0, v1, v2, v3);
            v0 ^= 0x80808080u;
            v1 ^= 0x80808080u;
            v2 ^= 0x80808080u;
            v3 ^= 0x80808080u;
            const uint32_t b0[4] = {u8x2_to_h2(v0, 0x4240), u8x2_to_h2(v0, 0x4341), u8x2_to_h2(v2, 0x4240),
                                    u8x2_to_h2(v2, 0x4341)};
            const uint32_t b1[4] = {u8x2_to_h2(v1, 0x4240), u8x2_to_h2(v1, 0x4341), u8x2_to_h2(v3, 0x4240),
                                    u8x2_to_h2(v3, 0x4341)};
#pragma unroll
            for (int e = 0; e < 4; ++e) {  // n-tiles 4cp .. 4cp+3
                mma16816(o[4 * cp + e], pa[pg], b0[e], b1[e]);
                if constexpr (kBig) mma16816(o[4 * cp + e], pl[pg], b0[e], b1[e]);
            }
        }
    }
}

// Where lane (g, r) parks O element (row, n-tile jn, column 2r + e) for the
// merge: fp16 kernel dim 8 jn + 2r + e; int8 kernel dim 16 (jn / 2) +
// 2 (2r + e) + jn % 2, whose bits 2-3 are r, so the row's bits XOR-ed into
// dim bits 0, 1 and 4 make the 32 lanes of one store hit 32 banks.
template <bool kI8> __device__ __forceinline__ int park_ofs(int row, int d) {
    if constexpr (kI8) return row * kHeadDim + (d ^ ((row & 3) | (((row >> 2) & 1) << 4)));
    return row * kHeadDim + d;
}

template <typename QT, bool kBig, bool kI8, bool kAttn>
__device__ __forceinline__ void tc_decode_body(const DecodeParams &p, const CUtensorMap &tm) {
    using Cfg = TcCfg<kI8>;
    constexpr int kTcStages = Cfg::kStages;
    constexpr int kTcStage = Cfg::kStage;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates
    const int split = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    const bool fused = !kI8 && p.positions != nullptr;
    int T = fused ? p.positions[s] + 1 : max(p.seq_lens[s], 0);
    if (fused && T <= 0) T = 0;
    if (T > p.max_pages * kPageTokens) {
        if (p.error_flag && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
            atomicOr(p.error_flag, 4);
        T = p.max_pages * kPageTokens;
    }
    const int npages = (T + kPageTokens - 1) / kPageTokens;
    const int p0 = split * p.chunk;
    const int h0 = kvh * p.group;
    const int nh = p.group;
    if (p0 >= npages) {  // nothing to read: exit (which releases the next launch)
        if (npages == 0 && split == 0) {
            grid_dependency_wait();  // the previous decode may still use the output
            QT *o = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h0) * kHeadDim;
            for (int i = threadIdx.x; i < nh * kHeadDim; i += kTcThreads) io_traits<QT>::store(o + i, 0.f);
        }
        return;
    }
    const int p1 = min(p0 + p.chunk, npages);
    const int nsplit = (npages + p.chunk - 1) / p.chunk;

    uint8_t *wbuf = smem + warp * kTcStages * kTcStage;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kTcWarps * kTcStages * kTcStage) + warp * kTcStages;
    float *s_m = reinterpret_cast<float *>(smem + kTcWarps * kTcStages * kTcStage + kTcWarps * kTcStages * 8 +
                                           Cfg::kStatBytes);
    float *s_l = s_m + kTcWarps * 16;
    int *s_flag = reinterpret_cast<int *>(s_l + kTcWarps * 16);
    uint4 *s_qlo = reinterpret_cast<uint4 *>(s_flag + 4);  // [8][32] A fragments (group > 8)
    int *wbt = reinterpret_cast<int *>(s_qlo + 8 * 32) + warp * kBtCache;  // this warp's physical pages

    if (lane == 0) {
        for (int i = 0; i < kTcStages; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
    }
    __syncwarp();

    // fused append: the CTA whose split holds the new token patches its rows
    // into the staged tiles (below) and writes them into the pool once the
    // previous launch on this stream has finished (it may read that slot:
    // the same pool appended at the same position again).
    const bool append_ok = fused && p.positions[s] >= 0 && p.positions[s] < p.max_pages * kPageTokens;
    const int lp_new = append_ok ? p.positions[s] / kPageTokens : -1;
    const int slot_new = append_ok ? p.positions[s] % kPageTokens : 0;
    const bool appends = append_ok && lp_new >= p0 && lp_new < p1;  // CTA-uniform
    // The next launch on this stream (the next layer's decode) may start
    // filling SMs once every CTA of this one has got here: its CTAs stream
    // their own pages and wait for this grid before they touch the split
    // workspace or the output, so this launch's last partial wave leaves no
    // SM idle.  The appending CTA lets it start only after its pool write is
    // visible device-wide (the next launch may read that page).
    if (!appends) grid_dependents_launch();

    const int n_pg = (p1 - p0 - warp + kTcWarps - 1) / kTcWarps;  // this warp's pages
    const int n_my = (n_pg + Cfg::kPages - 1) / Cfg::kPages;          // and stages
    const int32_t *bt = p.block_table + (size_t)s * p.max_pages;
    const uint32_t wbase = smem_addr(wbuf);
    // the warp's block-table entries, staged once (one global round trip per
    // warp instead of two per page)
    for (int i = lane; i < min(n_pg, kBtCache); i += 32) wbt[i] = bt[p0 + warp + kTcWarps * i];
    __syncwarp();
    auto phys_of = [&](int i) { return i < kBtCache ? wbt[i] : bt[p0 + warp + kTcWarps * i]; };

    auto page_ok = [&](int phys) { return phys >= 0 && phys < p.num_pages; };
    auto issue = [&](int i, int st) {
        uint64_t *bar = &bars[st];
        if constexpr (kI8) {  // pages 2i and (if any) 2i + 1 of this warp
            const int pa_ = phys_of(2 * i), pb_ = 2 * i + 1 < n_pg ? phys_of(2 * i + 1) : 0;
            const bool va = page_ok(pa_), vb = 2 * i + 1 < n_pg && page_ok(pb_);
            if ((!va || (2 * i + 1 < n_pg && !vb)) && p.error_flag) atomicOr(p.error_flag, 2);
            const uint32_t dst = wbase + st * kTcStage, b = smem_addr(bar);
            mbar_arrive_expect_tx(bar, (va ? 2 * kBox : 0) + (vb ? 2 * kBox : 0));
            if (va) {
                const int kb = (pa_ * 2) * p.hkv + kvh;  // (page, K, head) block; V block = kb + hkv
                tma_load_2d(dst, &tm, 0, kb * kPageTokens, b);
                tma_load_2d(dst + kBox, &tm, 0, (kb + p.hkv) * kPageTokens, b);
            }
            if (vb) {
                const int kb = (pb_ * 2) * p.hkv + kvh;
                tma_load_2d(dst + 2 * kBox, &tm, 0, kb * kPageTokens, b);
                tma_load_2d(dst + 3 * kBox, &tm, 0, (kb + p.hkv) * kPageTokens, b);
            }
            return;
        }
        const int phys = phys_of(i);
        if (phys < 0 || phys >= p.num_pages) {
            if (p.error_flag) atomicOr(p.error_flag, 2);
            mbar_arrive_expect_tx(bar, 0);
            return;
        }
        const int kb = (phys * 2) * p.hkv + kvh;  // (page, K, head) block; V block = kb + hkv
        const int yk = kb * kPageTokens;
        const int yv = yk + p.hkv * kPageTokens;
        const uint32_t dst = wbase + st * kTcStage;
        const uint32_t b = smem_addr(bar);
        mbar_arrive_expect_tx(bar, kTcStage);
        tma_load_2d(dst, &tm, 0, yk, b);
        tma_load_2d(dst + kBox, &tm, 64, yk, b);
        tma_load_2d(dst + 2 * kBox, &tm, 0, yv, b);
        tma_load_2d(dst + 3 * kBox, &tm, 64, yv, b);
    };
    if (lane == 0)
        for (int i = 0; i < min(kTcStages, n_my); ++i) issue(i, i);

    // Q as m16n8k16 A fragments: rows = q-heads of this kv-head (zero padded),
    // k = head_dim in 8 steps of 16.
    // Q as fp16 hi + lo A fragments.  int8: k-step kk of lane (gq, tq)
    // covers dims 32 tq + 4 kk .. +3 (the order the codes are read in), and
    // qs0 / qs1 are the sums of what the mma is fed for rows gq / gq + 8.
    uint32_t qa[8][4];
    float qs0 = 0.f, qs1 = 0.f;
    {
        const QT *qb = reinterpret_cast<const QT *>(p.q) + ((size_t)s * p.hq + h0) * kHeadDim;
        const bool r0 = gq < nh, r1 = kBig && gq + 8 < nh;
        auto ld = [&](bool ok, int row, int col) -> float {
            return ok ? io_traits<QT>::load(qb + row * kHeadDim + col) : 0.f;
        };
        auto split = [](float x, float y, uint32_t &hi, uint32_t &lo, float &sum) {
            hi = pack_h2(x, y);
            const float2 h = h2_to_f2(hi);
            lo = pack_h2(x - h.x, y - h.y);
            const float2 l = h2_to_f2(lo);
            sum += (h.x + h.y) + (l.x + l.y);
        };
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int c0 = kI8 ? 32 * tq + 4 * kk : 16 * kk + 2 * tq;
            const int c8 = kI8 ? c0 + 2 : c0 + 8;
            uint32_t lo[4];
            split(ld(r0, gq, c0), ld(r0, gq, c0 + 1), qa[kk][0], lo[0], qs0);
            split(ld(r0, gq, c8), ld(r0, gq, c8 + 1), qa[kk][2], lo[2], qs0);
            if constexpr (kBig) {
                split(ld(r1, gq + 8, c0), ld(r1, gq + 8, c0 + 1), qa[kk][1], lo[1], qs1);
                split(ld(r1, gq + 8, c8), ld(r1, gq + 8, c8 + 1), qa[kk][3], lo[3], qs1);
                if (warp == 0) s_qlo[kk * 32 + lane] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            } else {  // rows 8-15: q lo
                qa[kk][1] = lo[0];
                qa[kk][3] = lo[2];
            }
        }
        qs0 += __shfl_xor_sync(0xffffffffu, qs0, 1);
        qs0 += __shfl_xor_sync(0xffffffffu, qs0, 2);
        qs1 += __shfl_xor_sync(0xffffffffu, qs1, 1);
        qs1 += __shfl_xor_sync(0xffffffffu, qs1, 2);
    }
    if constexpr (kBig) __syncthreads();  // q lo fragments visible to every warp
    const uint32_t qlo = smem_addr(s_qlo);

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
    float z0 = 0.f, z1 = 0.f;  // int8 zero-point terms

    // attention mass of one page: the rows' sums over its tokens, with the
    // running max they are relative to (warp-uniform call)
    auto record_mass = [&](int lp, float a, float b) {
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        if constexpr (kBig) {
            b += __shfl_xor_sync(0xffffffffu, b, 1);
            b += __shfl_xor_sync(0xffffffffu, b, 2);
        }
        if (tq == 0) {
            if (gq < nh)
                *reinterpret_cast<float2 *>(p.attn_pm + (((size_t)s * p.hq + h0 + gq) * p.max_pages + lp) * 2) =
                    make_float2(m0, a);
            if (kBig && gq + 8 < nh)
                *reinterpret_cast<float2 *>(p.attn_pm + (((size_t)s * p.hq + h0 + gq + 8) * p.max_pages + lp) * 2) =
                    make_float2(m1, b);
        }
    };

    // int8: {scale, zero_point} of stage i's K a, V a, K b, V b blocks, one
    // per lane 0-3, loaded while stage i - 1 is processed
    auto stats_of = [&](int i) -> float2 {
        if (!kI8 || lane >= 4) return make_float2(0.f, 0.f);
        const int pg = 2 * i + (lane >> 1);
        if (pg >= n_pg) return make_float2(0.f, 0.f);
        const int ph = phys_of(pg);
        if (!page_ok(ph)) return make_float2(0.f, 0.f);
        const int blk = (ph * 2 + (lane & 1)) * p.hkv + kvh;
        return __ldg(reinterpret_cast<const float2 *>(p.stats + (size_t)blk * 4) + 1);
    };
    float2 st_next = stats_of(0);

    bool ok = true;
    int done = 0;
    for (int i = 0; i < n_my; ++i) {
        const int st = i % kTcStages;
        const uint32_t par = (i / kTcStages) & 1;
        const float2 st_cur = st_next;
        if (kI8 && i + 1 < n_my) st_next = stats_of(i + 1);
        if (!mbar_wait_bounded(&bars[st], par, p.error_flag)) {
            ok = false;
            break;
        }
        done = i + 1;
        const uint32_t sbase = wbase + st * kTcStage;
        if constexpr (kI8) {
            const int lpa = p0 + warp + kTcWarps * (2 * i);
            const bool va = page_ok(phys_of(2 * i));
            const bool vb = 2 * i + 1 < n_pg && page_ok(phys_of(2 * i + 1));
            if (va || vb) {
                float psum[2][2];
                tc_pair_i8<kBig>(sbase, st_cur, va, vb, qa, qlo, qs0, qs1, o, m0, m1, l0,
                                 l1, z0, z1, lpa * kPageTokens + 2 * (lane & 3),
                                 (lpa + kTcWarps) * kPageTokens + 2 * (lane & 3), T, p.scale_log2, lane, psum);
                if constexpr (kAttn) {
                    if (va) record_mass(lpa, psum[0][0], psum[0][1]);
                    if (vb) record_mass(lpa + kTcWarps, psum[1][0], psum[1][1]);
                }
            }
        }
        const int lp = p0 + warp + kTcWarps * i;
        const int phys = phys_of(i);
        if (!kI8 && phys >= 0 && phys < p.num_pages) {
            if (lp == lp_new) {  // fused append: patch the new rows into the staged tiles
                const int kv = lane >> 4, c = lane & 15;
                const uint8_t *src = (kv ? p.new_v : p.new_k) + ((size_t)s * p.hkv + kvh) * 256;
                uint8_t *tile = wbuf + st * kTcStage + kv * 2 * kBox + (c >> 3) * kBox;
                *reinterpret_cast<uint4 *>(tile + swz(slot_new, c & 7)) =
                    reinterpret_cast<const uint4 *>(src)[c];
                __syncwarp();
            }
            float ps0_, ps1_;
            tc_page<kBig>(sbase, qa, qlo, o, m0, m1, l0, l1, lp * kPageTokens + 2 * (lane & 3), T,
                          p.scale_log2, lane, ps0_, ps1_);
            if constexpr (kAttn) record_mass(lp, ps0_, ps1_);
        }
        __syncwarp();
        if (lane == 0 && i + kTcStages < n_my) {
            fence_proxy_async_smem();
            issue(i + kTcStages, st);
        }
    }

    // Streaming done: wait for the previous launch before touching the split
    // workspace, the output or the appended slot, which it may still be using.
    grid_dependency_wait();
    if (appends) {
        if (warp == 0) {
            const int phys = p.block_table[(size_t)s * p.max_pages + (size_t)lp_new];
            if (phys >= 0 && phys < p.num_pages) {
                const int kv = lane >> 4, e = lane & 15;  // 2 rows x 16 vectors of 16 B
                const uint8_t *src = (kv ? p.new_v : p.new_k) + ((size_t)s * p.hkv + kvh) * 256;
                uint8_t *dst = const_cast<uint8_t *>(p.pool) +
                               ((((size_t)phys * 2 + kv) * p.hkv + kvh) * kPageTokens + slot_new) * 256;
                reinterpret_cast<uint4 *>(dst)[e] = reinterpret_cast<const uint4 *>(src)[e];
                __threadfence();
            } else if (p.error_flag && lane == 0) {
                atomicOr(p.error_flag, 2);
            }
        }
        __syncthreads();
        grid_dependents_launch();
    }
    if (threadIdx.x == 0) s_flag[0] = 0;
    __syncthreads();
    if (!ok) {
        for (int i = done; i < min(done + kTcStages, n_my); ++i)
            (void)mbar_wait_bounded(&bars[i % kTcStages], (i / kTcStages) & 1, nullptr);
        if (lane == 0) s_flag[0] = 1;
    }
    __syncthreads();
    if (s_flag[0]) {
        if (nsplit > 1 && threadIdx.x == 0) {
            int *ctr = p.counters + (size_t)s * p.hkv + kvh;
            if (atomicAdd(ctr, 1) == nsplit - 1) atomicExch(ctr, 0);
        }
        return;
    }

    // ---- merge the 4 warps: each parks O (fp32 [16 rows][128]) in its stage 0
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    if constexpr (kBig) {
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    }
    float *wacc = reinterpret_cast<float *>(wbuf);
    if constexpr (kI8) {
        z0 += __shfl_xor_sync(0xffffffffu, z0, 1);
        z0 += __shfl_xor_sync(0xffffffffu, z0, 2);
        z1 += __shfl_xor_sync(0xffffffffu, z1, 1);
        z1 += __shfl_xor_sync(0xffffffffu, z1, 2);
#pragma unroll
        for (int n = 0; n < 16; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = 16 * (n >> 1) + 2 * (2 * tq + e) + (n & 1);
                if constexpr (kBig) {
                    wacc[park_ofs<true>(gq, d)] = o[n][e] + z0;
                    wacc[park_ofs<true>(gq + 8, d)] = o[n][2 + e] + z1;
                } else {
                    wacc[park_ofs<true>(gq, d)] = (o[n][e] + o[n][2 + e]) + z0;
                }
            }
    } else {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            *reinterpret_cast<float2 *>(wacc + gq * kHeadDim + 8 * n + 2 * tq) = make_float2(o[n][0], o[n][1]);
            if constexpr (kBig)
                *reinterpret_cast<float2 *>(wacc + (gq + 8) * kHeadDim + 8 * n + 2 * tq) =
                    make_float2(o[n][2], o[n][3]);
        }
    }
    if (tq == 0) {
        s_m[warp * 16 + gq] = m0;
        s_l[warp * 16 + gq] = l0;
        s_m[warp * 16 + gq + 8] = kBig ? m1 : -CUDART_INF_F;
        s_l[warp * 16 + gq + 8] = kBig ? l1 : 0.f;
    }
    __syncthreads();
    // per row, once: the maximum M over the warps, each warp's weight
    // exp2(m_w - M) (written over m_w) and the merged L, M (over l_0, l_1).
    // Thread g owns every entry of row g, so the rewrite is race free.
    if (threadIdx.x < 16) {
        const int g = threadIdx.x;
        float mw[kTcWarps], M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, mw[w] = s_m[w * 16 + g]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) {
            const float sw = mw[w] == -CUDART_INF_F ? 0.f : exp2f(mw[w] - M);
            L += sw * s_l[w * 16 + g];
            s_m[w * 16 + g] = sw;
        }
        s_l[g] = L;
        s_l[16 + g] = M;
    }
    __syncthreads();
    // a thread per (row, 4 dims): the warps' parked O weighted and summed in
    // warp order
    for (int idx = threadIdx.x; idx < nh * (kHeadDim / 4); idx += kTcThreads) {
        const int g = idx / (kHeadDim / 4), d = 4 * (idx % (kHeadDim / 4));
        float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) {
            const float sw = s_m[w * 16 + g];
            const float *pw = reinterpret_cast<const float *>(smem + w * kTcStages * kTcStage);
            if constexpr (kI8) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o4[e] += sw * pw[park_ofs<true>(g, d + e)];
            } else {
                const float4 v = *reinterpret_cast<const float4 *>(pw + park_ofs<false>(g, d));
                o4[0] += sw * v.x;
                o4[1] += sw * v.y;
                o4[2] += sw * v.z;
                o4[3] += sw * v.w;
            }
        }
        const float L = s_l[g], M = s_l[16 + g];
        const int h = h0 + g;
        if (nsplit == 1) {
            QT *out = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h) * kHeadDim + d;
            const float inv_l = 1.f / L;
#pragma unroll
            for (int e = 0; e < 4; ++e) io_traits<QT>::store(out + e, o4[e] * inv_l);
            if (kAttn && d == 0)
                *reinterpret_cast<float2 *>(p.attn_ml + ((size_t)s * p.hq + h) * 2) = make_float2(M, L);
        } else {
            const size_t pi = ((size_t)s * p.hq + h) * p.max_splits + split;
            *reinterpret_cast<float4 *>(p.part_o + pi * kHeadDim + d) = make_float4(o4[0], o4[1], o4[2], o4[3]);
            if (d == 0) {
                p.part_ml[pi * 2] = M;
                p.part_ml[pi * 2 + 1] = L;
            }
        }
    }
    if (nsplit == 1) return;

    // ---- last CTA of (sequence, kv-head) folds the splits
    __syncthreads();
    if (threadIdx.x == 0) {  // release this CTA's partials, acquire the others if last
        int *ctr = p.counters + (size_t)s * p.hkv + kvh;
        const int ticket = atomic_add_acq_rel(ctr, 1);
        const int last = ticket == nsplit - 1;
        if (last) atomicExch(ctr, 0);
        s_flag[1] = last;
    }
    __syncthreads();
    if (!s_flag[1]) return;
    if (nh * nsplit <= kCombineFloats) {
        // the splits' weights exp2(m_c - M) and each row's M and L once, in
        // the (now idle) staging ring: one warp per row, lanes over splits
        float *wts = reinterpret_cast<float *>(smem);  // [nh][nsplit]
        float *row_m = wts + kCombineFloats, *row_l = row_m + 16;
        for (int g = warp; g < nh; g += kTcWarps) {
            const float2 *ml = reinterpret_cast<const float2 *>(p.part_ml) + ((size_t)s * p.hq + h0 + g) * p.max_splits;
            float mx = -CUDART_INF_F;
            for (int c = lane; c < nsplit; c += 32) mx = fmaxf(mx, __ldcg(&ml[c].x));
#pragma unroll
            for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            float l = 0.f;
            for (int c = lane; c < nsplit; c += 32) {
                const float2 v = __ldcg(ml + c);
                const float w = v.x == -CUDART_INF_F ? 0.f : exp2f(v.x - mx);
                wts[g * nsplit + c] = w;
                l += w * v.y;
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            if (lane == 0) {
                row_m[g] = mx;
                row_l[g] = l;
            }
        }
        __syncthreads();
        // O: a thread per (row, 4 dims), the splits' partial sums read in
        // groups of 8 (float4), summed in split order
        for (int idx = threadIdx.x; idx < nh * (kHeadDim / 4); idx += kTcThreads) {
            const int g = idx / (kHeadDim / 4), d4 = idx % (kHeadDim / 4);
            const size_t base = ((size_t)s * p.hq + h0 + g) * p.max_splits;
            const float4 *po = reinterpret_cast<const float4 *>(p.part_o + base * kHeadDim) + d4;
            const float *w = wts + g * nsplit;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            auto add = [&](float wc, float4 v) {
                o.x += wc * v.x;
                o.y += wc * v.y;
                o.z += wc * v.z;
                o.w += wc * v.w;
            };
            int c = 0;
            for (; c + 8 <= nsplit; c += 8) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(po + (size_t)(c + u) * (kHeadDim / 4));
#pragma unroll
                for (int u = 0; u < 8; ++u) add(w[c + u], v[u]);
            }
            for (; c < nsplit; ++c) add(w[c], __ldcg(po + (size_t)c * (kHeadDim / 4)));
            const float inv_l = 1.f / row_l[g];
            QT *out = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h0 + g) * kHeadDim + 4 * d4;
            io_traits<QT>::store(out + 0, o.x * inv_l);
            io_traits<QT>::store(out + 1, o.y * inv_l);
            io_traits<QT>::store(out + 2, o.z * inv_l);
            io_traits<QT>::store(out + 3, o.w * inv_l);
            if (kAttn && d4 == 0)
                *reinterpret_cast<float2 *>(p.attn_ml + ((size_t)s * p.hq + h0 + g) * 2) =
                    make_float2(row_m[g], row_l[g]);
        }
        return;
    }
    for (int idx = threadIdx.x; idx < nh * kHeadDim; idx += kTcThreads) {
        const int g = idx / kHeadDim, d = idx % kHeadDim;
        const size_t base = ((size_t)s * p.hq + h0 + g) * p.max_splits;
        float M, L;
        const float O = fold_splits(p.part_ml, p.part_o, base, nsplit, d, M, L);
        QT *out = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h0 + g) * kHeadDim;
        io_traits<QT>::store(out + d, O / L);
        if (kAttn && d == 0)
            *reinterpret_cast<float2 *>(p.attn_ml + ((size_t)s * p.hq + h0 + g) * 2) = make_float2(M, L);
    }
}

template <typename QT, bool kBig, bool kI8, bool kAttn>
__global__ void __launch_bounds__(kTcThreads, 3)
tc_decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tm) {
    tc_decode_body<QT, kBig, kI8, kAttn>(p, tm);
    if (p.done) grid_done_signal(p.done, p.epoch);  // every exit of the body is CTA-uniform
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// 2D view of the pool: rows of 128 fp16 (one token of one (page, K|V, head)
// block), box = 64 dims x 16 tokens, 128-byte swizzle.
bool make_pool_map(CUtensorMap *tm, const void *pool, long long rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || rows <= 0 || rows > (1ll << 31)) return false;
    cuuint64_t gdim[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)kHeadDim * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kPageTokens};
    cuuint32_t estride[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(pool), gdim, gstride, box,
              estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2D view of an int8 pool: rows of 128 codes, box = 128 x 16 bytes (one
// (page, K|V, head) block), 128-byte swizzle.
bool make_pool_map_i8(CUtensorMap *tm, const void *pool, long long rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || rows <= 0 || rows > (1ll << 31)) return false;
    cuuint64_t gdim[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)kHeadDim};
    cuuint32_t box[2] = {(cuuint32_t)kHeadDim, (cuuint32_t)kPageTokens};
    cuuint32_t estride[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(pool), gdim, gstride, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename QT, bool kBig, bool kI8, bool kAttn>
int launch_tc(const DecodeParams &p, int batch, cudaStream_t st, const CUtensorMap &tm) {
    auto kern = tc_decode_kernel<QT, kBig, kI8, kAttn>;
    constexpr int smem = TcCfg<kI8>::kSmem;
    static std::atomic<bool> attr_done[kMaxDevices];
    if (ensure_smem_attr(attr_done, kern, smem) != KVX_OK) return KVX_ECUDA;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.max_splits, p.hkv, batch);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = kAttn ? 0 : 1;  // plain decode only
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, p, tm) != cudaSuccess) {
        cudaGetLastError();
        return KVX_ECUDA;
    }
    return launch_status();
}

template <bool kI8, bool kAttn>
int launch_tc_io2(const DecodeParams &p, int io_dtype, int batch, cudaStream_t st, const CUtensorMap &tm) {
    const bool big = p.group > 8;
    if (io_dtype == KVX_F32)
        return big ? launch_tc<float, true, kI8, kAttn>(p, batch, st, tm)
                   : launch_tc<float, false, kI8, kAttn>(p, batch, st, tm);
    return big ? launch_tc<__half, true, kI8, kAttn>(p, batch, st, tm)
               : launch_tc<__half, false, kI8, kAttn>(p, batch, st, tm);
}

// Attention-mass recording is a separate instantiation, so the plain
// decode carries none of its code.
template <bool kI8>
int launch_tc_io(const DecodeParams &p, int io_dtype, int batch, cudaStream_t st, const CUtensorMap &tm) {
    return p.attn_pm ? launch_tc_io2<kI8, true>(p, io_dtype, batch, st, tm)
                     : launch_tc_io2<kI8, false>(p, io_dtype, batch, st, tm);
}

}  // namespace

int launch_decode_tc(DecodeParams &p, int kv_dtype, int io_dtype, int batch, cudaStream_t st) {
    if (p.group > 16) return KVX_EUNSUPPORTED;
    if (kv_dtype == KVX_I8 && (p.positions || !p.stats)) return KVX_EUNSUPPORTED;
    CUtensorMap tm;
    const long long rows = (long long)p.num_pages * 2 * p.hkv * kPageTokens;
    if (kv_dtype == KVX_I8) {
        if (!make_pool_map_i8(&tm, p.pool, rows)) return KVX_EUNSUPPORTED;
        return launch_tc_io<true>(p, io_dtype, batch, st, tm);
    }
    if (kv_dtype != KVX_F16 || !make_pool_map(&tm, p.pool, rows)) return KVX_EUNSUPPORTED;
    return launch_tc_io<false>(p, io_dtype, batch, st, tm);
}

}  // namespace kvx
