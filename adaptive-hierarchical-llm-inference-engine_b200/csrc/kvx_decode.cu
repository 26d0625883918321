// kvx_decode.cu -- paged GQA decode attention for sm_100a.
//
// Semantics: TensorOps::attention (runtime/tensor_ops.cpp:179-219) for one
// query row per (sequence, q-head), scale 1/sqrt(head_dim), over the tokens
// of the sequence gathered through its block table; q-head h reads kv-head
// h / (num_q_heads / num_kv_heads).
//
// Design (memory bound: every K/V byte is read once per step):
//  * grid = (head_group x split, kv_head, sequence).  A split is a chunk of
//    `chunk` consecutive logical pages; one CTA of 4 warps owns it and its
//    warps take the chunk's pages round-robin.
//  * Each warp streams its pages through a private 2-stage shared-memory
//    ring: lane 0 issues two bulk copies (cp.async.bulk, the TMA engine; K
//    block + V block of one (page, head), 4 KiB each at fp16) that complete
//    on an mbarrier; all lanes wait with a bounded poll.  No register
//    staging, one instruction per 4 KiB.
//  * Q.K: lane (grp = lane/8, sub = lane%8) owns 16 dims (two 16-byte
//    vectors per row); the 8 lanes of a group read one 128-byte segment of a
//    row per instruction (bank-conflict free) and reduce with 3 shuffles.
//    Softmax is online in the log2 domain (q pre-scaled by scale*log2 e).
//  * P.V: lane owns 4 output dims; one row per instruction, conflict free.
//  * Warps merge through shared memory.  A sequence with one split writes
//    its rows directly; otherwise every split writes (m, l, o) partials and
//    takes a ticket on a per-(sequence, kv-head, head-group) counter; the
//    last CTA to arrive folds the splits (flash-decoding combine) and resets
//    the counter to zero, so no second launch is needed.
//  * Fused append (kvx_append_decode): the token at positions[s] is written
//    into its page by one CTA, and every CTA that reads that page patches
//    the row into its shared-memory copy, so readers never depend on the
//    write landing first.
//  * int8 pages: the (page, head) block's {scale, zeroPoint} rides in the
//    same bulk transfer; dequantisation is folded algebraically:
//    q.(zp + c*s) = zp*sum(q) + s*(q.c), p.(zp + c*s) = zp*sum(p) + (p*s).c.
#include <cuda_fp16.h>
#include <math_constants.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "kvx_common.cuh"
#include "kvx_decode_params.cuh"

namespace kvx {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxHeadsPerCta = 4;



template <typename KVT> struct KvTraits;
// kVec: elements per 16-byte vector; kStages: ring depth per warp (fp32
// pages are 32 KiB per stage, so one stage keeps a CTA inside 227 KB).
template <> struct KvTraits<float> {
    static constexpr int kVec = 4;
    static constexpr bool kI8 = false;
    static constexpr int kStages = 1;
};
template <> struct KvTraits<__half> {
    static constexpr int kVec = 8;
    static constexpr bool kI8 = false;
    static constexpr int kStages = 2;
};
template <> struct KvTraits<int8_t> {
    static constexpr int kVec = 16;
    static constexpr bool kI8 = true;
    static constexpr int kStages = 3;
};

// 16 bytes of K/V elements -> kVec floats (int8: code + 128, exact).
template <typename KVT> __device__ __forceinline__ void unpack16(const uint4 &w, float *f);
template <> __device__ __forceinline__ void unpack16<float>(const uint4 &w, float *f) {
    f[0] = __uint_as_float(w.x);
    f[1] = __uint_as_float(w.y);
    f[2] = __uint_as_float(w.z);
    f[3] = __uint_as_float(w.w);
}
template <> __device__ __forceinline__ void unpack16<__half>(const uint4 &w, float *f) {
    float2 a = h2_to_f2(w.x), b = h2_to_f2(w.y), c = h2_to_f2(w.z), d = h2_to_f2(w.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
// int8 code c (two's complement byte) -> float(c + 128): flip the sign bit
// to get the unsigned byte, place it in the mantissa of 2^23 and subtract.
__device__ __forceinline__ void unpack_u8x4(uint32_t w, float *f) {
    uint32_t u = w ^ 0x80808080u;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        f[i] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u | i)) - 8388608.0f;
}
template <> __device__ __forceinline__ void unpack16<int8_t>(const uint4 &w, float *f) {
    unpack_u8x4(w.x, f);
    unpack_u8x4(w.y, f + 4);
    unpack_u8x4(w.z, f + 8);
    unpack_u8x4(w.w, f + 12);
}

// 4 consecutive elements of a V row -> floats.
template <typename KVT> __device__ __forceinline__ void load_v4(const KVT *row, int lane, float *f);
template <> __device__ __forceinline__ void load_v4<float>(const float *row, int lane, float *f) {
    float4 v = *reinterpret_cast<const float4 *>(row + 4 * lane);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <> __device__ __forceinline__ void load_v4<__half>(const __half *row, int lane, float *f) {
    uint2 v = *reinterpret_cast<const uint2 *>(row + 4 * lane);
    float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <> __device__ __forceinline__ void load_v4<int8_t>(const int8_t *row, int lane, float *f) {
    unpack_u8x4(*reinterpret_cast<const uint32_t *>(row + 4 * lane), f);
}

template <typename KVT> __host__ __device__ constexpr int block_bytes() { return kPageTokens * kHeadDim * (int)sizeof(KVT); }
template <typename KVT> __host__ __device__ constexpr int stage_bytes() {
    return 2 * block_bytes<KVT>() + (KvTraits<KVT>::kI8 ? 32 : 0);
}
template <typename KVT> __host__ __device__ constexpr int smem_bytes() {
    constexpr int kStages = KvTraits<KVT>::kStages;
    return kWarps * kStages * stage_bytes<KVT>() + kWarps * kStages * 8 +
           kWarps * kMaxHeadsPerCta * kPageTokens * 4 + 2 * kWarps * kMaxHeadsPerCta * 4;
}

template <typename KVT, typename QT, int G>
__device__ __forceinline__ void
paged_decode_body(const DecodeParams &p) {
    using TR = KvTraits<KVT>;
    constexpr int kVec = TR::kVec;
    constexpr int kNv = 16 / kVec;                // 16-byte vectors per lane per K row
    constexpr int kBlk = block_bytes<KVT>();
    constexpr int kStage = stage_bytes<KVT>();
    constexpr int kRowBytes = kHeadDim * (int)sizeof(KVT);
    constexpr int kStages = TR::kStages;

    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane >> 3, sub = lane & 7;
    const int hg = blockIdx.x % p.nhg, split = blockIdx.x / p.nhg;
    const int kvh = blockIdx.y, s = blockIdx.z;
    const bool fused = p.positions != nullptr;
    int T = fused ? p.positions[s] + 1 : max(p.seq_lens[s], 0);
    if (fused && T <= 0) T = 0;
    if (T > p.max_pages * kPageTokens) {  // context longer than the block table row
        if (p.error_flag && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
            atomicOr(p.error_flag, 4);
        T = p.max_pages * kPageTokens;
    }
    const int npages = (T + kPageTokens - 1) / kPageTokens;
    const int p0 = split * p.chunk;
    const int h0 = kvh * p.group + hg * G;  // first q-head of this CTA
    const int nh = min(G, p.group - hg * G);
    if (p0 >= npages) {  // whole CTA: this split is past the sequence
        if (npages == 0 && split == 0) {  // empty context: zero rows (no attention)
            QT *o = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h0) * kHeadDim;
            for (int i = threadIdx.x; i < nh * kHeadDim; i += kThreads) io_traits<QT>::store(o + i, 0.f);
        }
        return;
    }
    const int p1 = min(p0 + p.chunk, npages);
    const int nsplit = (npages + p.chunk - 1) / p.chunk;

    uint8_t *wbuf = smem + warp * kStages * kStage;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kWarps * kStages * kStage) + warp * kStages;
    float *sp = reinterpret_cast<float *>(smem + kWarps * kStages * kStage + kWarps * kStages * 8) +
                warp * kMaxHeadsPerCta * kPageTokens;
    float *s_m = reinterpret_cast<float *>(smem + kWarps * kStages * kStage + kWarps * kStages * 8 +
                                           kWarps * kMaxHeadsPerCta * kPageTokens * 4);
    float *s_l = s_m + kWarps * kMaxHeadsPerCta;

    if (lane == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
    }
    __syncwarp();

    constexpr int kRowVecs = kRowBytes / 16;
    // page / slot of the appended token (none when its position is out of range)
    const bool append_ok = fused && p.positions[s] >= 0 && p.positions[s] < p.max_pages * kPageTokens;
    const int lp_new = append_ok ? p.positions[s] / kPageTokens : -1;
    const int slot_new = append_ok ? p.positions[s] % kPageTokens : 0;
    if constexpr (!TR::kI8) {
        if (fused && hg == 0 && lp_new >= p0 && lp_new < p1 && warp == 0) {
            const int phys = p.block_table[(size_t)s * p.max_pages + lp_new];
            if (phys >= 0 && phys < p.num_pages) {
                for (int v = lane; v < 2 * kRowVecs; v += 32) {
                    const int kv = v / kRowVecs, e = v % kRowVecs;
                    const uint8_t *src = (kv ? p.new_v : p.new_k) + ((size_t)s * p.hkv + kvh) * kRowBytes;
                    uint8_t *dst = const_cast<uint8_t *>(p.pool) +
                                   ((((size_t)phys * 2 + kv) * p.hkv + kvh) * kPageTokens + slot_new) * kRowBytes;
                    reinterpret_cast<uint4 *>(dst)[e] = reinterpret_cast<const uint4 *>(src)[e];
                }
            } else if (p.error_flag && lane == 0) {
                atomicOr(p.error_flag, 2);
            }
        }
    }

    const int n_my = (p1 - p0 - warp + kWarps - 1) / kWarps;  // pages of this warp
    const int32_t *bt = p.block_table + (size_t)s * p.max_pages;

    auto issue = [&](int i, int st) {
        const int lp = p0 + warp + kWarps * i;
        const int phys = bt[lp];
        uint64_t *bar = &bars[st];
        if (phys < 0 || phys >= p.num_pages) {
            if (p.error_flag) atomicOr(p.error_flag, 2);
            mbar_arrive_expect_tx(bar, 0);  // completes the phase with no data
            return;
        }
        const size_t kb = ((size_t)phys * 2) * p.hkv + kvh;
        const size_t vb = kb + p.hkv;
        uint8_t *dst = wbuf + st * kStage;
        mbar_arrive_expect_tx(bar, kStage);
        bulk_g2s(dst, p.pool + kb * kBlk, kBlk, bar);
        bulk_g2s(dst + kBlk, p.pool + vb * kBlk, kBlk, bar);
        if constexpr (TR::kI8) {
            bulk_g2s(dst + 2 * kBlk, p.stats + kb * 4, 16, bar);
            bulk_g2s(dst + 2 * kBlk + 16, p.stats + vb * 4, 16, bar);
        }
    };

    if (lane == 0)
        for (int i = 0; i < min(kStages, n_my); ++i) issue(i, i);

    // q for this lane's dims, pre-scaled into the log2 domain.
    float qv[G][16];
    float qsum[G];
    {
        const QT *qb = reinterpret_cast<const QT *>(p.q) + ((size_t)s * p.hq + h0) * kHeadDim;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            qsum[g] = 0.f;
#pragma unroll
            for (int j = 0; j < kNv; ++j)
#pragma unroll
                for (int e = 0; e < kVec; ++e) {
                    const int d = (sub + 8 * j) * kVec + e;
                    float v = g < nh ? io_traits<QT>::load(qb + g * kHeadDim + d) * p.scale_log2 : 0.f;
                    qv[g][j * kVec + e] = v;
                    qsum[g] += v;
                }
            if constexpr (TR::kI8) {
                qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 1);
                qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 2);
                qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 4);
            }
        }
    }

    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -CUDART_INF_F;
        l[g] = 0.f;
        acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    }

    bool ok = true;
    int done = 0;
    for (int i = 0; i < n_my; ++i) {
        const int st = i % kStages;
        const uint32_t par = (i / kStages) & 1;
        if (!mbar_wait_bounded(&bars[st], par, p.error_flag)) {
            ok = false;
            break;
        }
        done = i + 1;
        const int lp = p0 + warp + kWarps * i;
        const int phys = bt[lp];
        if (phys >= 0 && phys < p.num_pages) {
            const uint8_t *kbuf = wbuf + st * kStage;
            if constexpr (!TR::kI8) {
                if (lp == lp_new) {  // fused append: patch the new row into smem
                    uint8_t *kb = wbuf + st * kStage;
                    for (int v = lane; v < 2 * kRowVecs; v += 32) {
                        const int kv = v / kRowVecs, e = v % kRowVecs;
                        const uint8_t *src = (kv ? p.new_v : p.new_k) + ((size_t)s * p.hkv + kvh) * kRowBytes;
                        reinterpret_cast<uint4 *>(kb + kv * kBlk + slot_new * kRowBytes)[e] =
                            reinterpret_cast<const uint4 *>(src)[e];
                    }
                    __syncwarp();
                }
            }
            const KVT *Vs = reinterpret_cast<const KVT *>(kbuf + kBlk);
            float kscale = 1.f, kzp = 0.f, vscale = 1.f, vzp = 0.f;
            if constexpr (TR::kI8) {
                const float4 ks = *reinterpret_cast<const float4 *>(kbuf + 2 * kBlk);
                const float4 vs = *reinterpret_cast<const float4 *>(kbuf + 2 * kBlk + 16);
                kscale = ks.z; kzp = ks.w; vscale = vs.z; vzp = vs.w;
            }
            // ---- scores for rows grp, grp+4, grp+8, grp+12 ----
            float sc[4][G];
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const int r = grp + 4 * r4;
                float kf[16];
#pragma unroll
                for (int j = 0; j < kNv; ++j) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(kbuf + r * kRowBytes + (sub + 8 * j) * 16);
                    unpack16<KVT>(w, kf + j * kVec);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float a = 0.f;
#pragma unroll
                    for (int e = 0; e < 16; ++e) a = fmaf(qv[g][e], kf[e], a);
                    sc[r4][g] = a;
                }
            }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1)
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4)
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        sc[r4][g] += __shfl_xor_sync(0xffffffffu, sc[r4][g], off);
            const int tok0 = lp * kPageTokens;
            float mx[G];
#pragma unroll
            for (int g = 0; g < G; ++g) mx[g] = -CUDART_INF_F;
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const bool valid = tok0 + grp + 4 * r4 < T;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float v = sc[r4][g];
                    if constexpr (TR::kI8) v = fmaf(kscale, v, kzp * qsum[g]);
                    v = valid ? v : -CUDART_INF_F;
                    sc[r4][g] = v;
                    mx[g] = fmaxf(mx[g], v);
                }
            }
            float alpha[G], psum[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], 8));
                mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], 16));
                const float mn = fmaxf(m[g], mx[g]);
                alpha[g] = exp2f(m[g] - mn);
                m[g] = mn;
                psum[g] = 0.f;
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4) {
                    const float e = exp2f(sc[r4][g] - mn);
                    sc[r4][g] = e;
                    psum[g] += e;
                }
                l[g] = l[g] * alpha[g] + psum[g];
            }
            if (sub == 0) {
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4)
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        sp[g * kPageTokens + grp + 4 * r4] = sc[r4][g] * (TR::kI8 ? vscale : 1.f);
            }
            __syncwarp();
            // ---- P.V ----
            float pz[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                acc[g][0] *= alpha[g]; acc[g][1] *= alpha[g];
                acc[g][2] *= alpha[g]; acc[g][3] *= alpha[g];
                pz[g] = 0.f;
            }
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                float pt[G][4];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 v = *reinterpret_cast<const float4 *>(sp + g * kPageTokens + 4 * t4);
                    pt[g][0] = v.x; pt[g][1] = v.y; pt[g][2] = v.z; pt[g][3] = v.w;
                }
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    float vf[4];
                    load_v4<KVT>(Vs + (4 * t4 + tt) * kHeadDim, lane, vf);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        acc[g][0] = fmaf(pt[g][tt], vf[0], acc[g][0]);
                        acc[g][1] = fmaf(pt[g][tt], vf[1], acc[g][1]);
                        acc[g][2] = fmaf(pt[g][tt], vf[2], acc[g][2]);
                        acc[g][3] = fmaf(pt[g][tt], vf[3], acc[g][3]);
                    }
                }
            }
            if constexpr (TR::kI8) {
                // zp * sum_t p_t, added to every dim (p without the scale factor)
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float zp_add = vzp * psum[g];
                    // psum is this lane group's 4 rows; total over the 4 groups
                    float z = zp_add + __shfl_xor_sync(0xffffffffu, zp_add, 8);
                    z += __shfl_xor_sync(0xffffffffu, z, 16);
                    pz[g] = z;
                    acc[g][0] += pz[g]; acc[g][1] += pz[g]; acc[g][2] += pz[g]; acc[g][3] += pz[g];
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + kStages < n_my) {
            fence_proxy_async_smem();
            issue(i + kStages, st);
        }
    }
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    if (!ok) {
        // Drain copies this warp may still have in flight; the CTA then
        // leaves this split unwritten (error_flag is set).
        for (int i = done; i < min(done + kStages, n_my); ++i)
            (void)mbar_wait_bounded(&bars[i % kStages], (i / kStages) & 1, nullptr);
        if (lane == 0) s_fail = 1;
    }
    __syncthreads();
    if (s_fail) {
        if (nsplit > 1 && threadIdx.x == 0) {
            int *ctr = p.counters + ((size_t)s * p.hkv + kvh) * p.nhg + hg;
            if (atomicAdd(ctr, 1) == nsplit - 1) atomicExch(ctr, 0);
        }
        return;
    }

    // ---- merge the warps of the CTA ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
        l[g] += __shfl_xor_sync(0xffffffffu, l[g], 8);
        l[g] += __shfl_xor_sync(0xffffffffu, l[g], 16);
    }
    // each warp parks its accumulator in its own (now idle) stage buffer
    float *wacc = reinterpret_cast<float *>(wbuf);
#pragma unroll
    for (int g = 0; g < G; ++g)
        *reinterpret_cast<float4 *>(wacc + g * kHeadDim + 4 * lane) =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            s_m[warp * kMaxHeadsPerCta + g] = m[g];
            s_l[warp * kMaxHeadsPerCta + g] = l[g];
        }
    }
    __syncthreads();
    // per head, once: the maximum M over the warps, each warp's weight
    // exp2(m_w - M) (written over m_w) and the merged L, M (over l_0, l_1).
    // Thread g owns every entry of head g, so the rewrite is race free.
    if (threadIdx.x < nh) {
        const int g = threadIdx.x;
        float mw[kWarps], M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w] = s_m[w * kMaxHeadsPerCta + g]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float sw = mw[w] == -CUDART_INF_F ? 0.f : exp2f(mw[w] - M);
            L += sw * s_l[w * kMaxHeadsPerCta + g];
            s_m[w * kMaxHeadsPerCta + g] = sw;
        }
        s_l[g] = L;
        s_l[kMaxHeadsPerCta + g] = M;
    }
    __syncthreads();
    // a thread per (head, 4 dims): the warps' parked accumulators weighted
    // and summed in warp order
    for (int idx = threadIdx.x; idx < nh * (kHeadDim / 4); idx += kThreads) {
        const int g = idx / (kHeadDim / 4), d = 4 * (idx % (kHeadDim / 4));
        float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float sw = s_m[w * kMaxHeadsPerCta + g];
            const float4 v = *reinterpret_cast<const float4 *>(
                reinterpret_cast<const float *>(smem + w * kStages * kStage) + g * kHeadDim + d);
            o4.x += sw * v.x;
            o4.y += sw * v.y;
            o4.z += sw * v.z;
            o4.w += sw * v.w;
        }
        const float L = s_l[g], M = s_l[kMaxHeadsPerCta + g];
        const int h = h0 + g;
        if (nsplit == 1) {
            QT *o = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h) * kHeadDim + d;
            const float inv_l = 1.f / L;
            io_traits<QT>::store(o + 0, o4.x * inv_l);
            io_traits<QT>::store(o + 1, o4.y * inv_l);
            io_traits<QT>::store(o + 2, o4.z * inv_l);
            io_traits<QT>::store(o + 3, o4.w * inv_l);
        } else {
            const size_t pi = ((size_t)s * p.hq + h) * p.max_splits + split;
            *reinterpret_cast<float4 *>(p.part_o + pi * kHeadDim + d) = o4;
            if (d == 0) {
                p.part_ml[pi * 2] = M;
                p.part_ml[pi * 2 + 1] = L;
            }
        }
    }
    if (nsplit == 1) return;

    // ---- split combine by the last CTA of this (sequence, kv-head, head-group)
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {  // release this CTA's partials, acquire the others if last
        int *ctr = p.counters + ((size_t)s * p.hkv + kvh) * p.nhg + hg;
        const int ticket = atomic_add_acq_rel(ctr, 1);
        s_last = ticket == nsplit - 1;
        if (s_last) atomicExch(ctr, 0);  // every split has arrived: reset for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    for (int idx = threadIdx.x; idx < nh * kHeadDim; idx += kThreads) {
        const int g = idx / kHeadDim, d = idx % kHeadDim;
        const size_t base = ((size_t)s * p.hq + h0 + g) * p.max_splits;
        float M, L;
        const float O = fold_splits(p.part_ml, p.part_o, base, nsplit, d, M, L);
        QT *o = reinterpret_cast<QT *>(p.out) + ((size_t)s * p.hq + h0 + g) * kHeadDim;
        io_traits<QT>::store(o + d, O / L);
    }
}

template <typename KVT, typename QT, int G>
__global__ void __launch_bounds__(kThreads)
paged_decode_kernel(const DecodeParams p) {
    paged_decode_body<KVT, QT, G>(p);
    if (p.done) grid_done_signal(p.done, p.epoch);  // every exit of the body is CTA-uniform
}

constexpr int kMinChunk = 4;

int choose_chunk(int batch, int hkv, int nhg, int max_pages) {
    if (const char *e = getenv("KVX_DECODE_CHUNK")) {
        int c = atoi(e);
        if (c >= kMinChunk) return c;
    }
    // SIMT kernel: aim at ~4 waves of 3 resident CTAs per SM, counting half
    // of max_pages as the mean sequence length; at least 8 pages (2 per
    // warp) and at most 32 splits per sequence, as a CTA's fixed cost and the
    // last CTA's combine outweigh more parallelism for small batches
    const long long work = (long long)batch * hkv * nhg * max_pages;
    const long long target = (long long)sm_count() * 3 * 4;
    long long c = (work / 2 + target - 1) / target;
    c = std::max<long long>(c, std::max<long long>((max_pages + 31) / 32, 8));
    if (c < kMinChunk) c = kMinChunk;
    if (c > 64) c = 64;
    return (int)((c + kWarps - 1) / kWarps * kWarps);
}

// Tensor-core decode: the largest chunk that still leaves about two waves
// of resident CTAs (3 per SM), counting half of max_pages as the mean
// sequence length -- twice that for GQA groups above 4, at least 64 pages
// and at most 32 splits per sequence -- then evened out over the longest
// sequence's splits.
// Every CTA pays a fixed cost (q fragments, pipeline fill, the merge of its
// warps, the split combine), so fewer and longer CTAs win while all SMs stay
// busy; programmatic dependent launch lets the next launch fill the SMs
// that one launch's last wave leaves idle.  page_scale > 1 for pages that
// carry less data each (int8: half the bytes, the same per-page cost).
//
// When that choice launches at most 3 waves, wave quantisation decides: 512
// CTAs on 444 resident slots (1.15 waves) leave the second wave at 15 %
// occupancy and ran 20-25 % slower than 352 or 704 CTAs of the same work
// (B4 x 16384, B8 x 8192).  Those launches instead take the chunk that
// minimises  max(1, ceil(ctas / slots)) * (chunk + 24)  -- waves times the
// length of one CTA, with 24 pages standing for its fixed cost -- over 1-32
// splits per sequence and chunks of 16-256 pages.  Larger launches keep the
// first rule: their last wave is a small part of the time.
//
// int8 pools (page_scale > 1) take the longest chunk up to 256 pages that
// still gives every SM a CTA: measured over B32 x 4096, B32 x 8192 and
// B8 x 32768 at GQA 3 and 8, 256-page CTAs ran 1.03-1.22x the chunk the rule
// above picks, and no shorter chunk beat them by more than 1 %.
int choose_chunk_tc(int batch, int hkv, int group, int max_pages, int page_scale) {
    if (const char *e = getenv("KVX_DECODE_CHUNK")) {
        int c = atoi(e);
        if (c >= kMinChunk) return c;
    }
    if (page_scale > 1) {
        const long long rows = (long long)batch * hkv;
        long long c = std::min<long long>(256, (rows * max_pages + sm_count() - 1) / sm_count());
        c = std::max<long long>(c, std::max<long long>((max_pages + 31) / 32, 64));
        const long long nsplit = (max_pages + c - 1) / c;
        c = (max_pages + nsplit - 1) / nsplit;
        return (int)((c + kWarps - 1) / kWarps * kWarps);
    }
    const long long work = (long long)batch * hkv * max_pages * page_scale;
    const long long slots = (long long)sm_count() * 3;
    const long long target = slots * 2;
    long long c = (work / 2 + target - 1) / target;
    if (group > 4) c *= 2;  // a CTA's merge and combine grow with the rows it carries
    // at most 32 splits per sequence: the last CTA folds them all (small
    // batches with long contexts), and at least 64 pages (16 per warp) a CTA
    c = std::max<long long>(c, std::max<long long>((max_pages + 31) / 32, 64));
    c = std::min<long long>(std::max<long long>(c, kMinChunk), 256);
    const long long nsplit = (max_pages + c - 1) / c;
    c = (max_pages + nsplit - 1) / nsplit;
    c = (c + kWarps - 1) / kWarps * kWarps;

    const long long rows = (long long)batch * hkv;
    auto ctas = [&](long long chunk) { return rows * ((max_pages + chunk - 1) / chunk); };
    if (ctas(c) > 3 * slots) return (int)c;
    long long best = c, best_cost = -1;
    for (int k = 1; k <= 32; ++k) {
        long long ck = (max_pages + k - 1) / k;
        ck = (ck + kWarps - 1) / kWarps * kWarps;
        if (ck > 256) continue;
        if (ck < 16 && k > 1) break;
        const long long waves = std::max<long long>(1, (ctas(ck) + slots - 1) / slots);
        const long long cost = waves * (ck + 24);
        if (best_cost < 0 || cost < best_cost) best = ck, best_cost = cost;  // ties: fewer splits
    }
    return (int)best;
}

template <typename KVT, typename QT, int G>
int launch(DecodeParams &p, int batch, cudaStream_t st) {
    auto kern = paged_decode_kernel<KVT, QT, G>;
    constexpr int smem = smem_bytes<KVT>();
    static std::atomic<bool> attr_done[kMaxDevices];
    if (ensure_smem_attr(attr_done, kern, smem) != KVX_OK) return KVX_ECUDA;
    dim3 grid(p.nhg * p.max_splits, p.hkv, batch);
    kern<<<grid, kThreads, smem, st>>>(p);
    return launch_status();
}

template <typename KVT, typename QT>
int dispatch_g(DecodeParams &p, int batch, cudaStream_t st, int G) {
    switch (G) {
    case 1: return launch<KVT, QT, 1>(p, batch, st);
    case 2: return launch<KVT, QT, 2>(p, batch, st);
    case 3: return launch<KVT, QT, 3>(p, batch, st);
    case 4: return launch<KVT, QT, 4>(p, batch, st);
    default: return KVX_EUNSUPPORTED;
    }
}

template <typename QT>
int dispatch_kv(DecodeParams &p, int dtype, int batch, cudaStream_t st, int G) {
    switch (dtype) {
    case KVX_F32: return dispatch_g<float, QT>(p, batch, st, G);
    case KVX_F16: return dispatch_g<__half, QT>(p, batch, st, G);
    case KVX_I8: return dispatch_g<int8_t, QT>(p, batch, st, G);
    default: return KVX_EINVAL;
    }
}

size_t max_splits_for(int max_pages) { return (size_t)(max_pages + kMinChunk - 1) / kMinChunk; }

size_t workspace_bytes(int batch, int hq, int max_pages) {
    const size_t splits = max_splits_for(max_pages);
    size_t b = (size_t)batch * hq * splits * (kHeadDim + 2) * sizeof(float);
    b += (size_t)batch * hq * sizeof(int32_t);  // split arrival counters
    return (b + 15) / 16 * 16;
}

int run_decode(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
               const int32_t *seq_lens, const int32_t *positions, const void *new_k,
               const void *new_v, int32_t batch, int32_t num_q_heads, const void *q, void *out,
               int32_t io_dtype, float sm_scale, void *workspace, size_t workspace_bytes_,
               int32_t *error_flag, void *stream, int min_chunk = 0, float *attn = nullptr,
               uint32_t *done = nullptr, uint32_t epoch = 0) {
    if (!kv || !kv->pool || !block_table || !q || !out) return KVX_EINVAL;
    if (!seq_lens && !positions) return KVX_EINVAL;
    if (batch <= 0 || max_pages <= 0 || kv->num_kv_heads <= 0 || num_q_heads <= 0) return KVX_EINVAL;
    if (num_q_heads % kv->num_kv_heads != 0) return KVX_EINVAL;
    if (kv->head_dim != kHeadDim || kv->page_tokens != kPageTokens) return KVX_EUNSUPPORTED;
    if (kv->dtype == KVX_I8 && !kv->stats) return KVX_EINVAL;
    if (positions && kv->dtype == KVX_I8) return KVX_EUNSUPPORTED;
    if (positions && (!new_k || !new_v)) return KVX_EINVAL;
    if (io_dtype != KVX_F32 && io_dtype != KVX_F16) return KVX_EINVAL;
    if ((reinterpret_cast<uintptr_t>(kv->pool) & 15) ||
        (kv->stats && (reinterpret_cast<uintptr_t>(kv->stats) & 15)) ||
        (reinterpret_cast<uintptr_t>(new_k) & 15) || (reinterpret_cast<uintptr_t>(new_v) & 15))
        return KVX_EINVAL;
    // min_chunk > 0 (fixed-size scratch): splits are capped at
    // ceil(max_pages / min_chunk) and the arrays are laid out for that cap
    const int min_chunk_r = min_chunk > 0 ? (min_chunk + kWarps - 1) / kWarps * kWarps : 0;
    const size_t need = min_chunk_r > 0
                            ? (size_t)batch * num_q_heads *
                                  ((size_t)(max_pages + min_chunk_r - 1) / min_chunk_r * (kHeadDim + 2) + 1) *
                                  sizeof(float)
                            : workspace_bytes(batch, num_q_heads, max_pages);
    if (!workspace || workspace_bytes_ < need) return KVX_ENOSPC;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15)) return KVX_EINVAL;

    DecodeParams p{};
    p.pool = static_cast<const uint8_t *>(kv->pool);
    p.stats = kv->stats;
    p.block_table = block_table;
    p.seq_lens = seq_lens;
    p.positions = positions;
    p.new_k = static_cast<const uint8_t *>(new_k);
    p.new_v = static_cast<const uint8_t *>(new_v);
    p.q = q;
    p.out = out;
    p.error_flag = error_flag;
    if (done && (reinterpret_cast<uintptr_t>(done) & 7)) return KVX_EINVAL;
    p.done = done;
    p.epoch = epoch;
    if (attn) {  // [batch][hq][max_pages][2] then [batch][hq][2]
        p.attn_pm = attn;
        p.attn_ml = attn + (size_t)batch * num_q_heads * max_pages * 2;
    }
    p.num_pages = kv->num_pages;
    p.hkv = kv->num_kv_heads;
    p.hq = num_q_heads;
    p.max_pages = max_pages;
    p.group = num_q_heads / kv->num_kv_heads;
    if (p.group > 4 * kMaxHeadsPerCta) return KVX_EUNSUPPORTED;
    // fp16 and int8 pools take the tensor-core kernel (all q-heads of a
    // kv-head in one CTA); fp32 pools the SIMT kernel (head groups of <= 4).
    const char *force_simt = getenv("KVX_DECODE_SIMT");
    const bool tc = (kv->dtype == KVX_F16 || kv->dtype == KVX_I8) && p.group <= 16 &&
                    !(force_simt && force_simt[0] == '1');
    p.nhg = tc ? 1 : (p.group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta;
    const int G = (p.group + p.nhg - 1) / p.nhg;
    p.chunk = std::max(tc ? choose_chunk_tc(batch, p.hkv, p.group, max_pages, kv->dtype == KVX_I8 ? 3 : 1)
                          : choose_chunk(batch, p.hkv, p.nhg, max_pages),
                       min_chunk_r);
    p.max_splits = (max_pages + p.chunk - 1) / p.chunk;
    const size_t splits_cap = min_chunk_r > 0 ? (size_t)(max_pages + min_chunk_r - 1) / min_chunk_r
                                              : max_splits_for(max_pages);
    p.part_o = static_cast<float *>(workspace);
    p.part_ml = p.part_o + (size_t)batch * num_q_heads * splits_cap * kHeadDim;
    p.counters = reinterpret_cast<int32_t *>(p.part_ml + (size_t)batch * num_q_heads * splits_cap * 2);
    const float scale = sm_scale > 0.f ? sm_scale : 1.0f / sqrtf((float)kHeadDim);
    p.scale_log2 = scale * 1.4426950408889634f;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (attn && !tc) return KVX_EUNSUPPORTED;  // attention mass: tensor-core path only
    if (tc) {
        const int rc = launch_decode_tc(p, kv->dtype, io_dtype, batch, st);
        if (rc != KVX_EUNSUPPORTED || attn) return rc;
        p.nhg = (p.group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta;  // no tensor map: SIMT kernel
        p.chunk = std::max(choose_chunk(batch, p.hkv, p.nhg, max_pages), min_chunk_r);
        p.max_splits = (max_pages + p.chunk - 1) / p.chunk;
        return io_dtype == KVX_F32 ? dispatch_kv<float>(p, kv->dtype, batch, st, (p.group + p.nhg - 1) / p.nhg)
                                   : dispatch_kv<__half>(p, kv->dtype, batch, st, (p.group + p.nhg - 1) / p.nhg);
    }
    return io_dtype == KVX_F32 ? dispatch_kv<float>(p, kv->dtype, batch, st, G)
                               : dispatch_kv<__half>(p, kv->dtype, batch, st, G);
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API size_t kvx_decode_workspace_bytes(int32_t batch, int32_t num_q_heads,
                                                     int32_t max_pages, int32_t page_tokens) {
    if (batch <= 0 || num_q_heads <= 0 || max_pages <= 0 || page_tokens != kPageTokens) return 0;
    return workspace_bytes(batch, num_q_heads, max_pages);
}

extern "C" KVX_API int kvx_decode_workspace_init(void *workspace, size_t workspace_bytes_,
                                                 void *stream) {
    if (!workspace) return KVX_EINVAL;
    return cudaMemsetAsync(workspace, 0, workspace_bytes_, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? KVX_OK
               : KVX_ECUDA;
}

extern "C" KVX_API int kvx_decode(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                                  const int32_t *seq_lens, int32_t batch, int32_t num_q_heads,
                                  const void *q, void *out, int32_t io_dtype, float sm_scale,
                                  void *workspace, size_t workspace_bytes_, int32_t *error_flag,
                                  void *stream) {
    if (!seq_lens) return KVX_EINVAL;
    return run_decode(kv, block_table, max_pages, seq_lens, nullptr, nullptr, nullptr, batch,
                      num_q_heads, q, out, io_dtype, sm_scale, workspace, workspace_bytes_,
                      error_flag, stream);
}

extern "C" KVX_API int kvx_append_decode(const kvx_paged *kv, const int32_t *block_table,
                                         int32_t max_pages, const int32_t *positions, int32_t batch,
                                         const void *new_k, const void *new_v, int32_t num_q_heads,
                                         const void *q, void *out, int32_t io_dtype, float sm_scale,
                                         void *workspace, size_t workspace_bytes_,
                                         int32_t *error_flag, void *stream) {
    if (!positions) return KVX_EINVAL;
    return run_decode(kv, block_table, max_pages, nullptr, positions, new_k, new_v, batch,
                      num_q_heads, q, out, io_dtype, sm_scale, workspace, workspace_bytes_,
                      error_flag, stream);
}

extern "C" KVX_API int kvx_append_decode_signal(const kvx_paged *kv, const int32_t *block_table,
                                                int32_t max_pages, const int32_t *positions, int32_t batch,
                                                const void *new_k, const void *new_v, int32_t num_q_heads,
                                                const void *q, void *out, int32_t io_dtype, float sm_scale,
                                                void *workspace, size_t workspace_bytes_,
                                                int32_t *error_flag, uint32_t *done, uint32_t epoch,
                                                void *stream) {
    if (!positions || !done) return KVX_EINVAL;
    return run_decode(kv, block_table, max_pages, nullptr, positions, new_k, new_v, batch,
                      num_q_heads, q, out, io_dtype, sm_scale, workspace, workspace_bytes_,
                      error_flag, stream, 0, nullptr, done, epoch);
}

// ---------------------------------------------------------------------------
// Decode that allocates nothing.
//
// Some callers of this library cannot allocate device memory at the moment
// they decode: a JVM scheduler thread reaching the engine through JNI holds
// only the buffers it was handed, an engine whose KV pool is capped to a
// fixed byte budget must not grow, and code running under another
// framework's allocator (or inside its stream capture) may not call
// cudaMalloc / cudaFree behind that allocator's back.  kvx_decode_noalloc
// serves them: its split-K scratch is a file-scope device array of
// kNoAllocScratchBytes that every GPU loading this library holds until the
// process exits.  The array is shared by all calls on a device and keeps the
// last call's contents; the arrival counters that must start at zero are
// cleared on the caller's stream before every launch, so calls that overlap
// on the GPU (different streams, no ordering) race on the array.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
constexpr int kNoAllocMaxDevices = 64;
void *g_noalloc_addr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device with cudaGetSymbolAddress (with that device current).
int noalloc_scratch(void **addr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KVX_ECUDA;
    if (dev < 0 || dev >= kNoAllocMaxDevices) return KVX_EUNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return KVX_ECUDA;
        g_noalloc_addr[dev] = ptr;
    }
    *addr = g_noalloc_addr[dev];
    return KVX_OK;
}
}  // namespace

extern "C" KVX_API size_t kvx_decode_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" KVX_API int kvx_decode_noalloc(const kvx_paged *kv, const int32_t *block_table,
                                          int32_t max_pages, const int32_t *seq_lens, int32_t batch,
                                          int32_t num_q_heads, const void *q, void *out,
                                          int32_t io_dtype, float sm_scale, int32_t *error_flag,
                                          void *stream) {
    if (!seq_lens || batch <= 0 || num_q_heads <= 0 || max_pages <= 0) return KVX_EINVAL;
    // smallest layout: one split per (sequence, q-head) + its counter
    const size_t rows = (size_t)batch * num_q_heads;
    const size_t per_split = rows * (kHeadDim + 2) * sizeof(float);
    if (rows * sizeof(int32_t) + per_split > kNoAllocScratchBytes) return KVX_ETOOBIG;
    const size_t fit = (kNoAllocScratchBytes - rows * sizeof(int32_t)) / per_split;  // >= 1
    // chunk so that ceil(max_pages / chunk) <= fit, a multiple of the 4 warps
    int min_chunk = (int)((max_pages + fit - 1) / fit);
    min_chunk = (min_chunk + kWarps - 1) / kWarps * kWarps;
    while ((size_t)((max_pages + min_chunk - 1) / min_chunk) > fit) min_chunk += kWarps;
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc != KVX_OK) return rc;
    const size_t splits_cap = (size_t)(max_pages + min_chunk - 1) / min_chunk;
    int32_t *counters = reinterpret_cast<int32_t *>(static_cast<float *>(scratch) + rows * splits_cap * (kHeadDim + 2));
    if (cudaMemsetAsync(counters, 0, rows * sizeof(int32_t), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return KVX_ECUDA;
    return run_decode(kv, block_table, max_pages, seq_lens, nullptr, nullptr, nullptr, batch,
                      num_q_heads, q, out, io_dtype, sm_scale, scratch, kNoAllocScratchBytes,
                      error_flag, stream, min_chunk);
}

namespace kvx {
namespace {

// Per (sequence, logical page): the attention the page received, averaged
// over the q-heads: mean_h sum_{t in page} softmax_h(t) =
// mean_h s_hp * exp2(m_hp - M_h) / L_h.  Zero for pages past the context.
__global__ void attn_mass_kernel(const float *__restrict__ pm, const float *__restrict__ ml,
                                 const int32_t *__restrict__ seq_lens, int batch, int hq, int max_pages,
                                 float *__restrict__ mass) {
    const size_t n = (size_t)batch * max_pages;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int s = (int)(e / max_pages), lp = (int)(e % max_pages);
        const int T = min(max(seq_lens[s], 0), max_pages * kPageTokens);
        float acc = 0.f;
        if (lp * kPageTokens < T) {
            for (int h = 0; h < hq; ++h) {
                const float2 f = *reinterpret_cast<const float2 *>(ml + ((size_t)s * hq + h) * 2);
                const float2 v = *reinterpret_cast<const float2 *>(pm + (((size_t)s * hq + h) * max_pages + lp) * 2);
                acc += v.y * exp2f(v.x - f.x) / f.y;
            }
            acc /= (float)hq;
        }
        mass[e] = acc;
    }
}

struct EvictMetricsRec {  // native-engine/include/AdvancedEvictionPolicy.h:19-27
    unsigned long long last_access_token;
    float total_attention, average_attention, access_frequency;
    uint32_t pad0;
    unsigned long long creation_time, page_size;
    int32_t page_id;
    uint32_t pad1;
};

// updateMetrics of AttentionBasedEvictionPolicy (:88-91: lastAccessToken =
// currentToken) with the attention the decode measured: per physical page
// read this step, averageAttention = the page's mass, totalAttention and
// accessFrequency accumulate.
__global__ void attn_to_metrics_kernel(const float *__restrict__ mass, const int32_t *__restrict__ bt,
                                       const int32_t *__restrict__ seq_lens, int batch, int max_pages,
                                       EvictMetricsRec *metrics, int num_metrics, unsigned long long token) {
    const size_t n = (size_t)batch * max_pages;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int s = (int)(e / max_pages), lp = (int)(e % max_pages);
        const int T = min(max(seq_lens[s], 0), max_pages * kPageTokens);
        if (lp * kPageTokens >= T) continue;
        const int phys = bt[e];
        if (phys < 0 || phys >= num_metrics) continue;
        EvictMetricsRec &m = metrics[phys];
        m.last_access_token = token;
        m.average_attention = mass[e];
        atomicAdd(&m.total_attention, mass[e]);
        atomicAdd(&m.access_frequency, 1.0f);
    }
}

size_t attn_bytes(int batch, int hq, int max_pages) {
    return ((size_t)batch * hq * max_pages * 2 + (size_t)batch * hq * 2) * sizeof(float);
}

}  // namespace
}  // namespace kvx

extern "C" KVX_API size_t kvx_decode_attn_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t max_pages,
                                                          int32_t page_tokens) {
    const size_t base = kvx_decode_workspace_bytes(batch, num_q_heads, max_pages, page_tokens);
    if (!base) return 0;
    return base + (attn_bytes(batch, num_q_heads, max_pages) + 15) / 16 * 16;
}

extern "C" KVX_API int kvx_decode_attn(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                                       const int32_t *seq_lens, int32_t batch, int32_t num_q_heads,
                                       const void *q, void *out, int32_t io_dtype, float sm_scale,
                                       void *workspace, size_t workspace_bytes_, float *page_mass,
                                       int32_t *error_flag, void *stream) {
    if (!seq_lens || !page_mass || !workspace || batch <= 0 || num_q_heads <= 0 || max_pages <= 0)
        return KVX_EINVAL;
    const size_t base = workspace_bytes(batch, num_q_heads, max_pages);
    if (workspace_bytes_ < base + attn_bytes(batch, num_q_heads, max_pages)) return KVX_ENOSPC;
    if (reinterpret_cast<uintptr_t>(page_mass) & 3) return KVX_EINVAL;
    float *attn = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + base);
    int rc = run_decode(kv, block_table, max_pages, seq_lens, nullptr, nullptr, nullptr, batch, num_q_heads, q, out,
                        io_dtype, sm_scale, workspace, base, error_flag, stream, 0, attn);
    if (rc != KVX_OK) return rc;
    const size_t n = (size_t)batch * max_pages;
    attn_mass_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        attn, attn + (size_t)batch * num_q_heads * max_pages * 2, seq_lens, batch, num_q_heads, max_pages, page_mass);
    return launch_status();
}

extern "C" KVX_API int kvx_attn_to_metrics(const float *page_mass, const int32_t *block_table, int32_t max_pages,
                                           const int32_t *seq_lens, int32_t batch, kvx_evict_metrics *metrics,
                                           int32_t num_metrics, uint64_t current_token, void *stream) {
    if (!page_mass || !block_table || !seq_lens || !metrics || batch <= 0 || max_pages <= 0 || num_metrics <= 0)
        return KVX_EINVAL;
    if (reinterpret_cast<uintptr_t>(metrics) & 7) return KVX_EINVAL;
    const size_t n = (size_t)batch * max_pages;
    attn_to_metrics_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 8), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(
        page_mass, block_table, seq_lens, batch, max_pages, reinterpret_cast<EvictMetricsRec *>(metrics), num_metrics,
        (unsigned long long)current_token);
    return launch_status();
}
