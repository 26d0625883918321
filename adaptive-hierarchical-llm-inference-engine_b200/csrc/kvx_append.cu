// kvx_append.cu -- paged append: scatter each sequence's new K/V rows into
// slot pos % page_tokens of physical page block_table[s][pos / page_tokens].
// Replaces KVManager::save_page (cache/kv_cache.cpp:111-127) on the append
// path of InferenceController::appendKVPage (runtime/inference.cpp:50-54).
//
// One thread per 16-byte vector of a (sequence, K|V, head) row: consecutive
// threads write consecutive bytes of a row (coalesced), rows land wherever
// the block table points.  Pure copy, bit-exact.
#include <algorithm>

#include "kvx_common.cuh"

namespace kvx {
namespace {

__global__ void __launch_bounds__(256)
append_kernel(uint8_t *pool, const uint8_t *new_k, const uint8_t *new_v,
              const int32_t *block_table, const int32_t *positions, int32_t *error_flag,
              int batch, int hkv, int max_pages, int num_pages, int page_tokens,
              int row_vecs /* 16-byte vectors per row */) {
    const long long total = (long long)batch * 2 * hkv * row_vecs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int v = (int)(i % row_vecs);
        long long r = i / row_vecs;            // row = ((s * 2) + kv) * hkv + h
        const int h = (int)(r % hkv);
        r /= hkv;
        const int kv = (int)(r % 2);
        const int s = (int)(r / 2);
        const int pos = positions[s];
        const int lp = pos / page_tokens;
        if (pos < 0 || lp >= max_pages) {
            if (error_flag && v == 0) atomicOr(error_flag, 2);
            continue;
        }
        const int phys = block_table[(size_t)s * max_pages + lp];
        if (phys < 0 || phys >= num_pages) {
            if (error_flag && v == 0) atomicOr(error_flag, 2);
            continue;
        }
        const int slot = pos % page_tokens;
        const size_t row_bytes = (size_t)row_vecs * 16;
        const size_t dst = ((((size_t)phys * 2 + kv) * hkv + h) * page_tokens + slot) * row_bytes;
        const size_t src = ((size_t)s * hkv + h) * row_bytes;
        const uint4 val = *reinterpret_cast<const uint4 *>((kv ? new_v : new_k) + src + v * 16);
        *reinterpret_cast<uint4 *>(pool + dst + v * 16) = val;
    }
}

// Chunked append: each sequence appends n_new consecutive tokens.  The
// launch's rows are numbered r = ((s * 2 + kv) * n_new + t) * hkv + h, so
// consecutive rows are consecutive in the source (new_k / new_v are
// [s][t][h][row]); the warps of the launch take equal contiguous ranges of
// them (balanced to one warp instruction, whatever the chunks' page
// alignment), and a warp instruction moves kRowsPerOp whole rows in 16-byte
// vectors (two rows at fp16).  A lane walks its rows incrementally (no
// division per row); the source address needs no table lookup, so a
// batch's source loads (up to 8 per lane) are all in flight before its
// stores, which go to slot pos % 16 of page block_table[s][pos / 16].
template <int kRowVecs>
__global__ void __launch_bounds__(256, 4)
append_chunk_kernel(uint8_t *pool, const uint8_t *new_k, const uint8_t *new_v,
                    const int32_t *block_table, const int32_t *positions, int32_t *error_flag,
                    int n_new, int hkv, int max_pages, int num_pages, uint32_t rows_total, uint32_t units_per_warp) {
    constexpr int kRowBytes = kRowVecs * 16;
    constexpr int kRowsPerOp = 32 / kRowVecs;  // rows one warp instruction covers
    constexpr int kBatch = 8;                  // loads in flight per lane
    // Dependent launch: the next launch on the stream may be scheduled now,
    // and this grid touches memory only once the previous one has finished
    // (it may have written the rows or the pool), so back-to-back appends
    // keep their order and lose only the launch gap.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31, r_lane = lane / kRowVecs, v = lane % kRowVecs;
    const uint32_t warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint64_t u0 = (uint64_t)warp * units_per_warp;
    const uint64_t units = ((uint64_t)rows_total + kRowsPerOp - 1) / kRowsPerOp;
    if (u0 >= units) return;
    const uint32_t n_units = (uint32_t)(units - u0 < units_per_warp ? units - u0 : units_per_warp);
    // this lane's first row, decomposed once
    uint32_t r = (uint32_t)(u0 * kRowsPerOp) + r_lane;
    uint32_t h = r % hkv, q = r / hkv;
    uint32_t t = q % n_new, q2 = q / n_new;
    uint32_t kv = q2 & 1, sq = q2 >> 1;
    for (uint32_t b0 = 0; b0 < n_units; b0 += kBatch) {
        uint4 val[kBatch];
        uint8_t *dst[kBatch];
#pragma unroll
        for (int o = 0; o < kBatch; ++o) {
            dst[o] = nullptr;
            if (b0 + o < n_units && r < rows_total) {
                const uint8_t *src = (kv ? new_v : new_k) + (((size_t)sq * n_new + t) * hkv + h) * kRowBytes + v * 16;
                val[o] = __ldcs(reinterpret_cast<const uint4 *>(src));
                const int start = positions[sq];
                const long long pos = (long long)start + t;
                const long long lp = pos >> 4;
                const int phys = start >= 0 && lp < max_pages ? block_table[(size_t)sq * max_pages + lp] : -1;
                if (phys >= 0 && phys < num_pages)
                    dst[o] = pool + ((((size_t)phys * 2 + kv) * hkv + h) * kPageTokens + (pos & 15)) * kRowBytes + v * 16;
                else if (error_flag && v == 0)
                    atomicOr(error_flag, 2);
            }
            // next row of this lane: kRowsPerOp further
            r += kRowsPerOp;
            h += kRowsPerOp;
            while (h >= (uint32_t)hkv) {
                h -= hkv;
                if (++t == (uint32_t)n_new) {
                    t = 0;
                    if (++kv == 2) kv = 0, ++sq;
                }
            }
        }
#pragma unroll
        for (int o = 0; o < kBatch; ++o)
            if (dst[o]) *reinterpret_cast<uint4 *>(dst[o]) = val[o];
    }
}

// Resident append_chunk_kernel blocks per SM of the current device, looked
// up once per device.
int append_resident_blocks(bool f16) {
    static std::atomic<int> cache[2][kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    const bool cached = dev >= 0 && dev < kMaxDevices;
    int n = cached ? cache[f16][dev].load(std::memory_order_relaxed) : 0;
    if (n <= 0) {
        const cudaError_t e =
            f16 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, append_chunk_kernel<16>, 256, 0)
                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, append_chunk_kernel<32>, 256, 0);
        if (e != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 4;
        }
        if (cached) cache[f16][dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_append_chunk(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                                        const int32_t *positions, int32_t batch, int32_t n_new,
                                        const void *new_k, const void *new_v, int32_t *error_flag,
                                        void *stream) {
    if (!kv || !kv->pool || !block_table || !positions || !new_k || !new_v) return KVX_EINVAL;
    if (batch < 0 || n_new < 0 || max_pages <= 0 || kv->num_kv_heads <= 0 || kv->num_pages <= 0)
        return KVX_EINVAL;
    if (kv->dtype != KVX_F32 && kv->dtype != KVX_F16) return KVX_EUNSUPPORTED;
    if (kv->page_tokens != kPageTokens || kv->head_dim != kHeadDim) return KVX_EUNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(kv->pool) | reinterpret_cast<uintptr_t>(new_k) |
         reinterpret_cast<uintptr_t>(new_v)) & 15)
        return KVX_EINVAL;
    if (batch == 0 || n_new == 0) return KVX_OK;
    const uint64_t rows_total = (uint64_t)batch * 2 * n_new * kv->num_kv_heads;
    if (rows_total > 0x7fffffffULL) return KVX_EUNSUPPORTED;
    // warps: enough to fill every SM (resident blocks x SMs), at least one
    // warp instruction of rows each; then an equal share of the rows each
    const int rows_per_op = kv->dtype == KVX_F16 ? 2 : 1;
    const uint64_t units = (rows_total + rows_per_op - 1) / rows_per_op;
    const uint64_t warp_cap = (uint64_t)append_resident_blocks(kv->dtype == KVX_F16) * sm_count() * 8;
    const uint64_t warps = std::min<uint64_t>(units, warp_cap);
    const uint32_t per = (uint32_t)((units + warps - 1) / warps);
    const uint64_t blocks = ((units + per - 1) / per + 7) / 8;
    auto *pool = static_cast<uint8_t *>(kv->pool);
    auto *k = static_cast<const uint8_t *>(new_k), *v = static_cast<const uint8_t *>(new_v);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e =
        kv->dtype == KVX_F16
            ? cudaLaunchKernelEx(&cfg, append_chunk_kernel<16>, pool, k, v, block_table, positions, error_flag, n_new,
                                 kv->num_kv_heads, max_pages, kv->num_pages, (uint32_t)rows_total, per)
            : cudaLaunchKernelEx(&cfg, append_chunk_kernel<32>, pool, k, v, block_table, positions, error_flag, n_new,
                                 kv->num_kv_heads, max_pages, kv->num_pages, (uint32_t)rows_total, per);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KVX_ECUDA;
    }
    return launch_status();
}

extern "C" KVX_API int kvx_append(const kvx_paged *kv, const int32_t *block_table,
                                  int32_t max_pages, const int32_t *positions, int32_t batch,
                                  const void *new_k, const void *new_v, int32_t *error_flag,
                                  void *stream) {
    if (!kv || !kv->pool || !block_table || !positions || !new_k || !new_v) return KVX_EINVAL;
    if (batch < 0 || max_pages <= 0 || kv->num_kv_heads <= 0 || kv->page_tokens <= 0 ||
        kv->head_dim <= 0 || kv->num_pages <= 0)
        return KVX_EINVAL;
    if (kv->dtype != KVX_F32 && kv->dtype != KVX_F16) return KVX_EUNSUPPORTED;
    const int esize = kv->dtype == KVX_F32 ? 4 : 2;
    const size_t row_bytes = (size_t)kv->head_dim * esize;
    if (row_bytes % 16) return KVX_EUNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(kv->pool) | reinterpret_cast<uintptr_t>(new_k) |
         reinterpret_cast<uintptr_t>(new_v)) & 15)
        return KVX_EINVAL;
    if (batch == 0) return KVX_OK;
    const int row_vecs = (int)(row_bytes / 16);
    const long long total = (long long)batch * 2 * kv->num_kv_heads * row_vecs;
    const int threads = 256;
    long long blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    append_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t *>(kv->pool), static_cast<const uint8_t *>(new_k),
        static_cast<const uint8_t *>(new_v), block_table, positions, error_flag, batch,
        kv->num_kv_heads, max_pages, kv->num_pages, kv->page_tokens, row_vecs);
    return launch_status();
}
