// kvx_append.cu -- paged append: scatter each sequence's new K/V rows into
// slot pos % page_tokens of physical page block_table[s][pos / page_tokens].
// Replaces KVManager::save_page (cache/kv_cache.cpp:111-127) on the append
// path of InferenceController::appendKVPage (runtime/inference.cpp:50-54).
//
// One thread per 16-byte vector of a (sequence, K|V, head) row: consecutive
// threads write consecutive bytes of a row (coalesced), rows land wherever
// the block table points.  Pure copy, bit-exact.
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

// Chunked append: each sequence appends n_new consecutive tokens.  A warp
// owns one run (sequence, page slice, K|V, head): the chunk's tokens that
// fall into one physical page, at most 16 rows that are contiguous in the
// page (one 4 KiB block at fp16) and head-strided in the source.  Lanes
// cover a row in 16-byte vectors (two rows per instruction at fp16); all of
// a run's loads are issued before its stores, so a warp keeps up to 8 rows
// in flight.  All index arithmetic is per warp, not per vector.
template <int kRowVecs>
__global__ void __launch_bounds__(256)
append_chunk_kernel(uint8_t *pool, const uint8_t *new_k, const uint8_t *new_v,
                    const int32_t *block_table, const int32_t *positions, int32_t *error_flag,
                    int batch, int n_new, int hkv, int max_pages, int num_pages, int slices) {
    constexpr int kRowBytes = kRowVecs * 16;
    constexpr int kRowsPerOp = 32 / kRowVecs;          // rows one warp instruction covers
    constexpr int kOps = (kPageTokens + kRowsPerOp - 1) / kRowsPerOp;
    // Dependent launch: the next launch on the stream may be scheduled now,
    // and this grid touches memory only once the previous one has finished
    // (it may have written the rows or the pool), so back-to-back appends
    // keep their order and lose only the launch gap.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const long long run = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const long long runs = (long long)batch * slices * 2 * hkv;
    if (run >= runs) return;
    const int h = (int)(run % hkv);
    const int kv = (int)((run / hkv) % 2);
    const int j = (int)((run / (2 * hkv)) % slices);
    const int s = (int)(run / (2LL * hkv * slices));
    const int start = positions[s];
    if (start < 0) {
        if (error_flag && lane == 0 && j == 0 && kv == 0 && h == 0) atomicOr(error_flag, 2);
        return;
    }
    const int lp = start / kPageTokens + j;
    const int t0 = max(start, lp * kPageTokens), t1 = min(start + n_new, (lp + 1) * kPageTokens);
    if (t0 >= t1) return;  // the chunk ends before this slice
    const int phys = lp < max_pages ? block_table[(size_t)s * max_pages + lp] : -1;
    if (phys < 0 || phys >= num_pages) {
        if (error_flag && lane == 0 && kv == 0 && h == 0) atomicOr(error_flag, 2);
        return;
    }
    const int r_lane = lane / kRowVecs, v = lane % kRowVecs;
    const uint8_t *src = (kv ? new_v : new_k) +
                         (((size_t)s * n_new + (t0 - start)) * hkv + h) * kRowBytes + v * 16;
    uint8_t *dst = pool + ((((size_t)phys * 2 + kv) * hkv + h) * kPageTokens + (t0 - lp * kPageTokens)) * kRowBytes +
                   v * 16;
    const int rows = t1 - t0;
    uint4 val[kOps];
#pragma unroll
    for (int o = 0; o < kOps; ++o) {
        const int r = o * kRowsPerOp + r_lane;
        if (r < rows) val[o] = __ldcs(reinterpret_cast<const uint4 *>(src + (size_t)r * hkv * kRowBytes));
    }
#pragma unroll
    for (int o = 0; o < kOps; ++o) {
        const int r = o * kRowsPerOp + r_lane;
        if (r < rows) *reinterpret_cast<uint4 *>(dst + (size_t)r * kRowBytes) = val[o];
    }
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
    // page slices a chunk can touch: it may start anywhere inside a page
    const int slices = (n_new + kPageTokens - 1) / kPageTokens + 1;
    const long long runs = (long long)batch * slices * 2 * kv->num_kv_heads;
    const long long blocks = (runs + 7) / 8;
    if (blocks > 0x7fffffffLL) return KVX_EINVAL;
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
            ? cudaLaunchKernelEx(&cfg, append_chunk_kernel<16>, pool, k, v, block_table, positions, error_flag, batch,
                                 n_new, kv->num_kv_heads, max_pages, kv->num_pages, slices)
            : cudaLaunchKernelEx(&cfg, append_chunk_kernel<32>, pool, k, v, block_table, positions, error_flag, batch,
                                 n_new, kv->num_kv_heads, max_pages, kv->num_pages, slices);
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
