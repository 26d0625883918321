/* Host-memory stand-in for the four CUDA runtime calls the reference's
 * native-engine/cpp/KVCacheGPU.cpp makes (cudaMalloc, cudaFree, cudaMemcpy,
 * cudaGetErrorString), so that its page policy runs on a CPU to produce the
 * golden traces (tests/golden/make_golden.py).  Test infrastructure only:
 * used by the oracle/_ref driver build, never by the library.
 * A 0-byte cudaMalloc succeeds with a null pointer, as the CUDA runtime's. */
#ifndef KVO_HOST_CUDA_RUNTIME_H
#define KVO_HOST_CUDA_RUNTIME_H
#include <stdlib.h>
#include <string.h>

typedef enum cudaError { cudaSuccess = 0, cudaErrorMemoryAllocation = 2 } cudaError_t;
enum cudaMemcpyKind {
    cudaMemcpyHostToHost = 0,
    cudaMemcpyHostToDevice = 1,
    cudaMemcpyDeviceToHost = 2,
    cudaMemcpyDeviceToDevice = 3,
    cudaMemcpyDefault = 4
};

static inline cudaError_t cudaMalloc(void **p, size_t n) {
    if (n == 0) {
        *p = NULL;
        return cudaSuccess;
    }
    *p = malloc(n);
    return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
static inline cudaError_t cudaFree(void *p) {
    free(p);
    return cudaSuccess;
}
static inline cudaError_t cudaMemcpy(void *dst, const void *src, size_t n, enum cudaMemcpyKind k) {
    (void)k;
    if (n) memcpy(dst, src, n);
    return cudaSuccess;
}
static inline const char *cudaGetErrorString(cudaError_t e) { return e == cudaSuccess ? "no error" : "out of memory"; }
#endif
