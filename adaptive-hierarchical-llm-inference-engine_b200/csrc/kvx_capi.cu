// kvx_capi.cu -- library-level entry points of the C ABI (version, status
// strings, device check).
#include <cuda_runtime.h>

#include "kvx.h"

extern "C" KVX_API const char *kvx_version(void) { return "kvx 0.1 sm_100a"; }

extern "C" KVX_API const char *kvx_status_string(int status) {
    switch (status) {
    case KVX_OK: return "ok";
    case KVX_EINVAL: return "invalid argument";
    case KVX_EBUSY: return "object pinned";
    case KVX_ECUDA: return "CUDA error";
    case KVX_EUNSUPPORTED: return "unsupported geometry or dtype";
    case KVX_ETIMEOUT: return "bounded device wait expired";
    case KVX_ENOSPC: return "workspace or pool too small";
    case KVX_ENODEV: return "no sm_100 device";
    case KVX_ETOOBIG: return "request exceeds the static scratch of kvx_decode_noalloc";
    default: return "unknown status";
    }
}

extern "C" KVX_API int kvx_device_check(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KVX_ENODEV;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return KVX_ENODEV;
    return major == 10 ? KVX_OK : KVX_ENODEV;
}
