/* kvx_cxx.h -- export macro for the C++ drop-in classes of the engine
 * library (kv_cache.h, kv_pager.h, kv_compress.h, scheduler.h,
 * runtime_contract.h, cuda_executor.h). */
#ifndef KVX_CXX_H
#define KVX_CXX_H
#if defined(_WIN32)
#define KVX_CXX_API __declspec(dllexport)
#else
#define KVX_CXX_API __attribute__((visibility("default")))
#endif
#endif
