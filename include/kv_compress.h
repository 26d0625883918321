/* kv_compress.h -- drop-in for the reference's compression/kv_compress.h
 * (same two functions, same bit-exact results): truncating fp32 -> fp16
 * (exponent > 15 -> +-Inf, NaN -> Inf, exponent <= -15 -> +-0) and its
 * inverse (fp16 subnormals -> +-0), as the reference's disk tier uses them
 * (compression/kv_compress.cpp:6-60).  Both run on the GPU
 * (kvx_f32_to_f16_trunc / kvx_f16_trunc_to_f32) on the current device and
 * throw std::runtime_error when no sm_100 device is usable. */
#pragma once

#include <cstdint>
#include <vector>

#include "kvx_cxx.h"

KVX_CXX_API std::vector<uint16_t> float32_to_float16(const std::vector<float> &in);
KVX_CXX_API std::vector<float> float16_to_float32(const std::vector<uint16_t> &in);
