// Scalar element access shared by the general-shape kernels: dtype conversions and the
// extraction of one code from the MLX packed layout (code k of a row at bit k*bits of the
// row's little-endian bitstream; a 3-bit code may straddle two words).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace q38 {
namespace dev {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
    return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
    return v;
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
    return __float2half_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
    return v;
}

__device__ __forceinline__ uint32_t get_code(const uint32_t* row, int64_t k, int bits) {
    const int64_t bit = k * bits;
    const int64_t w = bit >> 5;
    const int off = static_cast<int>(bit & 31);
    uint32_t v = row[w] >> off;
    if (off + bits > 32) v |= row[w + 1] << (32 - off);
    return v & ((1u << bits) - 1u);
}

}  // namespace dev
}  // namespace q38
