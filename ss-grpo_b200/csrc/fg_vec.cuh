// fg_vec.cuh -- 16-byte vector loads of logits rows (8 x bf16/f16, 4 x f32).
#pragma once

#include "fg_common.cuh"

namespace fg {

template <typename T>
struct Vec {
    static constexpr int N = 16 / sizeof(T);
};

// Converts one 16-byte vector to floats.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float* out);

template <>
__device__ __forceinline__ void unpack<float>(const uint4& u, float* out) {
    out[0] = __uint_as_float(u.x);
    out[1] = __uint_as_float(u.y);
    out[2] = __uint_as_float(u.z);
    out[3] = __uint_as_float(u.w);
}

template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& u, float* out) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

template <>
__device__ __forceinline__ void unpack<__half>(const uint4& u, float* out) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        const float2 f = __half22float2(h);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// Row can be read with 16-byte vectors: aligned base and whole vectors.
template <typename T>
__device__ __forceinline__ bool row_vectorizable(const T* row, int32_t V) {
    return ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) && (V % Vec<T>::N == 0);
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

}  // namespace fg
