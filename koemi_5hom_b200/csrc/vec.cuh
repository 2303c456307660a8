// 16-byte vector load/store helpers: a row is read as uint4 packets and
// unpacked to fp32 lanes (8 x 16-bit or 4 x fp32 per packet).
#pragma once

#include "common.cuh"

namespace koemi {

template <typename T>
struct Pack {
    static constexpr int kWidth = 16 / sizeof(T);
};

__device__ __forceinline__ void unpack(const uint4 &raw, float (&out)[8], __nv_bfloat16) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void unpack(const uint4 &raw, float (&out)[8], __half) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void unpack(const uint4 &raw, float (&out)[4], float) {
    out[0] = __uint_as_float(raw.x);
    out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z);
    out[3] = __uint_as_float(raw.w);
}

__device__ __forceinline__ uint4 pack(const float (&in)[8], __nv_bfloat16) {
    uint4 raw;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    return raw;
}
__device__ __forceinline__ uint4 pack(const float (&in)[8], __half) {
    uint4 raw;
    __half2 *h = reinterpret_cast<__half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
    return raw;
}
__device__ __forceinline__ uint4 pack(const float (&in)[4], float) {
    return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]),
                      __float_as_uint(in[3]));
}

__device__ __forceinline__ uint4 load_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 load_cached(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// A plain 16-byte store (global stores do not allocate in L1). Written as C++
// rather than inline asm so the compiler may schedule later loads ahead of
// it: a volatile asm store with a memory clobber serialised every
// load-after-store of a loop into one L2 round trip per iteration.
__device__ __forceinline__ void store_stream(void *p, const uint4 &v) { *reinterpret_cast<uint4 *>(p) = v; }

}  // namespace koemi
