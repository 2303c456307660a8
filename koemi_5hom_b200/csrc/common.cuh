// Shared helpers for the libkoemi_b200 translation units: error reporting,
// dtype conversion, bounded mbarrier waits and TMA tensor-map plumbing.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <utility>

#include "../../include/koemi_b200.h"

namespace koemi {

// ------------------------------------------------------------------ host side

// Records a printf-style message as the calling thread's last error and
// returns `code`, so call sites read `return fail(KOEMI_ERR_INVALID, ...)`.
int fail(int code, const char *format, ...);
void clear_error();

// Per-device status word (int), allocated once per device on first use. A
// bounded device-side wait that gives up stores KOEMI_ERR_TIMEOUT into it.
int *device_status_word();

// Number of SMs of the current device (cached per device).
int sm_count();

// Encodes a tiled TMA descriptor through the driver entry point (no -lcuda).
int encode_tensor_map(CUtensorMap *map, CUtensorMapDataType type, uint32_t rank, const void *base,
                      const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                      CUtensorMapSwizzle swizzle);

inline size_t dtype_size(int dtype) {
    switch (dtype) {
        case KOEMI_F32: return 4;
        case KOEMI_F16: return 2;
        case KOEMI_BF16: return 2;
        case KOEMI_F64: return 8;
        case KOEMI_I32: return 4;
        case KOEMI_I64: return 8;
        case KOEMI_BOOL: return 1;
        default: return 0;
    }
}

inline bool aligned(const void *pointer, size_t bytes) {
    return (reinterpret_cast<uintptr_t>(pointer) % bytes) == 0;
}

inline cudaStream_t as_stream(void *stream) { return reinterpret_cast<cudaStream_t>(stream); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Launch helper for the decode-path kernels. With kProgrammaticLaunch the
// kernel may start while the previous kernel of the stream is finishing (its
// CTAs take SMs as they free up and run their prologue); every kernel
// launched through here therefore calls pdl_wait() before it touches global
// memory written or read by earlier work. Measured on the config-5 decode
// step it gained nothing (consecutive kernels are already ~0.35 us apart) and
// cost ~5% at 32 streams, so it is off; the waits are then no-ops. `cluster`
// with more than one CTA also sets thread-block cluster dims.
constexpr bool kProgrammaticLaunch = false;
// The same with the programmatic attribute chosen per launch: the weight-
// streaming GEMMs whose weights no earlier kernel writes set it, start loading
// those weights while the previous kernel finishes, and wait (pdl_wait) before
// they read anything that kernel wrote.
template <typename... KernelArgs, typename... Args>
inline cudaError_t launch_programmatic(bool programmatic, void (*kernel)(KernelArgs...), dim3 grid, dim3 block,
                                       size_t smem, cudaStream_t stream, dim3 cluster, Args &&...args) {
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attributes[2];
    attributes[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[0].val.programmaticStreamSerializationAllowed = programmatic ? 1 : 0;
    unsigned count = 1;
    if (cluster.x * cluster.y * cluster.z > 1) {
        attributes[1].id = cudaLaunchAttributeClusterDimension;
        attributes[1].val.clusterDim.x = cluster.x;
        attributes[1].val.clusterDim.y = cluster.y;
        attributes[1].val.clusterDim.z = cluster.z;
        count = 2;
    }
    config.attrs = attributes;
    config.numAttrs = count;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

template <typename... KernelArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, dim3 cluster, Args &&...args) {
    return launch_programmatic(kProgrammaticLaunch, kernel, grid, block, smem, stream, cluster,
                               std::forward<Args>(args)...);
}

#define KOEMI_CUDA_TRY(expr)                                                                      \
    do {                                                                                          \
        cudaError_t koemi_error_ = (expr);                                                        \
        if (koemi_error_ != cudaSuccess) {                                                        \
            return ::koemi::fail(KOEMI_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                  \
                                 cudaGetErrorString(koemi_error_), __FILE__, __LINE__);           \
        }                                                                                         \
    } while (0)

#define KOEMI_LAUNCH_CHECK() KOEMI_CUDA_TRY(cudaGetLastError())

// ---------------------------------------------------------------- device side

// Programmatic dependent launch: pdl_trigger lets the next kernel of the
// stream be scheduled; pdl_wait blocks until the previous kernel has finished
// and its memory is visible (a no-op for kernels launched without the
// attribute).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename T>
struct Accum {
    using type = float;
};
template <>
struct Accum<double> {
    using type = double;
};

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ double to_acc(double v) { return v; }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_acc(float v);
template <>
__device__ __forceinline__ float from_acc<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <typename T>
__device__ __forceinline__ T from_acc(double v) {
    return static_cast<T>(v);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }
// SiLU through the fast exponential and divide intrinsics (relative error
// ~1e-6); for streaming kernels whose issue rate would otherwise bound them.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
    return v;
}

// Spin budget of every bounded wait: about a second or more at B200 clocks
// before the waiting thread records KOEMI_ERR_TIMEOUT and gives up.
constexpr uint32_t kWaitSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

// Waits for `phase` of `bar` with a bounded spin. Returns false (after
// recording KOEMI_ERR_TIMEOUT in *status) when the budget runs out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, int *status) {
    for (uint32_t spin = 0; spin < kWaitSpinLimit; ++spin) {
        if (mbar_try_wait(bar, phase)) return true;
    }
    if (status != nullptr) atomicExch(status, KOEMI_ERR_TIMEOUT);
    return false;
}

// 2D/3D tiled TMA load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ bool elect_one_lane() { return (threadIdx.x & 31) == 0; }

}  // namespace koemi
