// Operand builders of the prefill window path (model/network.py:305-386 and
// model/memory.py:297-361, 405-455 in the reference): the fp32 rows that a
// window produces are converted once into the compute dtype in the layout the
// next tensor-core product reads.
//
//   koemi_window_pack_rows      up to 8 fp32 row blocks side by side in one
//                               output row (the fusion input [h | memory |
//                               local | salient], the shifted prior)
//   koemi_window_slot_operands  the slots [carried ring ; window] of a ring
//                               read as stacked keys [B, S, d] and transposed
//                               values [B, d, S] (S padded with zero slots)
//
// Both are HBM-bound copies: every fp32 element is read once and its 16-bit
// image written once, loads and stores 16 or 8 bytes wide and coalesced (the
// transpose goes through a shared-memory tile).
#include "common.cuh"

namespace koemi {
namespace {

constexpr int kPackThreads = 256;
constexpr int kPackUnits = 4;  // float4 units per thread
constexpr int kMaxParts = 8;

struct PackArgs {
    const float *source[kMaxParts];
    int64_t stride[kMaxParts];
    int64_t offset[kMaxParts + 1];  // first output column of each part; offset[parts] = total width
    int parts;
    int64_t rows;
    int64_t out_stride;
};

template <typename T>
__device__ __forceinline__ void store4(T *dst, float4 v);

template <>
__device__ __forceinline__ void store4<float>(float *dst, float4 v) {
    *reinterpret_cast<float4 *>(dst) = v;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *dst, float4 v) {
    uint2 raw;
    *reinterpret_cast<__nv_bfloat162 *>(&raw.x) = __floats2bfloat162_rn(v.x, v.y);
    *reinterpret_cast<__nv_bfloat162 *>(&raw.y) = __floats2bfloat162_rn(v.z, v.w);
    *reinterpret_cast<uint2 *>(dst) = raw;
}
template <>
__device__ __forceinline__ void store4<__half>(__half *dst, float4 v) {
    uint2 raw;
    *reinterpret_cast<__half2 *>(&raw.x) = __floats2half2_rn(v.x, v.y);
    *reinterpret_cast<__half2 *>(&raw.y) = __floats2half2_rn(v.z, v.w);
    *reinterpret_cast<uint2 *>(dst) = raw;
}

// grid (column chunks of kPackThreads * kPackUnits float4 units, row blocks);
// each thread issues its kPackUnits loads before its stores.
template <typename T>
__global__ __launch_bounds__(kPackThreads) void pack_rows_kernel(const __grid_constant__ PackArgs a, T *__restrict__ out) {
    const int64_t units = a.offset[a.parts] / 4;
    for (int64_t r = blockIdx.y; r < a.rows; r += gridDim.y) {
        float4 v[kPackUnits];
        int64_t col[kPackUnits];
#pragma unroll
        for (int j = 0; j < kPackUnits; ++j) {
            const int64_t u = static_cast<int64_t>(blockIdx.x) * (kPackThreads * kPackUnits) + j * kPackThreads + threadIdx.x;
            col[j] = u < units ? u * 4 : -1;
            if (col[j] >= 0) {
                int p = 0;
                while (p + 1 < a.parts && col[j] >= a.offset[p + 1]) ++p;
                const float *src = a.source[p] + r * a.stride[p] + (col[j] - a.offset[p]);
                if (a.stride[p] % 4 == 0) {
                    v[j] = __ldg(reinterpret_cast<const float4 *>(src));
                } else {  // rows of an even stride: two 8-byte loads
                    const float2 lo = __ldg(reinterpret_cast<const float2 *>(src));
                    const float2 hi = __ldg(reinterpret_cast<const float2 *>(src + 2));
                    v[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kPackUnits; ++j) {
            if (col[j] >= 0) store4(out + r * a.out_stride + col[j], v[j]);
        }
    }
}

constexpr int kSlotTile = 64;  // slots x features per CTA

// grid (slot tiles, feature tiles, streams), 256 threads. Slot s of stream b
// is carried row s (s < carried), window row s - carried (s < carried +
// length), else a zero slot; keys go out row-major, values through a shared
// tile as columns of the transposed [width, padded] block.
template <typename T>
__global__ __launch_bounds__(256) void slot_operands_kernel(const float *__restrict__ carried_keys,
                                                            const float *__restrict__ carried_values,
                                                            int64_t carried_stride, int64_t carried,
                                                            const float *__restrict__ keys,
                                                            const float *__restrict__ values, int64_t window_stride,
                                                            int64_t length, int64_t width, int64_t padded,
                                                            T *__restrict__ keys_out, T *__restrict__ values_t_out) {
    __shared__ float tile[kSlotTile][kSlotTile + 1];
    const int64_t b = blockIdx.z;
    const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kSlotTile;
    const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kSlotTile;
    const int c4 = threadIdx.x & 15;
    const int64_t col = c0 + 4 * c4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = static_cast<int>(threadIdx.x >> 4) + 16 * i;
        const int64_t slot = s0 + r;
        float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
        if (col < width && slot < padded) {
            if (slot < carried) {
                const int64_t at = b * carried_stride + slot * width + col;
                k = __ldg(reinterpret_cast<const float4 *>(carried_keys + at));
                v = __ldg(reinterpret_cast<const float4 *>(carried_values + at));
            } else if (slot < carried + length) {
                const int64_t at = b * window_stride + (slot - carried) * width + col;
                k = __ldg(reinterpret_cast<const float4 *>(keys + at));
                v = __ldg(reinterpret_cast<const float4 *>(values + at));
            }
            store4(keys_out + (b * padded + slot) * width + col, k);
        }
        tile[r][4 * c4 + 0] = v.x;
        tile[r][4 * c4 + 1] = v.y;
        tile[r][4 * c4 + 2] = v.z;
        tile[r][4 * c4 + 3] = v.w;
    }
    __syncthreads();
    // 64 feature columns x 32 slot pairs; a warp stores 32 consecutive pairs
#pragma unroll
    for (int it = 0; it < (kSlotTile * kSlotTile / 2) / 256; ++it) {
        const int idx = it * 256 + static_cast<int>(threadIdx.x);
        const int cl = idx >> 5;
        const int jp = idx & 31;
        const int64_t slot = s0 + 2 * jp;
        const int64_t c = c0 + cl;
        if (c < width && slot < padded) {
            T *dst = values_t_out + (b * width + c) * padded + slot;
            const float lo = tile[2 * jp][cl], hi = tile[2 * jp + 1][cl];
            if constexpr (sizeof(T) == 2) {
                T pair[2] = {from_acc<T>(lo), from_acc<T>(hi)};
                *reinterpret_cast<uint32_t *>(dst) = *reinterpret_cast<const uint32_t *>(pair);
            } else {
                *reinterpret_cast<float2 *>(dst) = make_float2(lo, hi);
            }
        }
    }
}

template <typename F>
int by_dtype(int dtype, F &&run) {
    switch (dtype) {
        case KOEMI_F32: return run(float());
        case KOEMI_BF16: return run(__nv_bfloat16());
        case KOEMI_F16: return run(__half());
        default: return fail(KOEMI_ERR_UNSUPPORTED, "window operands are written as fp32, bf16 or fp16 (dtype %d)", dtype);
    }
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_window_pack_rows(const float *const *sources, const int64_t *strides, const int64_t *widths,
                                      int parts, int64_t rows, void *out, int64_t out_stride, int dtype,
                                      void *stream) {
    clear_error();
    if (parts < 1 || parts > kMaxParts) return fail(KOEMI_ERR_INVALID, "pack_rows takes 1 to %d parts (got %d)", kMaxParts, parts);
    if (rows < 0) return fail(KOEMI_ERR_INVALID, "negative row count");
    PackArgs args{};
    int64_t total = 0;
    for (int p = 0; p < parts; ++p) {
        const bool wide = strides[p] % 4 == 0;
        if (widths[p] < 0 || widths[p] % 4 != 0 || strides[p] % 2 != 0 ||
            (widths[p] > 0 && !aligned(sources[p], wide ? 16 : 8))) {
            return fail(KOEMI_ERR_INVALID,
                        "pack_rows part %d: widths must be multiples of 4, row strides even and the rows aligned "
                        "(16 bytes, 8 for strides that are not multiples of 4)", p);
        }
        args.source[p] = sources[p];
        args.stride[p] = strides[p];
        args.offset[p] = total;
        total += widths[p];
    }
    args.offset[parts] = total;
    args.parts = parts;
    args.rows = rows;
    args.out_stride = out_stride;
    if (out_stride < total || out_stride % 4 != 0) return fail(KOEMI_ERR_INVALID, "pack_rows output stride too small or not a multiple of 4");
    if (rows == 0 || total == 0) return KOEMI_OK;
    if (!aligned(out, 16)) return fail(KOEMI_ERR_INVALID, "pack_rows output must be 16-byte aligned");
    const int64_t chunks = ceil_div(total / 4, kPackThreads * kPackUnits);
    if (chunks > 2147483647) return fail(KOEMI_ERR_INVALID, "pack_rows rows too wide");
    const unsigned row_blocks = static_cast<unsigned>(rows < 65535 ? rows : 65535);
    return by_dtype(dtype, [&](auto tag) -> int {
        using T = decltype(tag);
        pack_rows_kernel<T><<<dim3(static_cast<unsigned>(chunks), row_blocks), kPackThreads, 0, as_stream(stream)>>>(
            args, static_cast<T *>(out));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    });
}

extern "C" int koemi_window_slot_operands(const float *carried_keys, const float *carried_values,
                                          int64_t carried_stride, int64_t carried, const float *keys,
                                          const float *values, int64_t window_stride, int64_t length, int64_t batch,
                                          int64_t width, int64_t padded, void *keys_out, void *values_t_out, int dtype,
                                          void *stream) {
    clear_error();
    if (batch < 0 || carried < 0 || length < 0 || width < 0) return fail(KOEMI_ERR_INVALID, "negative slot operand sizes");
    if (padded < carried + length || padded % 8 != 0) {
        return fail(KOEMI_ERR_INVALID, "padded slot count %lld must be a multiple of 8 and at least carried + length (%lld)",
                    static_cast<long long>(padded), static_cast<long long>(carried + length));
    }
    if (width % 4 != 0) return fail(KOEMI_ERR_INVALID, "slot operand width must be a multiple of 4");
    if (batch > 65535) return fail(KOEMI_ERR_INVALID, "slot operands take at most 65535 streams per call");
    if (batch == 0 || width == 0 || padded == 0) return KOEMI_OK;
    const bool ok = (carried == 0 || (aligned(carried_keys, 16) && aligned(carried_values, 16) && carried_stride % 4 == 0)) &&
                    (length == 0 || (aligned(keys, 16) && aligned(values, 16) && window_stride % 4 == 0)) &&
                    aligned(keys_out, 16) && aligned(values_t_out, 16);
    if (!ok) return fail(KOEMI_ERR_INVALID, "slot operands need 16-byte aligned rows");
    const dim3 grid(static_cast<unsigned>(ceil_div(padded, kSlotTile)), static_cast<unsigned>(ceil_div(width, kSlotTile)),
                    static_cast<unsigned>(batch));
    if (grid.y > 65535) return fail(KOEMI_ERR_INVALID, "slot operand width too large");
    return by_dtype(dtype, [&](auto tag) -> int {
        using T = decltype(tag);
        slot_operands_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(
            carried_keys, carried_values, carried_stride, carried, keys, values, window_stride, length, width, padded,
            static_cast<T *>(keys_out), static_cast<T *>(values_t_out));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    });
}
