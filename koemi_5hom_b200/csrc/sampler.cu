// Greedy token selection at decode: one pass over each row of fp32 logits,
// the PAD column scored as -inf, returning the index of the largest score
// with the semantics of torch.argmax on the masked row (the first index among
// equal maxima; NaN counts as larger than every number, the first NaN wins).
// Replaces TokenSampler's greedy path (runtime/fast_decode.py:40-87:
// index_fill of PAD with -inf, then argmax), which reads and writes a masked
// copy of the logits before reading them again.
#include "common.cuh"

namespace koemi {
namespace {

constexpr int kSamplerThreads = 512;

struct Best {
    float value;
    int64_t index;
};

// a ranks before b in argmax order
__device__ __forceinline__ bool before(const Best &a, const Best &b) {
    const bool na = isnan(a.value), nb = isnan(b.value);
    if (na != nb) return na;
    if (!na && a.value != b.value) return a.value > b.value;
    return a.index < b.index;
}

__device__ __forceinline__ void take(Best &best, float v, int64_t i, int64_t pad) {
    if (i == pad) v = -INFINITY;
    const Best candidate{v, i};
    if (before(candidate, best)) best = candidate;
}

__global__ __launch_bounds__(kSamplerThreads) void greedy_kernel(const float *__restrict__ logits, int64_t row_stride,
                                                                 int64_t vocab, int64_t pad, int64_t *__restrict__ out) {
    const int64_t row = blockIdx.x;
    const float *x = logits + row * row_stride;
    Best best{-INFINITY, vocab};  // ranks after every real entry
    const bool vector = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int64_t quads = vector ? vocab / 4 : 0;
    // eight packets per thread requested before any is compared
    constexpr int kInFlight = 8;
    for (int64_t q0 = threadIdx.x; q0 < quads; q0 += kInFlight * kSamplerThreads) {
        float4 v[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int64_t q = q0 + u * kSamplerThreads;
            v[u] = q < quads ? __ldg(reinterpret_cast<const float4 *>(x) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int64_t q = q0 + u * kSamplerThreads;
            if (q < quads) {
                take(best, v[u].x, 4 * q, pad);
                take(best, v[u].y, 4 * q + 1, pad);
                take(best, v[u].z, 4 * q + 2, pad);
                take(best, v[u].w, 4 * q + 3, pad);
            }
        }
    }
    for (int64_t i = 4 * quads + threadIdx.x; i < vocab; i += kSamplerThreads) take(best, x[i], i, pad);
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        Best other{__shfl_xor_sync(0xffffffffu, best.value, offset), __shfl_xor_sync(0xffffffffu, best.index, offset)};
        if (before(other, best)) best = other;
    }
    __shared__ Best warps[kSamplerThreads / 32];
    if ((threadIdx.x & 31) == 0) warps[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        Best result = warps[0];
        for (int w = 1; w < kSamplerThreads / 32; ++w) {
            if (before(warps[w], result)) result = warps[w];
        }
        out[row] = result.index < vocab ? result.index : 0;
    }
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_sampler_greedy(const float *logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                    int64_t pad_id, int64_t *out, void *stream) {
    clear_error();
    if (rows < 0 || vocab < 1 || row_stride < vocab) return fail(KOEMI_ERR_INVALID, "bad greedy sampler sizes");
    if (rows == 0) return KOEMI_OK;
    if (rows > 2147483647) return fail(KOEMI_ERR_INVALID, "too many rows");
    if (logits == nullptr || out == nullptr) return fail(KOEMI_ERR_INVALID, "logits and out must be non-NULL");
    greedy_kernel<<<static_cast<unsigned>(rows), kSamplerThreads, 0, as_stream(stream)>>>(logits, row_stride, vocab,
                                                                                          pad_id, out);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}
