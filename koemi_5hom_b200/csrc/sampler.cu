// Greedy token selection at decode: one pass over each row of fp32 logits,
// the PAD column scored as -inf, returning the index of the largest score
// with the semantics of torch.argmax on the masked row (the first index among
// equal maxima; NaN counts as larger than every number, the first NaN wins).
// Replaces TokenSampler's greedy path (runtime/fast_decode.py:40-87:
// index_fill of PAD with -inf, then argmax), which reads and writes a masked
// copy of the logits before reading them again. The temperature path below
// replaces its softmax + multinomial chain with one pass per row.
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

// ------------------------------------------------------ temperature sampling
// Sampling from softmax(logits / T) as a Gumbel-max: the index of the
// largest logit_v / T + g_v with g_v = -log(-log(u_v)) and u_v uniform in
// (0, 1) is distributed exactly as softmax(logits / T). The uniforms come from
// a counter-based generator, so every (seed, stream, step, column) has its own
// number and a stream's draws do not depend on the batch it decodes in:
//   key  = splitmix64(seed ^ splitmix64(stream ^ splitmix64(step)))
//   bits = splitmix64(key + v * 0x9E3779B97F4A7C15)
//   u    = ((bits >> 41) + 0.5) / 2^23   (exact in fp32, never 0 or 1)
// splitmix64 is Steele, Lea and Flood's SplitMix finaliser (OOPSLA 2014):
//   z += 0x9E3779B97F4A7C15; z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9;
//   z = (z ^ (z >> 27)) * 0x94D049BB133111EB; return z ^ (z >> 31).
// The PAD column, NaN logits and (with `thresholds`) logits below the row's
// threshold are never chosen; ties go to the lower index.

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ void take_sample(Best &best, float logit, int64_t i, int64_t pad, float inv_t,
                                            float threshold, uint64_t key) {
    if (i == pad || isnan(logit) || logit < threshold) return;
    const uint64_t bits = splitmix64(key + static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull);
    const float u = (static_cast<float>(bits >> 41) + 0.5f) * (1.0f / 8388608.0f);
    const float score = logit * inv_t - logf(-logf(u));
    if (score > best.value || (score == best.value && i < best.index)) best = Best{score, i};
}

__global__ __launch_bounds__(kSamplerThreads) void gumbel_kernel(const float *__restrict__ logits, int64_t row_stride,
                                                                 int64_t vocab, int64_t pad, float inv_t, uint64_t seed,
                                                                 int64_t stream_offset, const int64_t *__restrict__ step,
                                                                 const float *__restrict__ thresholds,
                                                                 int64_t *__restrict__ out) {
    const int64_t row = blockIdx.x;
    const float *x = logits + row * row_stride;
    const uint64_t stream = static_cast<uint64_t>(stream_offset + row);
    const uint64_t key = splitmix64(seed ^ splitmix64(stream ^ splitmix64(static_cast<uint64_t>(*step))));
    const float threshold = thresholds != nullptr ? thresholds[row] : -INFINITY;
    Best best{-INFINITY, vocab};
    const bool vector = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int64_t quads = vector ? vocab / 4 : 0;
    for (int64_t q = threadIdx.x; q < quads; q += kSamplerThreads) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + q);
        take_sample(best, v.x, 4 * q, pad, inv_t, threshold, key);
        take_sample(best, v.y, 4 * q + 1, pad, inv_t, threshold, key);
        take_sample(best, v.z, 4 * q + 2, pad, inv_t, threshold, key);
        take_sample(best, v.w, 4 * q + 3, pad, inv_t, threshold, key);
    }
    for (int64_t i = 4 * quads + threadIdx.x; i < vocab; i += kSamplerThreads) {
        take_sample(best, x[i], i, pad, inv_t, threshold, key);
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        const Best other{__shfl_xor_sync(0xffffffffu, best.value, offset), __shfl_xor_sync(0xffffffffu, best.index, offset)};
        if (other.value > best.value || (other.value == best.value && other.index < best.index)) best = other;
    }
    __shared__ Best warps[kSamplerThreads / 32];
    if ((threadIdx.x & 31) == 0) warps[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        Best result = warps[0];
        for (int w = 1; w < kSamplerThreads / 32; ++w) {
            const Best &o = warps[w];
            if (o.value > result.value || (o.value == result.value && o.index < result.index)) result = o;
        }
        // a row with nothing to choose (every column masked) yields 0, as
        // greedy does for a row of -inf
        out[row] = result.index < vocab ? result.index : 0;
    }
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_sampler_temperature(const float *logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                         int64_t pad_id, float temperature, uint64_t seed, int64_t stream_offset,
                                         const int64_t *step, const float *thresholds, int64_t *out, void *stream) {
    clear_error();
    if (rows < 0 || vocab < 1 || row_stride < vocab) return fail(KOEMI_ERR_INVALID, "bad temperature sampler sizes");
    if (!(temperature > 0.0f)) return fail(KOEMI_ERR_INVALID, "temperature must be positive");
    if (rows == 0) return KOEMI_OK;
    if (rows > 2147483647) return fail(KOEMI_ERR_INVALID, "too many rows");
    if (logits == nullptr || out == nullptr || step == nullptr) {
        return fail(KOEMI_ERR_INVALID, "logits, step and out must be non-NULL");
    }
    gumbel_kernel<<<static_cast<unsigned>(rows), kSamplerThreads, 0, as_stream(stream)>>>(
        logits, row_stride, vocab, pad_id, 1.0f / temperature, seed, stream_offset, step, thresholds, out);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

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
