// Associative memory over a window (prefill): the rank-one decayed memory of
// HierarchicalAssociativeMemory.scan_and_read (model/memory.py:97-144,
// 146-242, 248-255) for T positions of every stream, in its sequential form:
//
//   den_t  = n_{t-1} . q_t,   reg_t = den_t + 2^-8
//   read_t[i] = (den_t / reg_t) * (B_{t-1}[i] . q_t) / reg_t
//   B_t[i] = decay_t B_{t-1}[i] + write_t value_t[i] f_t,   n_t = decay_t n_{t-1} + write_t f_t
//
// which is what the reference's chunk-pairwise closed form computes (every
// write strictly before t, decayed by the product of the later decays). The
// state (basis rows [d, m], normaliser [m]) is read once and written once per
// window and value and read rows stream through once, where the closed form
// materialises [T, T] pair weights.
//
// Grid (stream, row block), 128 threads: every thread owns R = 64 / m
// consecutive basis rows (2 for 32 features) in registers, so the staged
// per-position operands (query features, features, gates) are read from
// shared memory once per R rows and the dot products need no shuffles; the
// kernel is FMA-bound (2 m FMAs per row and position). Per chunk of 64
// positions the CTA stages the features, query features and gates, warp 0
// walks the normaliser recurrence (one FMA per step and feature, the state
// before each position kept), every position's read scale (den / reg) / reg
// follows in parallel, then every thread steps its rows through the chunk,
// its value rows loaded from global two positions ahead and its read rows
// stored straight back (R consecutive floats per thread: coalesced).
#include "common.cuh"

namespace koemi {
namespace {

constexpr int kWindowThreads = 128;
constexpr int kWindowChunk = 64;
constexpr float kReadEpsilon = 1.0f / 256.0f;

template <int kM>
constexpr int rows_per_thread() {
    return kM >= 32 ? 2 : 64 / kM;
}

// R consecutive floats of a row block starting at `p` (rows past `live`
// read as zero). kVec: p is 8-byte (R = 2) or 16-byte aligned and live is a
// multiple of the vector width.
template <int kR, bool kVec>
__device__ __forceinline__ void load_rows(const float *p, int live, float (&out)[kR]) {
    if constexpr (kVec && kR % 4 == 0) {
#pragma unroll
        for (int i = 0; i < kR; i += 4) {
            const float4 v = i < live ? __ldg(reinterpret_cast<const float4 *>(p + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            out[i] = v.x;
            out[i + 1] = v.y;
            out[i + 2] = v.z;
            out[i + 3] = v.w;
        }
    } else if constexpr (kVec && kR == 2) {
        const float2 v = live > 0 ? __ldg(reinterpret_cast<const float2 *>(p)) : make_float2(0.f, 0.f);
        out[0] = v.x;
        out[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < kR; ++i) out[i] = i < live ? __ldg(p + i) : 0.0f;
    }
}

template <int kR, bool kVec>
__device__ __forceinline__ void store_rows(float *p, int live, const float (&in)[kR]) {
    if constexpr (kVec && kR % 4 == 0) {
#pragma unroll
        for (int i = 0; i < kR; i += 4) {
            if (i < live) *reinterpret_cast<float4 *>(p + i) = make_float4(in[i], in[i + 1], in[i + 2], in[i + 3]);
        }
    } else if constexpr (kVec && kR == 2) {
        if (live > 0) *reinterpret_cast<float2 *>(p) = make_float2(in[0], in[1]);
    } else {
#pragma unroll
        for (int i = 0; i < kR; ++i) {
            if (i < live) p[i] = in[i];
        }
    }
}

template <int kM, bool kVec>
__global__ __launch_bounds__(kWindowThreads) void assoc_window_kernel(
    const float *__restrict__ decay, const float *__restrict__ write, const float *__restrict__ value,
    const float *__restrict__ features, const float *__restrict__ query_features, float *__restrict__ basis,
    float *__restrict__ normalizer, float *__restrict__ read_out, int64_t length, int64_t d) {
    static_assert(kM % 4 == 0 && kM <= 32, "4, 8, 16 or 32 features");
    constexpr int kR = rows_per_thread<kM>();
    constexpr int kQ = kM / 4;
    __shared__ __align__(16) float sf[kWindowChunk][kM];
    __shared__ __align__(16) float sq[kWindowChunk][kM];
    __shared__ __align__(16) float sn[kWindowChunk][kM];
    __shared__ float sdecay[kWindowChunk], swrite[kWindowChunk], sscale[kWindowChunk];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.x;
    const int64_t row = static_cast<int64_t>(blockIdx.y) * (kWindowThreads * kR) + threadIdx.x * kR;
    const int live = static_cast<int>(max(static_cast<int64_t>(0), min(static_cast<int64_t>(kR), d - row)));

    float x[kR][kM];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        const float *brow = basis + (b * d + row + r) * kM;
#pragma unroll
        for (int q = 0; q < kQ; ++q) {
            const float4 v = r < live ? reinterpret_cast<const float4 *>(brow)[q] : make_float4(0.f, 0.f, 0.f, 0.f);
            x[r][4 * q] = v.x;
            x[r][4 * q + 1] = v.y;
            x[r][4 * q + 2] = v.z;
            x[r][4 * q + 3] = v.w;
        }
    }
    float nrm = warp == 0 && lane < kM ? normalizer[b * kM + lane] : 0.0f;

    // value rows two positions ahead
    const float *vbase = value + b * length * d + row;
    float v0[kR], v1[kR] = {};
    load_rows<kR, kVec>(vbase, live, v0);
    if (length > 1) load_rows<kR, kVec>(vbase + d, live, v1);

    for (int64_t t0 = 0; t0 < length; t0 += kWindowChunk) {
        const int n = static_cast<int>(length - t0 < kWindowChunk ? length - t0 : kWindowChunk);
        __syncthreads();  // the previous chunk's readers are done with the staging buffers
        for (int i = threadIdx.x; i < n * kM; i += kWindowThreads) {
            const int64_t at = (b * length + t0) * kM + i;
            sf[i / kM][i % kM] = features[at];
            sq[i / kM][i % kM] = query_features[at];
        }
        for (int i = threadIdx.x; i < n; i += kWindowThreads) {
            sdecay[i] = decay[b * length + t0 + i];
            swrite[i] = write[b * length + t0 + i];
        }
        __syncthreads();
        if (warp == 0 && lane < kM) {  // normaliser before each position
            for (int t = 0; t < n; ++t) {
                sn[t][lane] = nrm;
                nrm = sdecay[t] * nrm + swrite[t] * sf[t][lane];
            }
        }
        __syncthreads();
        for (int t = threadIdx.x; t < n; t += kWindowThreads) {  // confidence and regulariser
            float den = 0.0f;
#pragma unroll
            for (int m = 0; m < kM; ++m) den += sn[t][m] * sq[t][m];
            const float reg = den + kReadEpsilon;
            sscale[t] = den / reg / reg;  // read = (den / reg) (B . q) / reg
        }
        __syncthreads();
        for (int t = 0; t < n; ++t) {
            const int64_t tt = t0 + t;
            float v2[kR] = {};
            if (tt + 2 < length) load_rows<kR, kVec>(vbase + (tt + 2) * d, live, v2);
            float num[kR];
#pragma unroll
            for (int r = 0; r < kR; ++r) num[r] = 0.0f;
#pragma unroll
            for (int q = 0; q < kQ; ++q) {
                const float4 qv = reinterpret_cast<const float4 *>(sq[t])[q];
#pragma unroll
                for (int r = 0; r < kR; ++r) {
                    num[r] += x[r][4 * q] * qv.x + x[r][4 * q + 1] * qv.y + x[r][4 * q + 2] * qv.z + x[r][4 * q + 3] * qv.w;
                }
            }
            const float scale = sscale[t];
            float out[kR];
#pragma unroll
            for (int r = 0; r < kR; ++r) out[r] = scale * num[r];
            store_rows<kR, kVec>(read_out + (b * length + tt) * d + row, live, out);
            const float dk = sdecay[t], wr = swrite[t];
#pragma unroll
            for (int q = 0; q < kQ; ++q) {
                const float4 fv = reinterpret_cast<const float4 *>(sf[t])[q];
#pragma unroll
                for (int r = 0; r < kR; ++r) {
                    const float v = wr * v0[r];
                    x[r][4 * q] = dk * x[r][4 * q] + v * fv.x;
                    x[r][4 * q + 1] = dk * x[r][4 * q + 1] + v * fv.y;
                    x[r][4 * q + 2] = dk * x[r][4 * q + 2] + v * fv.z;
                    x[r][4 * q + 3] = dk * x[r][4 * q + 3] + v * fv.w;
                }
            }
#pragma unroll
            for (int r = 0; r < kR; ++r) {
                v0[r] = v1[r];
                v1[r] = v2[r];
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kR; ++r) {
        if (r < live) {
            float *brow = basis + (b * d + row + r) * kM;
#pragma unroll
            for (int q = 0; q < kQ; ++q) {
                reinterpret_cast<float4 *>(brow)[q] = make_float4(x[r][4 * q], x[r][4 * q + 1], x[r][4 * q + 2], x[r][4 * q + 3]);
            }
        }
    }
    if (blockIdx.y == 0 && warp == 0 && lane < kM) normalizer[b * kM + lane] = nrm;
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_assoc_window_scan_read(const float *decay, const float *write, const float *value,
                                            const float *features, const float *query_features, float *basis,
                                            float *normalizer, float *read_out, int64_t batch, int64_t length,
                                            int64_t width, int64_t feature_count, void *stream) {
    clear_error();
    if (batch < 0 || length < 0 || width < 0) return fail(KOEMI_ERR_INVALID, "negative associative window sizes");
    if (batch == 0 || length == 0 || width == 0) return KOEMI_OK;
    if (feature_count != 4 && feature_count != 8 && feature_count != 16 && feature_count != 32) {
        return fail(KOEMI_ERR_UNSUPPORTED,
                    "the window associative kernel is built for 4, 8, 16 or 32 memory features (got %lld); "
                    "pad the features with zeros to the next of these", static_cast<long long>(feature_count));
    }
    if (!aligned(basis, 16)) return fail(KOEMI_ERR_INVALID, "basis must be 16-byte aligned");
    if (batch > 2147483647) return fail(KOEMI_ERR_INVALID, "too many streams");
    const bool vec = width % 4 == 0 && aligned(value, 16) && aligned(read_out, 16);
    auto run = [&](auto kernel, int rows_per_cta) -> int {
        const int64_t blocks_y = ceil_div(width, rows_per_cta);
        if (blocks_y > 65535) return fail(KOEMI_ERR_INVALID, "width too large");
        kernel<<<dim3(static_cast<unsigned>(batch), static_cast<unsigned>(blocks_y)), kWindowThreads, 0,
                 as_stream(stream)>>>(decay, write, value, features, query_features, basis, normalizer, read_out,
                                      length, width);
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    auto pick = [&](auto features_tag) -> int {
        constexpr int kM = decltype(features_tag)::value;
        constexpr int rows = kWindowThreads * rows_per_thread<kM>();
        return vec ? run(assoc_window_kernel<kM, true>, rows) : run(assoc_window_kernel<kM, false>, rows);
    };
    switch (feature_count) {
        case 4: return pick(std::integral_constant<int, 4>());
        case 8: return pick(std::integral_constant<int, 8>());
        case 16: return pick(std::integral_constant<int, 16>());
        default: return pick(std::integral_constant<int, 32>());
    }
}
