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
// window; value and read rows stream through once, so the kernel is
// HBM-bound where the closed form materialises [T, T] pair weights.
//
// Grid (stream, row block): m/4 threads own one basis row as float4 packets
// in registers; per chunk of 64 positions the CTA stages the features,
// query features, gates and its rows' values in shared memory (coalesced),
// warp 0 walks the normaliser recurrence to produce each position's
// confidence and regulariser, then every row steps through the chunk.
#include "common.cuh"

namespace koemi {
namespace {

constexpr int kWindowThreads = 256;
constexpr float kReadEpsilon = 1.0f / 256.0f;

// Positions staged per chunk: 64, or 32 for 4 features (256 rows per CTA
// then, and the staged values must stay within the static shared memory).
template <int kM>
constexpr int window_chunk() {
    return kM >= 8 ? 64 : 32;
}

template <int kM>
__global__ __launch_bounds__(kWindowThreads) void assoc_window_kernel(
    const float *__restrict__ decay, const float *__restrict__ write, const float *__restrict__ value,
    const float *__restrict__ features, const float *__restrict__ query_features, float *__restrict__ basis,
    float *__restrict__ normalizer, float *__restrict__ read_out, int64_t length, int64_t d) {
    static_assert(kM % 4 == 0 && kM <= 32 && 32 % (kM / 4) == 0, "4, 8, 16 or 32 features");
    constexpr int kWindowChunk = window_chunk<kM>();
    constexpr int kParts = kM / 4;
    constexpr int kRows = kWindowThreads / kParts;
    __shared__ __align__(16) float sf[kWindowChunk][kM];
    __shared__ __align__(16) float sq[kWindowChunk][kM];
    __shared__ float sval[kWindowChunk][kRows];
    __shared__ float sdecay[kWindowChunk], swrite[kWindowChunk], sconf[kWindowChunk], sreg[kWindowChunk];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.x;
    const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kRows;
    const int local_row = threadIdx.x / kParts;
    const int part = threadIdx.x % kParts;
    const int64_t row = row0 + local_row;
    const bool live = row < d;
    float *brow = basis + (b * d + row) * kM;
    float4 x = live ? reinterpret_cast<const float4 *>(brow)[part] : make_float4(0.f, 0.f, 0.f, 0.f);
    float nrm = warp == 0 && lane < kM ? normalizer[b * kM + lane] : 0.0f;

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
        for (int i = threadIdx.x; i < n * kRows; i += kWindowThreads) {
            const int t = i / kRows, r = i % kRows;
            sval[t][r] = row0 + r < d ? value[(b * length + t0 + t) * d + row0 + r] : 0.0f;
        }
        __syncthreads();
        if (warp == 0) {  // normaliser recurrence: each position's confidence and regulariser
            for (int t = 0; t < n; ++t) {
                float den = lane < kM ? nrm * sq[t][lane] : 0.0f;
                den = warp_sum(den);
                if (lane == 0) {
                    const float reg = den + kReadEpsilon;
                    sconf[t] = den / reg;
                    sreg[t] = reg;
                }
                if (lane < kM) nrm = sdecay[t] * nrm + swrite[t] * sf[t][lane];
            }
        }
        __syncthreads();
        for (int t = 0; t < n; ++t) {
            const float4 qv = reinterpret_cast<const float4 *>(sq[t])[part];
            float num = x.x * qv.x + x.y * qv.y + x.z * qv.z + x.w * qv.w;
#pragma unroll
            for (int o = 1; o < kParts; o <<= 1) num += __shfl_xor_sync(0xffffffffu, num, o);
            if (live && part == 0) read_out[(b * length + t0 + t) * d + row] = sconf[t] * num / sreg[t];
            const float4 fv = reinterpret_cast<const float4 *>(sf[t])[part];
            const float dk = sdecay[t];
            const float v = swrite[t] * sval[t][local_row];
            x.x = dk * x.x + v * fv.x;
            x.y = dk * x.y + v * fv.y;
            x.z = dk * x.z + v * fv.z;
            x.w = dk * x.w + v * fv.w;
        }
    }
    if (live) reinterpret_cast<float4 *>(brow)[part] = x;
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
    auto run = [&](auto kernel, int rows_per_cta) -> int {
        const int64_t blocks_y = ceil_div(width, rows_per_cta);
        if (blocks_y > 65535) return fail(KOEMI_ERR_INVALID, "width too large");
        kernel<<<dim3(static_cast<unsigned>(batch), static_cast<unsigned>(blocks_y)), kWindowThreads, 0,
                 as_stream(stream)>>>(decay, write, value, features, query_features, basis, normalizer, read_out,
                                      length, width);
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    switch (feature_count) {
        case 4: return run(assoc_window_kernel<4>, kWindowThreads / 1);
        case 8: return run(assoc_window_kernel<8>, kWindowThreads / 2);
        case 16: return run(assoc_window_kernel<16>, kWindowThreads / 4);
        default: return run(assoc_window_kernel<32>, kWindowThreads / 8);
    }
}
