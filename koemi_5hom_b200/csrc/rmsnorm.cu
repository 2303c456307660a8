// Core front: single-pass RMSNorm row kernels.
//
// One warp owns one row. When the row fits (up to 8 x 16-byte packets per
// lane, i.e. 2048 bf16 / 1024 fp32 columns) it is held in registers between
// the sum of squares and the output pass, so every input byte is read from
// HBM once and every output byte written once; longer rows take a two-pass
// variant whose second read is served by L1/L2. All arithmetic is fp32.
// Reference kernel: core/rmsnorm_silu.cu:63-91 (one block per row, two passes
// over the row, default stream); model norm: model/layers.py:8-16.
#include <cmath>
#include <type_traits>

#include "vec.cuh"

namespace koemi {
namespace {

enum Mode : int { kSilu = 0, kGated = 1, kPlain = 2 };

constexpr int kRowsPerBlock = 8;
constexpr int kThreads = kRowsPerBlock * 32;

struct RowArgs {
    const void *x;
    const void *gate;      // kGated
    const void *residual;  // kPlain, may be null
    const void *weight;
    const uint8_t *keep;   // kPlain, may be null
    void *y;
    float *inv_rms;        // may be null
    int64_t rows;
    int64_t hidden;
    float eps;
};

template <typename T, int kMode>
__device__ __forceinline__ void finish_pack(float (&v)[Pack<T>::kWidth], const float (&w)[Pack<T>::kWidth],
                                            const float (&g)[Pack<T>::kWidth], float inv) {
#pragma unroll
    for (int e = 0; e < Pack<T>::kWidth; ++e) {
        const float n = v[e] * inv * w[e];
        if (kMode == kSilu) {
            v[e] = silu_fast(n);
        } else if (kMode == kGated) {
            v[e] = silu_fast(g[e]) * n;
        } else {
            v[e] = n;
        }
    }
}

// Stores W fp32 results (one input packet's worth) as TO: 16 bytes, 8 bytes
// (four 16-bit values from an fp32 packet) or 32 bytes (eight fp32 values
// from a 16-bit packet).
template <typename TO, int W>
__device__ __forceinline__ void store_converted(TO *dst, const float (&v)[W]) {
    if constexpr (sizeof(TO) * W == 16) {
        store_stream(dst, pack(v, TO()));
    } else if constexpr (sizeof(TO) * W == 8) {
        union {
            TO h[4];
            uint2 u;
        } out;
#pragma unroll
        for (int e = 0; e < 4; ++e) out.h[e] = from_acc<TO>(v[e]);
        *reinterpret_cast<uint2 *>(dst) = out.u;
    } else {
        static_assert(sizeof(TO) * W == 32, "unsupported packet conversion");
        const float lo[4] = {v[0], v[1], v[2], v[3]};
        const float hi[4] = {v[4], v[5], v[6], v[7]};
        store_stream(dst, pack(lo, float()));
        store_stream(dst + 4, pack(hi, float()));
    }
}

// Cached vector path: NV packets of T per lane stay in registers; the
// output may be another floating type TO.
template <typename T, typename TO, int kMode, int NV>
__global__ __launch_bounds__(kThreads) void rms_rows_cached(RowArgs args) {
    pdl_trigger();
    pdl_wait();
    constexpr int W = Pack<T>::kWidth;
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= args.rows) return;
    const int64_t packets = args.hidden / W;
    const T *xr = static_cast<const T *>(args.x) + row * args.hidden;
    const T *rr = args.residual ? static_cast<const T *>(args.residual) + row * args.hidden : nullptr;
    const T *gr = kMode == kGated ? static_cast<const T *>(args.gate) + row * args.hidden : nullptr;
    const T *wr = static_cast<const T *>(args.weight);
    TO *yr = static_cast<TO *>(args.y) + row * args.hidden;
    const bool keep = kMode != kPlain || args.keep == nullptr || args.keep[row] != 0;

    uint4 raw[NV];
    uint4 graw[NV];
    uint4 wraw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t p = lane + 32 * i;
        if (p < packets) {
            raw[i] = load_stream(xr + p * W);
            if (kMode == kGated) graw[i] = load_stream(gr + p * W);
            wraw[i] = load_cached(wr + p * W);  // all loads in flight before the first use
        }
    }
    float v[NV][W];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t p = lane + 32 * i;
        if (p < packets) {
            unpack(raw[i], v[i], T());
            if (kMode == kPlain && rr != nullptr) {
                float r[W];
                unpack(load_stream(rr + p * W), r, T());
#pragma unroll
                for (int e = 0; e < W; ++e) v[i][e] += r[e];
            }
#pragma unroll
            for (int e = 0; e < W; ++e) sum = fmaf(v[i][e], v[i][e], sum);
        }
    }
    sum = warp_sum(sum);
    const float inv = rsqrtf(sum / static_cast<float>(args.hidden) + args.eps);
    if (lane == 0 && args.inv_rms != nullptr) args.inv_rms[row] = inv;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t p = lane + 32 * i;
        if (p < packets) {
            if (!keep) {
                if constexpr (std::is_same<T, TO>::value) {
                    store_stream(yr + p * W, raw[i]);
                } else {
                    float x[W];
                    unpack(raw[i], x, T());
                    store_converted(yr + p * W, x);
                }
                continue;
            }
            float w[W], g[W];
            unpack(wraw[i], w, T());
            if (kMode == kGated) unpack(graw[i], g, T());
            finish_pack<T, kMode>(v[i], w, g, inv);
            store_converted(yr + p * W, v[i]);
        }
    }
}

// Scalar two-pass path for any width, alignment and in/out dtype pair.
template <typename T, typename TO, int kMode>
__global__ __launch_bounds__(kThreads) void rms_rows_scalar(RowArgs args) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= args.rows) return;
    const int64_t hidden = args.hidden;
    const T *xr = static_cast<const T *>(args.x) + row * hidden;
    const T *rr = args.residual ? static_cast<const T *>(args.residual) + row * hidden : nullptr;
    const T *gr = kMode == kGated ? static_cast<const T *>(args.gate) + row * hidden : nullptr;
    const T *wr = static_cast<const T *>(args.weight);
    TO *yr = static_cast<TO *>(args.y) + row * hidden;
    const bool keep = kMode != kPlain || args.keep == nullptr || args.keep[row] != 0;
    float sum = 0.0f;
    for (int64_t c = lane; c < hidden; c += 32) {
        float v = to_acc(xr[c]);
        if (rr != nullptr) v += to_acc(rr[c]);
        sum = fmaf(v, v, sum);
    }
    sum = warp_sum(sum);
    const float inv = rsqrtf(sum / static_cast<float>(hidden) + args.eps);
    if (lane == 0 && args.inv_rms != nullptr) args.inv_rms[row] = inv;
    for (int64_t c = lane; c < hidden; c += 32) {
        const float x = to_acc(xr[c]);
        if (!keep) {
            yr[c] = from_acc<TO>(x);
            continue;
        }
        float v = x;
        if (rr != nullptr) v += to_acc(rr[c]);
        const float n = v * inv * to_acc(wr[c]);
        float out;
        if (kMode == kSilu) {
            out = siluf_(n);
        } else if (kMode == kGated) {
            out = siluf_(to_acc(gr[c])) * n;
        } else {
            out = n;
        }
        yr[c] = from_acc<TO>(out);
    }
}

// Streamed path for many rows (the front at prefill and benchmark sizes):
// a persistent CTA per SM whose producer warp moves groups of 8 consecutive
// rows -- one contiguous block of x and one of the gate -- into a ring of
// shared-memory stages with 1D bulk copies (cp.async.bulk, completion on an
// mbarrier), while 8 consumer warps each normalise one row of the group
// from shared memory and store the result straight to HBM. Loads for later
// groups are in flight while earlier ones are computed, so HBM sees a steady
// stream instead of the load/compute/store bursts of one-shot row blocks.
// Two groups of 8 consumer warps take alternate stages, so each scheduler
// has four warps to hide the latency of the per-row reduction.
constexpr int kStreamWarps = 8;
constexpr int kStreamGroups = 2;
constexpr int kStreamThreads = (kStreamGroups * kStreamWarps + 1) * 32;
constexpr int kStreamMaxStages = 8;
constexpr size_t kStreamSmemBudget = 200 * 1024;

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

template <typename T, int kMode, int NV>
__global__ __launch_bounds__(kStreamThreads) void rms_rows_streamed(RowArgs args, int stages, int *status) {
    constexpr int W = Pack<T>::kWidth;
    constexpr int kArrays = kMode == kGated ? 2 : 1;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int64_t row_bytes = args.hidden * static_cast<int64_t>(sizeof(T));
    const int64_t stage_bytes = kStreamWarps * row_bytes * kArrays;
    unsigned char *ring = smem_raw;
    T *weight_s = reinterpret_cast<T *>(ring + stages * stage_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + stages * stage_bytes + ((row_bytes + 15) / 16) * 16);
    uint64_t *empty = full + kStreamMaxStages;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t groups = (args.rows + kStreamWarps - 1) / kStreamWarps;
    const int64_t packets = args.hidden / W;
    for (int64_t p = threadIdx.x; p < packets; p += kStreamThreads) {
        reinterpret_cast<uint4 *>(weight_s)[p] = load_cached(static_cast<const T *>(args.weight) + p * W);
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kStreamGroups * kStreamWarps) {
        if (lane == 0) {
            // Stage s, its fill count `round` (phase parity = round & 1).
            int s = 0, round = 0, issued = 0;
            for (int64_t g = blockIdx.x; g < groups; g += gridDim.x, ++issued) {
                if (round > 0 && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>((round - 1) & 1), status)) break;
                const int64_t first = g * kStreamWarps;
                const int64_t count = args.rows - first < kStreamWarps ? args.rows - first : kStreamWarps;
                const uint32_t bytes = static_cast<uint32_t>(count * row_bytes);
                mbar_arrive_expect_tx(&full[s], bytes * kArrays);
                unsigned char *dst = ring + s * stage_bytes;
                bulk_load(dst, static_cast<const T *>(args.x) + first * args.hidden, bytes, &full[s]);
                if (kMode == kGated) {
                    bulk_load(dst + kStreamWarps * row_bytes, static_cast<const T *>(args.gate) + first * args.hidden,
                              bytes, &full[s]);
                }
                if (++s == stages) {
                    s = 0;
                    ++round;
                }
            }
            // Drain: the newest copy of every stage has landed before the CTA
            // leaves (stage t was last filled in round `round` if t < s, else
            // in round - 1).
            for (int t = 0; t < stages && t < issued; ++t) {
                const int last_round = t < s ? round : round - 1;
                mbar_wait_bounded(&full[t], static_cast<uint32_t>(last_round & 1), nullptr);
            }
        }
        return;
    }

    // Consumer group `team` takes the block's groups k = team, team + 2, ...
    const int team = warp / kStreamWarps;
    const int member = warp % kStreamWarps;
    int s = team % stages, round = team / stages;
    for (int64_t g = blockIdx.x + int64_t(team) * gridDim.x; g < groups; g += int64_t(kStreamGroups) * gridDim.x) {
        if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(round & 1), status)) break;
        const int64_t row = g * kStreamWarps + member;
        if (row < args.rows) {
            const unsigned char *base = ring + s * stage_bytes + member * row_bytes;
            const uint4 *xs = reinterpret_cast<const uint4 *>(base);
            const uint4 *gs = reinterpret_cast<const uint4 *>(base + kStreamWarps * row_bytes);
            uint4 raw[NV];
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int64_t p = lane + 32 * i;
                if (p < packets) {
                    raw[i] = xs[p];
                    float v[W];
                    unpack(raw[i], v, T());
#pragma unroll
                    for (int e = 0; e < W; ++e) sum = fmaf(v[e], v[e], sum);
                }
            }
            sum = warp_sum(sum);
            const float inv = rsqrtf(sum / static_cast<float>(args.hidden) + args.eps);
            if (lane == 0 && args.inv_rms != nullptr) args.inv_rms[row] = inv;
            T *yr = static_cast<T *>(args.y) + row * args.hidden;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int64_t p = lane + 32 * i;
                if (p < packets) {
                    float v[W], w[W], gv[W];
                    unpack(raw[i], v, T());
                    unpack(reinterpret_cast<const uint4 *>(weight_s)[p], w, T());
                    if (kMode == kGated) unpack(gs[p], gv, T());
                    finish_pack<T, kMode>(v, w, gv, inv);
                    store_stream(yr + p * W, pack(v, T()));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        s += kStreamGroups;
        while (s >= stages) {
            s -= stages;
            ++round;
        }
    }
}

template <typename T, int kMode>
size_t streamed_smem(int64_t hidden, int *stages_out) {
    const size_t row_bytes = static_cast<size_t>(hidden) * sizeof(T);
    const size_t stage_bytes = kStreamWarps * row_bytes * (kMode == kGated ? 2 : 1);
    const size_t fixed = ((row_bytes + 15) / 16) * 16 + 2 * kStreamMaxStages * sizeof(uint64_t);
    int stages = static_cast<int>((kStreamSmemBudget - fixed) / stage_bytes);
    if (stages > kStreamMaxStages) stages = kStreamMaxStages;
    *stages_out = stages;
    return stages * stage_bytes + fixed;
}

// Streamed path when: same in/out dtype, SiLU or gated mode, 16-byte aligned
// rows of at most 8 packets per lane, and at least four groups per SM.
template <typename T, typename TO, int kMode>
bool try_launch_streamed(const RowArgs &args, cudaStream_t stream, int *rc) {
    if constexpr (!std::is_same<T, TO>::value || kMode == kPlain) {
        return false;
    } else {
        constexpr int W = Pack<T>::kWidth;
        const int64_t packets = args.hidden / W;
        if (args.hidden % W != 0 || packets > 32 * 8 || !aligned(args.x, 16) || !aligned(args.weight, 16) ||
            !aligned(args.y, 16) || (kMode == kGated && !aligned(args.gate, 16))) {
            return false;
        }
        const int64_t groups = ceil_div(args.rows, kStreamWarps);
        const int64_t sms = sm_count();
        if (groups < 4 * sms) return false;
        int stages = 0;
        const size_t smem = streamed_smem<T, kMode>(args.hidden, &stages);
        if (stages < 2) return false;
        auto kernel = packets > 32 * 4 ? rms_rows_streamed<T, kMode, 8> : rms_rows_streamed<T, kMode, 4>;
        *rc = KOEMI_OK;
        cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err == cudaSuccess) {
            kernel<<<static_cast<unsigned>(sms), kStreamThreads, smem, stream>>>(args, stages, device_status_word());
            err = cudaGetLastError();
        }
        if (err != cudaSuccess) *rc = fail(KOEMI_ERR_CUDA, "streamed RMSNorm launch failed: %s", cudaGetErrorString(err));
        return true;
    }
}

template <typename T, typename TO, int kMode>
int launch_rows(const RowArgs &args, cudaStream_t stream) {
    // few rows (decode steps): 2 rows per block so the rows spread over the SMs
    const int rows_per_block = args.rows >= static_cast<int64_t>(sm_count()) * 32 ? kRowsPerBlock : 2;
    const int threads = rows_per_block * 32;
    const unsigned blocks = static_cast<unsigned>(ceil_div(args.rows, rows_per_block));
    int streamed_rc = KOEMI_OK;
    if (try_launch_streamed<T, TO, kMode>(args, stream, &streamed_rc)) return streamed_rc;
    constexpr int W = Pack<T>::kWidth;
    bool vector_ok = args.hidden % W == 0 && aligned(args.x, 16) &&
                     aligned(args.weight, 16) && aligned(args.y, 16) &&
                     (args.residual == nullptr || aligned(args.residual, 16)) &&
                     (kMode != kGated || aligned(args.gate, 16));
    if (vector_ok) {
        const int64_t per_lane = ceil_div(args.hidden / W, 32);
        if (per_lane <= 1) {
            KOEMI_CUDA_TRY(launch_pdl(rms_rows_cached<T, TO, kMode, 1>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
        } else if (per_lane <= 2) {
            KOEMI_CUDA_TRY(launch_pdl(rms_rows_cached<T, TO, kMode, 2>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
        } else if (per_lane <= 4) {
            KOEMI_CUDA_TRY(launch_pdl(rms_rows_cached<T, TO, kMode, 4>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
        } else if (per_lane <= 8) {
            KOEMI_CUDA_TRY(launch_pdl(rms_rows_cached<T, TO, kMode, 8>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
        } else if (per_lane <= 16 && sizeof(T) == 4 && kMode == kPlain) {
            KOEMI_CUDA_TRY(launch_pdl(rms_rows_cached<T, TO, kMode, 16>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
        } else {
            vector_ok = false;
        }
        if (vector_ok) {
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        }
    }
    KOEMI_CUDA_TRY(launch_pdl(rms_rows_scalar<T, TO, kMode>, dim3(blocks), dim3(threads), 0, stream, dim3(1, 1, 1), args));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

template <int kMode>
int dispatch_rows(const RowArgs &args, int dtype, int out_dtype, cudaStream_t stream) {
    if (dtype == KOEMI_F32 && out_dtype == KOEMI_F32) return launch_rows<float, float, kMode>(args, stream);
    if (dtype == KOEMI_BF16 && out_dtype == KOEMI_BF16) return launch_rows<__nv_bfloat16, __nv_bfloat16, kMode>(args, stream);
    if (dtype == KOEMI_F16 && out_dtype == KOEMI_F16) return launch_rows<__half, __half, kMode>(args, stream);
    if (dtype == KOEMI_F32 && out_dtype == KOEMI_BF16) return launch_rows<float, __nv_bfloat16, kMode>(args, stream);
    if (dtype == KOEMI_F32 && out_dtype == KOEMI_F16) return launch_rows<float, __half, kMode>(args, stream);
    if (dtype == KOEMI_BF16 && out_dtype == KOEMI_F32) return launch_rows<__nv_bfloat16, float, kMode>(args, stream);
    if (dtype == KOEMI_F16 && out_dtype == KOEMI_F32) return launch_rows<__half, float, kMode>(args, stream);
    return fail(KOEMI_ERR_INVALID, "unsupported RMSNorm dtype pair (%d, %d)", dtype, out_dtype);
}

int check_rows(int64_t rows, int64_t hidden, float eps) {
    if (rows < 0 || hidden < 0) return fail(KOEMI_ERR_INVALID, "rows and hidden must be non-negative");
    if (!(eps > 0.0f) || !std::isfinite(eps)) return fail(KOEMI_ERR_INVALID, "eps must be a finite positive number");
    if (rows > (int64_t(1) << 31) * kRowsPerBlock) return fail(KOEMI_ERR_INVALID, "too many rows");
    return KOEMI_OK;
}

// ---------------------------------------------------------------- backward
// One block walks a contiguous range of rows; each thread owns the columns
// c = tid + 256 j and keeps its grad_weight partials in shared memory, so the
// per-block partials and the final column sum run in a fixed order
// (deterministic, unlike the float atomics of core/rmsnorm_silu.cu:130).
constexpr int kBackThreads = 256;

__device__ __forceinline__ float silu_grad(float v) {
    const float s = sigmoidf_(v);
    return s * (1.0f + v * (1.0f - s));
}

template <typename T>
__global__ __launch_bounds__(kBackThreads) void rmsnorm_silu_backward_kernel(
    const T *__restrict__ grad_y, const T *__restrict__ x, const T *__restrict__ weight,
    const float *__restrict__ inv_rms, T *__restrict__ grad_x, float *__restrict__ partials,
    int64_t rows, int64_t hidden) {
    extern __shared__ float shared[];
    float *partial = shared;            // [hidden]
    float *warp_sums = shared + hidden;  // [8]
    for (int64_t c = threadIdx.x; c < hidden; c += kBackThreads) partial[c] = 0.0f;
    const int64_t begin = rows * blockIdx.x / gridDim.x;
    const int64_t end = rows * (blockIdx.x + 1) / gridDim.x;
    for (int64_t row = begin; row < end; ++row) {
        const float inv = inv_rms[row];
        const T *xr = x + row * hidden;
        const T *gr = grad_y + row * hidden;
        float dot = 0.0f;
        for (int64_t c = threadIdx.x; c < hidden; c += kBackThreads) {
            const float xv = to_acc(xr[c]);
            const float w = to_acc(weight[c]);
            const float pre = xv * inv * w;
            const float d = to_acc(gr[c]) * silu_grad(pre);
            dot = fmaf(d * w, xv, dot);
        }
        dot = warp_sum(dot);
        if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = dot;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w = 0; w < kBackThreads / 32; ++w) total += warp_sums[w];
        const float scale = inv * inv * inv / static_cast<float>(hidden);
        for (int64_t c = threadIdx.x; c < hidden; c += kBackThreads) {
            const float xv = to_acc(xr[c]);
            const float w = to_acc(weight[c]);
            const float normalized = xv * inv;
            const float d = to_acc(gr[c]) * silu_grad(normalized * w);
            grad_x[row * hidden + c] = from_acc<T>(inv * d * w - xv * scale * total);
            partial[c] += d * normalized;
        }
        __syncthreads();
    }
    for (int64_t c = threadIdx.x; c < hidden; c += kBackThreads) {
        partials[static_cast<int64_t>(blockIdx.x) * hidden + c] = partial[c];
    }
}

__global__ void column_sum_kernel(const float *__restrict__ partials, float *__restrict__ out,
                                  int64_t blocks, int64_t hidden) {
    const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    float total = 0.0f;
    for (int64_t b = 0; b < blocks; ++b) total += partials[b * hidden + c];
    out[c] = total;
}

int64_t backward_blocks(int64_t rows) {
    const int64_t cap = static_cast<int64_t>(sm_count()) * 2;
    return rows < cap ? (rows > 0 ? rows : 1) : cap;
}

template <typename T>
int rmsnorm_silu_backward_typed(const void *grad_y, const void *x, const void *weight,
                                const float *inv_rms, void *grad_x, float *grad_weight,
                                int64_t rows, int64_t hidden, float *partials, cudaStream_t stream) {
    const int64_t blocks = backward_blocks(rows);
    const size_t smem = (static_cast<size_t>(hidden) + 8) * sizeof(float);
    if (smem > 227 * 1024) return fail(KOEMI_ERR_UNSUPPORTED, "hidden %lld is too wide for the backward", (long long)hidden);
    auto kernel = rmsnorm_silu_backward_kernel<T>;
    if (smem > 48 * 1024) {
        KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    }
    kernel<<<static_cast<unsigned>(blocks), kBackThreads, smem, stream>>>(
        static_cast<const T *>(grad_y), static_cast<const T *>(x), static_cast<const T *>(weight),
        inv_rms, static_cast<T *>(grad_x), partials, rows, hidden);
    KOEMI_LAUNCH_CHECK();
    column_sum_kernel<<<static_cast<unsigned>(ceil_div(hidden, 256)), 256, 0, stream>>>(
        partials, grad_weight, blocks, hidden);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_core_rmsnorm_silu_forward(const void *x, const void *weight, void *y,
                                               float *inv_rms, int64_t rows, int64_t hidden,
                                               float eps, int dtype, void *stream) {
    clear_error();
    int rc = check_rows(rows, hidden, eps);
    if (rc != KOEMI_OK) return rc;
    if (rows == 0 || hidden == 0) return KOEMI_OK;
    if (dtype == KOEMI_F64) return fail(KOEMI_ERR_INVALID, "RMSNorm-SiLU supports f32, f16 and bf16");
    RowArgs args{x, nullptr, nullptr, weight, nullptr, y, inv_rms, rows, hidden, eps};
    return dispatch_rows<kSilu>(args, dtype, dtype, as_stream(stream));
}

extern "C" int koemi_core_gated_rmsnorm_silu_forward(const void *x, const void *gate,
                                                     const void *weight, void *y, float *inv_rms,
                                                     int64_t rows, int64_t hidden, float eps,
                                                     int dtype, void *stream) {
    clear_error();
    int rc = check_rows(rows, hidden, eps);
    if (rc != KOEMI_OK) return rc;
    if (rows == 0 || hidden == 0) return KOEMI_OK;
    if (gate == nullptr) return fail(KOEMI_ERR_INVALID, "gate must be non-NULL");
    RowArgs args{x, gate, nullptr, weight, nullptr, y, inv_rms, rows, hidden, eps};
    return dispatch_rows<kGated>(args, dtype, dtype, as_stream(stream));
}

extern "C" int koemi_core_rmsnorm_forward(const void *x, const void *residual, const void *weight,
                                          const uint8_t *keep, void *y, int64_t rows,
                                          int64_t hidden, float eps, int dtype, int out_dtype,
                                          void *stream) {
    clear_error();
    int rc = check_rows(rows, hidden, eps);
    if (rc != KOEMI_OK) return rc;
    if (rows == 0 || hidden == 0) return KOEMI_OK;
    RowArgs args{x, nullptr, residual, weight, keep, y, nullptr, rows, hidden, eps};
    return dispatch_rows<kPlain>(args, dtype, out_dtype, as_stream(stream));
}

extern "C" size_t koemi_core_rmsnorm_silu_backward_workspace(int64_t rows, int64_t hidden) {
    if (rows <= 0 || hidden <= 0) return 0;
    return static_cast<size_t>(backward_blocks(rows)) * static_cast<size_t>(hidden) * sizeof(float);
}

extern "C" int koemi_core_rmsnorm_silu_backward(const void *grad_y, const void *x,
                                                const void *weight, const float *inv_rms,
                                                void *grad_x, float *grad_weight, int64_t rows,
                                                int64_t hidden, void *workspace,
                                                size_t workspace_bytes, int dtype, void *stream) {
    clear_error();
    if (rows < 0 || hidden < 0) return fail(KOEMI_ERR_INVALID, "rows and hidden must be non-negative");
    if (rows == 0 || hidden == 0) {
        if (hidden > 0 && grad_weight != nullptr) {
            KOEMI_CUDA_TRY(cudaMemsetAsync(grad_weight, 0, hidden * sizeof(float), as_stream(stream)));
        }
        return KOEMI_OK;
    }
    if (workspace_bytes < koemi_core_rmsnorm_silu_backward_workspace(rows, hidden)) {
        return fail(KOEMI_ERR_WORKSPACE, "RMSNorm-SiLU backward needs %zu workspace bytes",
                    koemi_core_rmsnorm_silu_backward_workspace(rows, hidden));
    }
    float *partials = static_cast<float *>(workspace);
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: return rmsnorm_silu_backward_typed<float>(grad_y, x, weight, inv_rms, grad_x, grad_weight, rows, hidden, partials, s);
        case KOEMI_F16: return rmsnorm_silu_backward_typed<__half>(grad_y, x, weight, inv_rms, grad_x, grad_weight, rows, hidden, partials, s);
        case KOEMI_BF16: return rmsnorm_silu_backward_typed<__nv_bfloat16>(grad_y, x, weight, inv_rms, grad_x, grad_weight, rows, hidden, partials, s);
        default: return fail(KOEMI_ERR_INVALID, "unsupported RMSNorm-SiLU dtype %d", dtype);
    }
}
