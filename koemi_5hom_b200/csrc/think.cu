// Think front: causal surprise with a fused online log-sum-exp, and salient
// admission with ring compaction.
//
// Surprise: a CTA owns 32 prior rows and one slice of the content vocabulary.
// It walks the slice in tiles of 64 vocab rows, forms the [32 x 64] logit tile
// from shared-memory tiles of prior and head (fp32 FMA), and folds each tile
// into per-row running (max, sum of exp) plus the target logit, so the
// [rows, C] logits never exist in memory (the reference materialises them in
// fp32 with at::mm, think/surprise_kernel.cu:195-215, then reduces each row,
// :85-134). A finishing kernel merges the per-slice partials of every row in
// slice order and writes s = 1 - exp(-NLL / ln C), 0 on invalid rows.
// 16-bit inputs take the tcgen05 path of umma.cu when the shape allows it.
#include <cmath>

#include "vec.cuh"

namespace koemi {

// Shared with surprise_umma.cu: merge of per-slice partial statistics.
int surprise_finish(const float *partials, int64_t slices, const int64_t *targets, const uint8_t *valid,
                    void *out, float *nll_out, int64_t rows, int64_t content_vocab, int out_dtype,
                    cudaStream_t stream);
int surprise_umma_forward(const void *prior, const void *weight, const void *bias, const int64_t *targets,
                          int64_t rows, int64_t width, int64_t content_vocab, int dtype, float *partials,
                          int64_t slices, cudaStream_t stream, bool *handled);
int64_t surprise_umma_slices(int64_t rows, int64_t width, int64_t content_vocab, int dtype);
int surprise_grad_umma(const void *prior, const void *weight, const void *bias, const int64_t *targets,
                       const float *row_lse, const float *row_scale, float *dlogits, int64_t rows, int64_t width,
                       int64_t content_vocab, int dtype, cudaStream_t stream, bool *handled);

namespace {

constexpr int kRowsTile = 32;
constexpr int kVocabTile = 64;
constexpr int kKTile = 32;
constexpr int kThreads = 256;

// partials layout: [slices][rows][3] = (max, sum_exp, target_logit or -inf)
template <typename T>
__global__ __launch_bounds__(kThreads) void surprise_partial_kernel(
    const T *__restrict__ prior, const T *__restrict__ weight, const T *__restrict__ bias,
    const int64_t *__restrict__ targets, float *__restrict__ partials, int64_t rows, int64_t width,
    int64_t vocab, int64_t slice_size) {
    __shared__ float a_tile[kKTile][kRowsTile + 1];
    __shared__ float b_tile[kKTile][kVocabTile + 1];
    __shared__ float logits[kRowsTile][kVocabTile + 1];
    const int tid = threadIdx.x;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRowsTile;
    const int64_t v_begin = static_cast<int64_t>(blockIdx.y) * slice_size;
    const int64_t v_end = min(vocab, v_begin + slice_size);
    // thread -> 2 rows x 4 vocab columns of the 32 x 64 tile
    const int tr = tid / 16;  // 0..15
    const int tc = tid % 16;  // 0..15
    // running stats for the rows owned by the warp-reduction step: thread t<32 owns row t
    float run_max = -INFINITY, run_sum = 0.0f, target_logit = -INFINITY;
    int64_t my_target = -1;
    if (tid < kRowsTile && row0 + tid < rows) my_target = targets[row0 + tid];

    for (int64_t v0 = v_begin; v0 < v_end; v0 += kVocabTile) {
        float acc[2][4] = {};
        for (int64_t k0 = 0; k0 < width; k0 += kKTile) {
            for (int i = tid; i < kRowsTile * kKTile; i += kThreads) {
                const int r = i / kKTile, k = i % kKTile;
                const int64_t gr = row0 + r, gk = k0 + k;
                a_tile[k][r] = (gr < rows && gk < width) ? to_acc(prior[gr * width + gk]) : 0.0f;
            }
            for (int i = tid; i < kVocabTile * kKTile; i += kThreads) {
                const int c = i / kKTile, k = i % kKTile;
                const int64_t gc = v0 + c, gk = k0 + k;
                b_tile[k][c] = (gc < v_end && gk < width) ? to_acc(weight[gc * width + gk]) : 0.0f;
            }
            __syncthreads();
#pragma unroll 8
            for (int k = 0; k < kKTile; ++k) {
                const float a0 = a_tile[k][tr * 2], a1 = a_tile[k][tr * 2 + 1];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float b = b_tile[k][tc * 4 + j];
                    acc[0][j] = fmaf(a0, b, acc[0][j]);
                    acc[1][j] = fmaf(a1, b, acc[1][j]);
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t gc = v0 + tc * 4 + j;
                logits[tr * 2 + i][tc * 4 + j] = gc < v_end ? acc[i][j] + to_acc(bias[gc]) : -INFINITY;
            }
        }
        __syncthreads();
        if (tid < kRowsTile) {
            float m = run_max;
            for (int c = 0; c < kVocabTile; ++c) m = fmaxf(m, logits[tid][c]);
            float s = m == -INFINITY ? 0.0f : run_sum * expf(run_max - m);
            if (m != -INFINITY) {
                for (int c = 0; c < kVocabTile; ++c) s += expf(logits[tid][c] - m);
            }
            run_max = m;
            run_sum = s;
            if (my_target >= v0 && my_target < v0 + kVocabTile && my_target < v_end) {
                target_logit = logits[tid][my_target - v0];
            }
        }
        __syncthreads();
    }
    if (tid < kRowsTile && row0 + tid < rows) {
        float *p = partials + (static_cast<int64_t>(blockIdx.y) * rows + row0 + tid) * 3;
        p[0] = run_max;
        p[1] = run_sum;
        p[2] = target_logit;
    }
}

// One warp per row: lanes stride over the vocabulary-slice partials, then
// the (max, sum) pairs and the target logit are combined across the warp.
template <typename TO>
__global__ void surprise_finish_kernel(const float *__restrict__ partials, int64_t slices,
                                       const int64_t *__restrict__ targets, const uint8_t *__restrict__ valid,
                                       TO *__restrict__ out, float *__restrict__ nll_out, int64_t rows,
                                       float log_vocab) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    float m = -INFINITY, total = 0.0f, target = -INFINITY;
    for (int64_t s = lane; s < slices; s += 32) {
        const float *p = partials + (s * rows + row) * 3;
        const float pm = p[0];
        if (pm != -INFINITY) {
            const float nm = fmaxf(m, pm);
            total = total * expf(m - nm) + p[1] * expf(pm - nm);
            m = nm;
        }
        target = fmaxf(target, p[2]);
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, offset);
        const float ot = __shfl_xor_sync(0xffffffffu, total, offset);
        target = fmaxf(target, __shfl_xor_sync(0xffffffffu, target, offset));
        const float nm = fmaxf(m, om);
        if (nm != -INFINITY) {
            total = (m == -INFINITY ? 0.0f : total * expf(m - nm)) + (om == -INFINITY ? 0.0f : ot * expf(om - nm));
        }
        m = nm;
    }
    if (lane == 0) {
        const bool ok = valid == nullptr || valid[row] != 0;
        const float nll = logf(total) + m - target;
        out[row] = from_acc<TO>(ok ? 1.0f - expf(-nll / log_vocab) : 0.0f);
        if (nll_out != nullptr) nll_out[row] = ok ? nll : 0.0f;
    }
}

// Surprise of the rows of a merged head pass, whose log-sum-exp partials were
// folded without a target (the target was not known yet): one warp per row
// computes the target logit prior . W[token] + b[token] in fp32 (16-byte
// loads of the bf16/f16 prior row and head row), merges the row's (max, sum)
// partials over the slices, and writes s = 1 - exp(-NLL / ln C); 0 where the
// row's token is invalid. Row r belongs to stream r % batch (rows are
// block-major: [block][stream]).
template <typename T>
__global__ void surprise_from_partials_kernel(const T *__restrict__ prior, const T *__restrict__ weight,
                                              const T *__restrict__ bias, const int64_t *__restrict__ tokens,
                                              const uint8_t *__restrict__ valid, const float *__restrict__ partials,
                                              int64_t slices, int64_t rows, int64_t batch, int64_t width,
                                              float log_vocab, float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t stream = row % batch;
    const bool ok = valid == nullptr || valid[stream] != 0;
    if (!ok) {
        if (lane == 0) out[row] = 0.0f;
        return;
    }
    const int64_t token = tokens[stream];
    constexpr int W = Pack<T>::kWidth;
    const T *p = prior + row * width;
    const T *w = weight + token * width;
    float dot = 0.0f;
    for (int64_t c = static_cast<int64_t>(lane) * W; c < width; c += 32 * W) {
        float a[8], b[8];
        unpack(load_cached(p + c), a, T());
        unpack(load_cached(w + c), b, T());
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(a[e], b[e], dot);
    }
    dot = warp_sum(dot);
    const float target = dot + to_acc(bias[token]);
    float m = -INFINITY, total = 0.0f;
    for (int64_t s = lane; s < slices; s += 32) {
        const float *q = partials + (s * rows + row) * 3;
        const float pm = q[0];
        if (pm != -INFINITY) {
            const float nm = fmaxf(m, pm);
            total = total * expf(m - nm) + q[1] * expf(pm - nm);
            m = nm;
        }
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, offset);
        const float ot = __shfl_xor_sync(0xffffffffu, total, offset);
        const float nm = fmaxf(m, om);
        if (nm != -INFINITY) {
            total = (m == -INFINITY ? 0.0f : total * expf(m - nm)) + (om == -INFINITY ? 0.0f : ot * expf(om - nm));
        }
        m = nm;
    }
    if (lane == 0) {
        const float nll = logf(total) + m - target;
        out[row] = 1.0f - expf(-nll / log_vocab);
    }
}

// Backward, per row: the target logit prior . W[t] + b[t] (fp32), the
// row's log-sum-exp lse = NLL + target logit (NLL saved by the forward) and
// dL/dNLL = grad * exp(-NLL / ln C) / ln C (zero on invalid rows), one warp
// per row.
template <typename T>
__global__ void surprise_grad_rows_kernel(const T *__restrict__ prior, const T *__restrict__ weight,
                                          const T *__restrict__ bias, const int64_t *__restrict__ targets,
                                          const uint8_t *__restrict__ valid, const T *__restrict__ grad,
                                          const float *__restrict__ nll, float *__restrict__ row_lse,
                                          float *__restrict__ row_scale, int64_t rows, int64_t width,
                                          float log_vocab) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const bool ok = valid == nullptr || valid[row] != 0;
    if (!ok) {
        if (lane == 0) {
            row_lse[row] = 0.0f;
            row_scale[row] = 0.0f;
        }
        return;
    }
    const int64_t t = targets[row];
    const T *p = prior + row * width;
    const T *w = weight + t * width;
    float dot = 0.0f;
    for (int64_t c = lane; c < width; c += 32) dot = fmaf(to_acc(p[c]), to_acc(w[c]), dot);
    dot = warp_sum(dot);
    if (lane == 0) {
        const float n = nll[row];
        row_lse[row] = n + dot + to_acc(bias[t]);
        row_scale[row] = to_acc(grad[row]) * expf(-n / log_vocab) / log_vocab;
    }
}

// Backward on FMA tiles (fp32 inputs and shapes TMA cannot take): a CTA
// forms a [32 x 64] logit tile as the forward kernel does and stores
// dlogits = scale * (exp(l - lse) - onehot(target)) for it.
template <typename T>
__global__ __launch_bounds__(kThreads) void surprise_grad_kernel(
    const T *__restrict__ prior, const T *__restrict__ weight, const T *__restrict__ bias,
    const int64_t *__restrict__ targets, const float *__restrict__ row_lse, const float *__restrict__ row_scale,
    float *__restrict__ dlogits, int64_t rows, int64_t width, int64_t vocab) {
    __shared__ float a_tile[kKTile][kRowsTile + 1];
    __shared__ float b_tile[kKTile][kVocabTile + 1];
    const int tid = threadIdx.x;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRowsTile;
    const int64_t v0 = static_cast<int64_t>(blockIdx.y) * kVocabTile;
    const int tr = tid / 16;
    const int tc = tid % 16;
    float acc[2][4] = {};
    for (int64_t k0 = 0; k0 < width; k0 += kKTile) {
        for (int i = tid; i < kRowsTile * kKTile; i += kThreads) {
            const int r = i / kKTile, k = i % kKTile;
            const int64_t gr = row0 + r, gk = k0 + k;
            a_tile[k][r] = (gr < rows && gk < width) ? to_acc(prior[gr * width + gk]) : 0.0f;
        }
        for (int i = tid; i < kVocabTile * kKTile; i += kThreads) {
            const int c = i / kKTile, k = i % kKTile;
            const int64_t gc = v0 + c, gk = k0 + k;
            b_tile[k][c] = (gc < vocab && gk < width) ? to_acc(weight[gc * width + gk]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kKTile; ++k) {
            const float a0 = a_tile[k][tr * 2], a1 = a_tile[k][tr * 2 + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float b = b_tile[k][tc * 4 + j];
                acc[0][j] = fmaf(a0, b, acc[0][j]);
                acc[1][j] = fmaf(a1, b, acc[1][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t r = row0 + tr * 2 + i;
        if (r >= rows) continue;
        const float lse = row_lse[r], scale = row_scale[r];
        const int64_t t = targets[r];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t c = v0 + tc * 4 + j;
            if (c < vocab) {
                const float l = acc[i][j] + to_acc(bias[c]);
                dlogits[r * vocab + c] = scale * (expf(l - lse) - (c == t ? 1.0f : 0.0f));
            }
        }
    }
}

int64_t simt_slices(int64_t rows, int64_t vocab) {
    // enough CTAs to cover the SMs several times, each slice >= 4 vocab tiles
    const int64_t row_tiles = ceil_div(rows, kRowsTile);
    const int64_t want = ceil_div(static_cast<int64_t>(sm_count()) * 4, row_tiles);
    const int64_t max_slices = ceil_div(vocab, kVocabTile * 4);
    int64_t s = want < max_slices ? want : max_slices;
    return s < 1 ? 1 : s;
}

// Row copy / fill of the admission kernel: one warp per row, 16-byte
// packets when the row allows them.
__device__ __forceinline__ void copy_row_f32(float *dst, const float *src, int64_t width, int lane) {
    if (width % 4 == 0 && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
        for (int64_t c = lane; c < width / 4; c += 32) {
            reinterpret_cast<float4 *>(dst)[c] = __ldg(reinterpret_cast<const float4 *>(src) + c);
        }
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = src[c];
    }
}

__device__ __forceinline__ void zero_row_f32(float *dst, int64_t width, int lane) {
    if (width % 4 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        for (int64_t c = lane; c < width / 4; c += 32) reinterpret_cast<float4 *>(dst)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = 0.0f;
    }
}

// --------------------------------------------------------- salient admission
// One CTA per batch row. Admission is valid && surprise > threshold
// (network.py:349). When carried + length fits the capacity the ring is the
// plain concatenation (salient_tail's short path, memory.py:444-445);
// otherwise the latest `capacity` admitted entries are kept in temporal order,
// packed at the end of the ring behind zeroed invalid slots.
__global__ void salient_admission_kernel(const float *__restrict__ carried_keys,
                                         const float *__restrict__ carried_values,
                                         const uint8_t *__restrict__ carried_valid,
                                         const float *__restrict__ keys, const float *__restrict__ values,
                                         const float *__restrict__ surprise, const uint8_t *__restrict__ valid,
                                         float threshold, float *__restrict__ out_keys,
                                         float *__restrict__ out_values, uint8_t *__restrict__ out_valid,
                                         uint8_t *__restrict__ admission_out, int64_t carried, int64_t length,
                                         int64_t width, int64_t capacity) {
    extern __shared__ int32_t rank[];  // [carried + length] inclusive prefix of flags
    __shared__ int32_t warp_totals[32];
    __shared__ int32_t running;
    const int64_t b = blockIdx.x;
    const int64_t total = carried + length;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    auto flag_of = [&](int64_t i) -> int {
        if (i < carried) return carried_valid[b * carried + i] != 0;
        const int64_t t = i - carried;
        return (valid == nullptr || valid[b * length + t] != 0) && surprise[b * length + t] > threshold;
    };
    if (threadIdx.x == 0) running = 0;
    __syncthreads();
    for (int64_t base = 0; base < total; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const int f = i < total ? flag_of(i) : 0;
        if (i < total && i >= carried && admission_out != nullptr) admission_out[b * length + (i - carried)] = f;
        const unsigned ballot = __ballot_sync(0xffffffffu, f);
        const int in_warp = __popc(ballot & ((2u << lane) - 1u));
        if (lane == 31) warp_totals[warp] = __popc(ballot);
        __syncthreads();
        int before = running;
        for (int w = 0; w < warp; ++w) before += warp_totals[w];
        if (i < total) rank[i] = before + in_warp;
        __syncthreads();
        if (threadIdx.x == 0) {
            int sum = 0;
            for (int w = 0; w < warps; ++w) sum += warp_totals[w];
            running += sum;
        }
        __syncthreads();
    }
    const int32_t admitted = running;
    if (total <= capacity) {
        // plain concatenation, entries kept as they are
        for (int64_t i = warp; i < total; i += warps) {
            const float *ks = i < carried ? carried_keys + (b * carried + i) * width : keys + (b * length + i - carried) * width;
            const float *vs = i < carried ? carried_values + (b * carried + i) * width : values + (b * length + i - carried) * width;
            copy_row_f32(out_keys + (b * total + i) * width, ks, width, lane);
            copy_row_f32(out_values + (b * total + i) * width, vs, width, lane);
            if (lane == 0) out_valid[b * total + i] = flag_of(i);
        }
        return;
    }
    const int32_t kept = admitted < capacity ? admitted : static_cast<int32_t>(capacity);
    const int32_t skip = admitted - kept;
    const int64_t lead = capacity - kept;
    // leading empty slots
    for (int64_t slot = warp; slot < lead; slot += warps) {
        zero_row_f32(out_keys + (b * capacity + slot) * width, width, lane);
        zero_row_f32(out_values + (b * capacity + slot) * width, width, lane);
        if (lane == 0) out_valid[b * capacity + slot] = 0;
    }
    for (int64_t i = warp; i < total; i += warps) {
        const int32_t r = rank[i];  // inclusive rank
        const bool f = (i == 0 ? r : r - rank[i - 1]) != 0;
        if (!f || r - 1 < skip) continue;
        const int64_t slot = lead + (r - 1 - skip);
        const float *ks = i < carried ? carried_keys + (b * carried + i) * width : keys + (b * length + i - carried) * width;
        const float *vs = i < carried ? carried_values + (b * carried + i) * width : values + (b * length + i - carried) * width;
        copy_row_f32(out_keys + (b * capacity + slot) * width, ks, width, lane);
        copy_row_f32(out_values + (b * capacity + slot) * width, vs, width, lane);
        if (lane == 0) out_valid[b * capacity + slot] = 1;
    }
}

}  // namespace

int surprise_finish(const float *partials, int64_t slices, const int64_t *targets, const uint8_t *valid,
                    void *out, float *nll_out, int64_t rows, int64_t content_vocab, int out_dtype,
                    cudaStream_t stream) {
    const float log_vocab = std::log(static_cast<float>(content_vocab));
    const unsigned blocks = static_cast<unsigned>(ceil_div(rows, 8));
    switch (out_dtype) {
        case KOEMI_F32: KOEMI_CUDA_TRY(launch_pdl(surprise_finish_kernel<float>, dim3(blocks), dim3(256), 0, stream, dim3(1, 1, 1), partials, slices, targets, valid, static_cast<float *>(out), nll_out, rows, log_vocab)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(surprise_finish_kernel<__half>, dim3(blocks), dim3(256), 0, stream, dim3(1, 1, 1), partials, slices, targets, valid, static_cast<__half *>(out), nll_out, rows, log_vocab)); break;
        case KOEMI_BF16: KOEMI_CUDA_TRY(launch_pdl(surprise_finish_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream, dim3(1, 1, 1), partials, slices, targets, valid, static_cast<__nv_bfloat16 *>(out), nll_out, rows, log_vocab)); break;
        default: return fail(KOEMI_ERR_INVALID, "unsupported surprise output dtype %d", out_dtype);
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

}  // namespace koemi

using namespace koemi;

extern "C" size_t koemi_think_surprise_workspace(int64_t rows, int64_t width, int64_t content_vocab,
                                                 int dtype) {
    if (rows <= 0 || content_vocab <= 0) return 256;
    int64_t slices = simt_slices(rows, content_vocab);
    const int64_t umma = surprise_umma_slices(rows, width, content_vocab, dtype);
    if (umma > slices) slices = umma;
    return static_cast<size_t>(slices) * rows * 3 * sizeof(float);
}

extern "C" int koemi_think_causal_surprise_forward(const void *prior, const void *weight,
                                                   const void *bias, const int64_t *target_ids,
                                                   const uint8_t *valid, void *out, float *nll_out,
                                                   int64_t rows, int64_t width,
                                                   int64_t content_vocab, int dtype, int out_dtype,
                                                   void *workspace, size_t workspace_bytes,
                                                   void *stream) {
    clear_error();
    if (rows < 0 || width < 1 || content_vocab < 2) return fail(KOEMI_ERR_INVALID, "need rows >= 0, width >= 1, content_vocab >= 2");
    if (rows == 0) return KOEMI_OK;
    const size_t need = koemi_think_surprise_workspace(rows, width, content_vocab, dtype);
    if (workspace_bytes < need) return fail(KOEMI_ERR_WORKSPACE, "surprise needs %zu workspace bytes", need);
    float *partials = static_cast<float *>(workspace);
    cudaStream_t s = as_stream(stream);
    bool handled = false;
    int64_t slices = 0;
    if (dtype == KOEMI_BF16 || dtype == KOEMI_F16) {
        slices = surprise_umma_slices(rows, width, content_vocab, dtype);
        if (slices > 0) {
            int rc = surprise_umma_forward(prior, weight, bias, target_ids, rows, width, content_vocab, dtype, partials, slices, s, &handled);
            if (rc != KOEMI_OK) return rc;
        }
    }
    if (!handled) {
        slices = simt_slices(rows, content_vocab);
        const int64_t slice_size = ceil_div(ceil_div(content_vocab, slices), kVocabTile) * kVocabTile;
        slices = ceil_div(content_vocab, slice_size);
        const dim3 grid(static_cast<unsigned>(ceil_div(rows, kRowsTile)), static_cast<unsigned>(slices));
        switch (dtype) {
            case KOEMI_F32: surprise_partial_kernel<float><<<grid, kThreads, 0, s>>>(static_cast<const float *>(prior), static_cast<const float *>(weight), static_cast<const float *>(bias), target_ids, partials, rows, width, content_vocab, slice_size); break;
            case KOEMI_F16: surprise_partial_kernel<__half><<<grid, kThreads, 0, s>>>(static_cast<const __half *>(prior), static_cast<const __half *>(weight), static_cast<const __half *>(bias), target_ids, partials, rows, width, content_vocab, slice_size); break;
            case KOEMI_BF16: surprise_partial_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16 *>(prior), static_cast<const __nv_bfloat16 *>(weight), static_cast<const __nv_bfloat16 *>(bias), target_ids, partials, rows, width, content_vocab, slice_size); break;
            default: return fail(KOEMI_ERR_INVALID, "surprise supports f32, f16 and bf16");
        }
        KOEMI_LAUNCH_CHECK();
    }
    return surprise_finish(partials, slices, target_ids, valid, out, nll_out, rows, content_vocab, out_dtype, s);
}

extern "C" int koemi_think_salient_admission(const float *carried_keys, const float *carried_values,
                                             const uint8_t *carried_valid, const float *keys,
                                             const float *values, const float *surprise,
                                             const uint8_t *valid, float threshold,
                                             float *out_keys, float *out_values, uint8_t *out_valid,
                                             uint8_t *admission_out, int64_t batch, int64_t carried,
                                             int64_t length, int64_t width, int64_t capacity,
                                             void *stream) {
    clear_error();
    if (batch < 0 || carried < 0 || length < 0 || width < 0 || capacity < 1) return fail(KOEMI_ERR_INVALID, "bad admission sizes");
    if (batch == 0) return KOEMI_OK;
    const int64_t total = carried + length;
    const size_t smem = static_cast<size_t>(total > 0 ? total : 1) * sizeof(int32_t);
    if (smem > 200 * 1024) return fail(KOEMI_ERR_UNSUPPORTED, "carried + length too long for one admission pass");
    if (smem > 48 * 1024) {
        KOEMI_CUDA_TRY(cudaFuncSetAttribute(salient_admission_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    }
    salient_admission_kernel<<<static_cast<unsigned>(batch), 512, smem, as_stream(stream)>>>(
        carried_keys, carried_values, carried_valid, keys, values, surprise, valid, threshold, out_keys,
        out_values, out_valid, admission_out, carried, length, width, capacity);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_think_surprise_from_partials(const void *prior, const void *head_weight, const void *head_bias,
                                                  const int64_t *token_ids, const uint8_t *valid,
                                                  const float *partials, int64_t slices, int64_t rows, int64_t batch,
                                                  int64_t width, int64_t vocab, int64_t pad_id, int dtype,
                                                  float *surprise, void *stream) {
    clear_error();
    if (rows < 0 || batch < 1 || width < 1 || vocab < 2 || slices < 1) return fail(KOEMI_ERR_INVALID, "bad surprise sizes");
    if (rows == 0) return KOEMI_OK;
    if (rows % batch != 0) return fail(KOEMI_ERR_INVALID, "rows must be a whole number of batches");
    if (width % 8 != 0 || !aligned(prior, 16) || !aligned(head_weight, 16)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "width must be a multiple of 8 with 16-byte aligned prior and head");
    }
    if (head_bias == nullptr || token_ids == nullptr || partials == nullptr || surprise == nullptr) {
        return fail(KOEMI_ERR_INVALID, "head_bias, token_ids, partials and surprise must be non-NULL");
    }
    // the content vocabulary is the head without its PAD column
    const int64_t content = pad_id >= 0 && pad_id < vocab ? vocab - 1 : vocab;
    const float log_vocab = std::log(static_cast<float>(content));
    const unsigned blocks = static_cast<unsigned>(ceil_div(rows, 8));
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_BF16: KOEMI_CUDA_TRY(launch_pdl(surprise_from_partials_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), static_cast<const __nv_bfloat16 *>(prior), static_cast<const __nv_bfloat16 *>(head_weight), static_cast<const __nv_bfloat16 *>(head_bias), token_ids, valid, partials, slices, rows, batch, width, log_vocab, surprise)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(surprise_from_partials_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), static_cast<const __half *>(prior), static_cast<const __half *>(head_weight), static_cast<const __half *>(head_bias), token_ids, valid, partials, slices, rows, batch, width, log_vocab, surprise)); break;
        default: return fail(KOEMI_ERR_INVALID, "the head-pass surprise takes bf16 or f16 rows");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" size_t koemi_think_surprise_backward_workspace(int64_t rows) {
    return rows <= 0 ? 256 : static_cast<size_t>(2 * rows) * sizeof(float) + 256;
}

extern "C" int koemi_think_causal_surprise_backward(const void *prior, const void *weight, const void *bias,
                                                    const int64_t *target_ids, const uint8_t *valid,
                                                    const void *grad_surprise, const float *nll, float *dlogits,
                                                    int64_t rows, int64_t width, int64_t content_vocab, int dtype,
                                                    void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    if (rows < 0 || width < 1 || content_vocab < 2) return fail(KOEMI_ERR_INVALID, "need rows >= 0, width >= 1, content_vocab >= 2");
    if (rows == 0) return KOEMI_OK;
    if (workspace_bytes < koemi_think_surprise_backward_workspace(rows)) {
        return fail(KOEMI_ERR_WORKSPACE, "surprise backward needs %zu workspace bytes", koemi_think_surprise_backward_workspace(rows));
    }
    if (prior == nullptr || weight == nullptr || bias == nullptr || target_ids == nullptr || grad_surprise == nullptr ||
        nll == nullptr || dlogits == nullptr) {
        return fail(KOEMI_ERR_INVALID, "surprise backward pointers must be non-NULL (valid may be NULL)");
    }
    float *row_lse = static_cast<float *>(workspace);
    float *row_scale = row_lse + rows;
    const float log_vocab = std::log(static_cast<float>(content_vocab));
    cudaStream_t s = as_stream(stream);
    const unsigned row_blocks = static_cast<unsigned>(ceil_div(rows, 8));
    switch (dtype) {
        case KOEMI_F32: surprise_grad_rows_kernel<float><<<row_blocks, 256, 0, s>>>(static_cast<const float *>(prior), static_cast<const float *>(weight), static_cast<const float *>(bias), target_ids, valid, static_cast<const float *>(grad_surprise), nll, row_lse, row_scale, rows, width, log_vocab); break;
        case KOEMI_F16: surprise_grad_rows_kernel<__half><<<row_blocks, 256, 0, s>>>(static_cast<const __half *>(prior), static_cast<const __half *>(weight), static_cast<const __half *>(bias), target_ids, valid, static_cast<const __half *>(grad_surprise), nll, row_lse, row_scale, rows, width, log_vocab); break;
        case KOEMI_BF16: surprise_grad_rows_kernel<__nv_bfloat16><<<row_blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(prior), static_cast<const __nv_bfloat16 *>(weight), static_cast<const __nv_bfloat16 *>(bias), target_ids, valid, static_cast<const __nv_bfloat16 *>(grad_surprise), nll, row_lse, row_scale, rows, width, log_vocab); break;
        default: return fail(KOEMI_ERR_INVALID, "surprise backward supports f32, f16 and bf16");
    }
    KOEMI_LAUNCH_CHECK();
    bool handled = false;
    int rc = surprise_grad_umma(prior, weight, bias, target_ids, row_lse, row_scale, dlogits, rows, width, content_vocab,
                                dtype, s, &handled);
    if (rc != KOEMI_OK || handled) return rc;
    const dim3 grid(static_cast<unsigned>(ceil_div(rows, kRowsTile)), static_cast<unsigned>(ceil_div(content_vocab, kVocabTile)));
    switch (dtype) {
        case KOEMI_F32: surprise_grad_kernel<float><<<grid, kThreads, 0, s>>>(static_cast<const float *>(prior), static_cast<const float *>(weight), static_cast<const float *>(bias), target_ids, row_lse, row_scale, dlogits, rows, width, content_vocab); break;
        case KOEMI_F16: surprise_grad_kernel<__half><<<grid, kThreads, 0, s>>>(static_cast<const __half *>(prior), static_cast<const __half *>(weight), static_cast<const __half *>(bias), target_ids, row_lse, row_scale, dlogits, rows, width, content_vocab); break;
        default: surprise_grad_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16 *>(prior), static_cast<const __nv_bfloat16 *>(weight), static_cast<const __nv_bfloat16 *>(bias), target_ids, row_lse, row_scale, dlogits, rows, width, content_vocab); break;
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}
