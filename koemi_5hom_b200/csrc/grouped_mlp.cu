// MoE front: grouped gated expert MLP over sorted expert segments.
//
// Work is scheduled on the device from segment_offsets, with no host read of
// the counts (the reference syncs on segment_offsets[-1].item(),
// moe/__init__.py:293): a tiny kernel turns per-expert row counts into a
// prefix of row tiles, and every CTA of the GEMM kernels maps its blockIdx.x
// to (expert, row tile) by binary search in that prefix. Blocks past the last
// tile exit. Rows of a tile that belong to the next expert are computed but
// never stored.
//
// Two contractions per pair: hidden = silu(x Wg^T + bg) * (x Wv^T + bv),
// then y = hidden Wo^T + bo. BF16/F16 run on tcgen05 tensor cores
// (umma.cu); F32 (and any shape the tensor-core path rejects) runs
// the fp32 FMA tiles below. Reference: moe/moe_kernels.cu:147-199 (one CTA
// per pair re-reading that expert's full weights).
#include "common.cuh"

namespace koemi {

int grouped_mlp_umma(const void *sorted_context, const int64_t *segment_offsets, const void *gate_w,
                     const void *gate_b, const void *value_w, const void *value_b, const void *out_w,
                     const void *out_b, void *output, int64_t pairs, int64_t input_width,
                     int64_t hidden_width, int64_t expert_count, int dtype, void *workspace,
                     size_t workspace_bytes, cudaStream_t stream, bool *handled, const int32_t *tile_prefix_in,
                     bool zero_tail);
size_t grouped_mlp_umma_workspace(int64_t pairs, int64_t input_width, int64_t hidden_width,
                                  int64_t expert_count, int dtype);

// Shared by both paths: tile_prefix[e] = row tiles of experts < e (E + 1 entries).
__global__ void tile_prefix_kernel(const int64_t *__restrict__ offsets, int64_t experts, int64_t tile_rows,
                                   int32_t *__restrict__ prefix) {
    pdl_trigger();
    pdl_wait();
    // one warp: 32 experts per round, inclusive shuffle scan plus a carry
    const int lane = threadIdx.x & 31;
    if (blockIdx.x != 0 || threadIdx.x >= 32) return;
    int32_t carry = 0;
    for (int64_t base = 0; base < experts; base += 32) {
        const int64_t e = base + lane;
        int32_t tiles = 0;
        if (e < experts) tiles = static_cast<int32_t>((offsets[e + 1] - offsets[e] + tile_rows - 1) / tile_rows);
        int32_t inclusive = tiles;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t other = __shfl_up_sync(0xffffffffu, inclusive, o);
            if (lane >= o) inclusive += other;
        }
        if (e < experts) prefix[e] = carry + inclusive - tiles;
        carry += __shfl_sync(0xffffffffu, inclusive, 31);
    }
    if (lane == 0) prefix[experts] = carry;
}

__device__ __forceinline__ int64_t find_expert(const int32_t *prefix, int64_t experts, int64_t tile) {
    int64_t lo = 0, hi = experts;  // largest e with prefix[e] <= tile
    while (lo + 1 < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (prefix[mid] <= tile) lo = mid; else hi = mid;
    }
    return lo;
}

__global__ void zero_tail_rows_kernel(void *out, const int64_t *__restrict__ offsets, int64_t experts,
                                      int64_t pairs, int64_t row_bytes) {
    pdl_trigger();
    pdl_wait();
    const int64_t valid_rows = offsets[experts];
    char *base = static_cast<char *>(out);
    const int64_t begin = valid_rows * row_bytes;
    const int64_t end = pairs * row_bytes;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (((reinterpret_cast<uintptr_t>(base) | static_cast<uintptr_t>(row_bytes)) & 15) == 0) {
        // whole rows of 16-byte packets: begin and end are multiples of 16
        uint4 *packets = reinterpret_cast<uint4 *>(base + begin);
        const int64_t count = (end - begin) / 16;
        for (int64_t i = first; i < count; i += stride) packets[i] = make_uint4(0, 0, 0, 0);
        return;
    }
    for (int64_t i = begin + first; i < end; i += stride) base[i] = 0;
}

namespace {

constexpr int kBM = 32;
constexpr int kBN = 64;
constexpr int kBK = 32;
constexpr int kThreads = 256;

// out[r, n] for rows r of one expert tile.
// kGated: out = silu(A Wg^T + bg) * (A Wv^T + bv) (fp32 hidden);
// else:   out = A Wo^T + bo (cast to TO).
template <typename TA, typename TW, typename TO, bool kGated>
__global__ __launch_bounds__(kThreads) void grouped_gemm_simt_kernel(
    const TA *__restrict__ a, const int64_t *__restrict__ offsets, const int32_t *__restrict__ prefix,
    const TW *__restrict__ w0, const TW *__restrict__ b0, const TW *__restrict__ w1,
    const TW *__restrict__ b1, TO *__restrict__ out, int64_t experts, int64_t k_width, int64_t n_width) {
    __shared__ float as[kBK][kBM + 1];
    __shared__ float ws0[kBK][kBN + 1];
    __shared__ float ws1[kGated ? kBK : 1][kBN + 1];
    const int64_t tile = blockIdx.x;
    if (tile >= prefix[experts]) return;
    const int64_t e = find_expert(prefix, experts, tile);
    const int64_t seg_begin = offsets[e];
    const int64_t seg_end = offsets[e + 1];
    const int64_t row0 = seg_begin + (tile - prefix[e]) * kBM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.y) * kBN;
    const TW *w0e = w0 + e * n_width * k_width;
    const TW *w1e = kGated ? w1 + e * n_width * k_width : nullptr;
    const int tid = threadIdx.x;
    const int tr = tid / 16, tc = tid % 16;  // 2 rows x 4 cols per thread
    float acc0[2][4] = {}, acc1[2][4] = {};
    for (int64_t k0 = 0; k0 < k_width; k0 += kBK) {
        for (int i = tid; i < kBM * kBK; i += kThreads) {
            const int r = i / kBK, k = i % kBK;
            const int64_t gr = row0 + r, gk = k0 + k;
            as[k][r] = (gr < seg_end && gk < k_width) ? to_acc(a[gr * k_width + gk]) : 0.0f;
        }
        for (int i = tid; i < kBN * kBK; i += kThreads) {
            const int c = i / kBK, k = i % kBK;
            const int64_t gc = n0 + c, gk = k0 + k;
            const bool ok = gc < n_width && gk < k_width;
            ws0[k][c] = ok ? to_acc(w0e[gc * k_width + gk]) : 0.0f;
            if (kGated) ws1[k][c] = ok ? to_acc(w1e[gc * k_width + gk]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kBK; ++k) {
            const float a0 = as[k][tr * 2], a1 = as[k][tr * 2 + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float x0 = ws0[k][tc * 4 + j];
                acc0[0][j] = fmaf(a0, x0, acc0[0][j]);
                acc0[1][j] = fmaf(a1, x0, acc0[1][j]);
                if (kGated) {
                    const float x1 = ws1[k][tc * 4 + j];
                    acc1[0][j] = fmaf(a0, x1, acc1[0][j]);
                    acc1[1][j] = fmaf(a1, x1, acc1[1][j]);
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t gr = row0 + tr * 2 + i;
        if (gr >= seg_end) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gc = n0 + tc * 4 + j;
            if (gc >= n_width) continue;
            float v;
            if (kGated) {
                const float g = acc0[i][j] + to_acc(b0[e * n_width + gc]);
                const float u = acc1[i][j] + to_acc(b1[e * n_width + gc]);
                v = siluf_(g) * u;
            } else {
                v = acc0[i][j] + to_acc(b0[e * n_width + gc]);
            }
            out[gr * n_width + gc] = from_acc<TO>(v);
        }
    }
}

template <typename T>
int grouped_mlp_simt(const void *x, const int64_t *offsets, const void *gw, const void *gb, const void *vw,
                     const void *vb, const void *ow, const void *ob, void *output, int64_t pairs, int64_t d,
                     int64_t h, int64_t experts, char *ws, cudaStream_t stream) {
    int32_t *prefix = reinterpret_cast<int32_t *>(ws);
    float *hidden = reinterpret_cast<float *>(ws + (((experts + 1) * sizeof(int32_t) + 255) & ~size_t(255)));
    KOEMI_CUDA_TRY(launch_pdl(tile_prefix_kernel, dim3(1), dim3(32), 0, stream, dim3(1, 1, 1), offsets, experts, kBM, prefix));
    KOEMI_LAUNCH_CHECK();
    const unsigned max_tiles = static_cast<unsigned>(ceil_div(pairs, kBM) + experts);
    grouped_gemm_simt_kernel<T, T, float, true><<<dim3(max_tiles, static_cast<unsigned>(ceil_div(h, kBN))), kThreads, 0, stream>>>(
        static_cast<const T *>(x), offsets, prefix, static_cast<const T *>(gw), static_cast<const T *>(gb),
        static_cast<const T *>(vw), static_cast<const T *>(vb), hidden, experts, d, h);
    KOEMI_LAUNCH_CHECK();
    grouped_gemm_simt_kernel<float, T, T, false><<<dim3(max_tiles, static_cast<unsigned>(ceil_div(d, kBN))), kThreads, 0, stream>>>(
        hidden, offsets, prefix, static_cast<const T *>(ow), static_cast<const T *>(ob), nullptr, nullptr,
        static_cast<T *>(output), experts, h, d);
    KOEMI_LAUNCH_CHECK();
    KOEMI_CUDA_TRY(launch_pdl(zero_tail_rows_kernel, dim3(256), dim3(256), 0, stream, dim3(1, 1, 1), output, offsets, experts, pairs, d * sizeof(T)));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

size_t simt_workspace(int64_t pairs, int64_t h, int64_t experts) {
    return (((experts + 1) * sizeof(int32_t) + 255) & ~size_t(255)) + static_cast<size_t>(pairs) * h * sizeof(float);
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" size_t koemi_moe_grouped_mlp_workspace(int64_t pairs, int64_t input_width, int64_t hidden_width,
                                                  int64_t expert_count, int dtype) {
    if (pairs < 0 || input_width < 0 || hidden_width < 0 || expert_count < 1) return 256;
    size_t need = simt_workspace(pairs, hidden_width, expert_count);
    const size_t umma = grouped_mlp_umma_workspace(pairs, input_width, hidden_width, expert_count, dtype);
    return need > umma ? need : umma;
}

extern "C" int koemi_moe_grouped_expert_mlp(const void *sorted_context, const int64_t *sorted_experts,
                                            const int64_t *segment_offsets, const void *gate_weights,
                                            const void *gate_biases, const void *value_weights,
                                            const void *value_biases, const void *output_weights,
                                            const void *output_biases, void *output, int64_t pairs,
                                            int64_t input_width, int64_t hidden_width,
                                            int64_t expert_count, int dtype, void *workspace,
                                            size_t workspace_bytes, void *stream) {
    (void)sorted_experts;  // the expert of each row is implied by segment_offsets
    clear_error();
    if (pairs < 0 || input_width < 1 || hidden_width < 1 || expert_count < 1) {
        return fail(KOEMI_ERR_INVALID, "need pairs >= 0 and positive widths and expert_count");
    }
    if (pairs == 0) return KOEMI_OK;
    const size_t need = koemi_moe_grouped_mlp_workspace(pairs, input_width, hidden_width, expert_count, dtype);
    if (workspace_bytes < need) return fail(KOEMI_ERR_WORKSPACE, "grouped MLP needs %zu workspace bytes", need);
    cudaStream_t s = as_stream(stream);
    if (dtype == KOEMI_BF16 || dtype == KOEMI_F16) {
        bool handled = false;
        int rc = grouped_mlp_umma(sorted_context, segment_offsets, gate_weights, gate_biases, value_weights,
                                  value_biases, output_weights, output_biases, output, pairs, input_width,
                                  hidden_width, expert_count, dtype, workspace, workspace_bytes, s, &handled, nullptr,
                                  true);
        if (rc != KOEMI_OK || handled) return rc;
    }
    char *ws = static_cast<char *>(workspace);
    switch (dtype) {
        case KOEMI_F32: return grouped_mlp_simt<float>(sorted_context, segment_offsets, gate_weights, gate_biases, value_weights, value_biases, output_weights, output_biases, output, pairs, input_width, hidden_width, expert_count, ws, s);
        case KOEMI_F16: return grouped_mlp_simt<__half>(sorted_context, segment_offsets, gate_weights, gate_biases, value_weights, value_biases, output_weights, output_biases, output, pairs, input_width, hidden_width, expert_count, ws, s);
        case KOEMI_BF16: return grouped_mlp_simt<__nv_bfloat16>(sorted_context, segment_offsets, gate_weights, gate_biases, value_weights, value_biases, output_weights, output_biases, output, pairs, input_width, hidden_width, expert_count, ws, s);
        default: return fail(KOEMI_ERR_INVALID, "grouped MLP supports f32, f16 and bf16");
    }
}

extern "C" int koemi_moe_tile_prefix(const int64_t *segment_offsets, int64_t expert_count, int32_t *tile_prefix,
                                     void *stream) {
    clear_error();
    if (segment_offsets == nullptr || tile_prefix == nullptr || expert_count < 1) {
        return fail(KOEMI_ERR_INVALID, "tile prefix needs offsets, an output and expert_count >= 1");
    }
    KOEMI_CUDA_TRY(launch_pdl(tile_prefix_kernel, dim3(1), dim3(32), 0, as_stream(stream), dim3(1, 1, 1),
                              segment_offsets, expert_count, static_cast<int64_t>(128), tile_prefix));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_moe_grouped_expert_mlp_mapped(const void *sorted_context, const int32_t *tile_prefix,
                                                   const int64_t *segment_offsets, const void *gate_weights,
                                                   const void *gate_biases, const void *value_weights,
                                                   const void *value_biases, const void *output_weights,
                                                   const void *output_biases, void *output, int64_t pairs,
                                                   int64_t input_width, int64_t hidden_width, int64_t expert_count,
                                                   int dtype, void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return fail(KOEMI_ERR_INVALID, "the mapped expert MLP takes bf16 or f16 rows");
    if (pairs < 0 || input_width < 1 || hidden_width < 1 || expert_count < 1 || tile_prefix == nullptr) {
        return fail(KOEMI_ERR_INVALID, "need pairs >= 0, positive widths and expert_count, and a tile prefix");
    }
    if (pairs == 0) return KOEMI_OK;
    const size_t need = grouped_mlp_umma_workspace(pairs, input_width, hidden_width, expert_count, dtype);
    if (workspace_bytes < need) return fail(KOEMI_ERR_WORKSPACE, "mapped expert MLP needs %zu workspace bytes", need);
    bool handled = false;
    const int rc = grouped_mlp_umma(sorted_context, segment_offsets, gate_weights, gate_biases, value_weights,
                                    value_biases, output_weights, output_biases, output, pairs, input_width,
                                    hidden_width, expert_count, dtype, workspace, workspace_bytes, as_stream(stream),
                                    &handled, tile_prefix, false);
    if (rc != KOEMI_OK) return rc;
    if (!handled) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the mapped expert MLP needs widths that are multiples of 8 and 16-byte aligned operands");
    }
    return KOEMI_OK;
}

