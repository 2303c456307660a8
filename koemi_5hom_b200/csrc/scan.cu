// Dense front: affine recurrent scan h_t = a_t * h_{t-1} + b_t.
//
// Layout: retention/increment/states are [batch, length, features] row-major
// (features contiguous). One CTA owns 32 features of one batch row and walks
// the whole sequence in chunks of 64 positions. Each chunk is staged into
// shared memory by TMA (3D tensor map, box {32 features, 64 positions, 1})
// through a multi-stage mbarrier pipeline, so HBM streams while the previous
// chunks are being combined. Inside a chunk, warp w owns positions
// [8w, 8w + 8) and lane l owns feature l: every thread first composes its 8
// affine maps into one (A, B) pair, the 8 per-warp pairs are exchanged through
// shared memory to form each warp's carry-in from the running fp32 state, and
// the thread then replays its 8 steps from that carry to produce h_t, which is
// stored straight from registers (32 consecutive features per warp store).
// Reference behaviour: dense/affine_scan.cu:18-56 (sequential per lane) and
// model/scan.py:17-30 (log-step doubling); both compute the same recurrence.
#include "common.cuh"

namespace koemi {
namespace {

constexpr int kFeatureTile = 32;
constexpr int kWarps = 8;
constexpr int kStepsPerWarp = 8;
constexpr int kChunk = kWarps * kStepsPerWarp;
constexpr int kThreads = kWarps * 32;

template <typename T>
struct TensorMapType;
template <>
struct TensorMapType<__nv_bfloat16> {
    static constexpr CUtensorMapDataType value = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <>
struct TensorMapType<__half> {
    static constexpr CUtensorMapDataType value = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};
template <>
struct TensorMapType<float> {
    static constexpr CUtensorMapDataType value = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
};

template <typename T>
constexpr int stages_for() {
    return sizeof(T) == 2 ? 6 : 4;
}

template <typename T, bool kTma, bool kBroadcast>
__global__ __launch_bounds__(kThreads) void scan_forward_kernel(
    const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
    const T *__restrict__ retention, const T *__restrict__ increment, const T *__restrict__ initial,
    T *__restrict__ states, int64_t length, int64_t features, int *status) {
    using Acc = typename Accum<T>::type;
    constexpr int kStages = kTma ? stages_for<T>() : 1;
    constexpr int kTileElems = kChunk * kFeatureTile;

    extern __shared__ __align__(128) unsigned char smem_raw[];
    T *tile_a = reinterpret_cast<T *>(smem_raw);
    T *tile_b = tile_a + (kTma ? kStages * kTileElems : 0);
    Acc *xchg = reinterpret_cast<Acc *>(tile_b + (kTma ? kStages * kTileElems : 0));
    uint64_t *full = reinterpret_cast<uint64_t *>(xchg + 2 * kWarps * 2 * kFeatureTile);

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t f0 = static_cast<int64_t>(blockIdx.x) * kFeatureTile;
    const int64_t batch = blockIdx.y;
    const int64_t f = f0 + lane;
    const bool f_ok = f < features;
    const int64_t chunks = (length + kChunk - 1) / kChunk;
    const T *ret_row = retention + (kBroadcast ? batch * length : batch * length * features);
    const T *inc_row = increment + batch * length * features;
    T *out_row = states + batch * length * features;

    constexpr uint32_t kStageBytes = (kBroadcast ? 1u : 2u) * kTileElems * sizeof(T);
    auto issue = [&](int64_t chunk) {
        const int s = static_cast<int>(chunk % kStages);
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        const int32_t pos = static_cast<int32_t>(chunk * kChunk);
        if (!kBroadcast) {
            tma_load_3d(tile_a + s * kTileElems, &map_a, &full[s], static_cast<int32_t>(f0), pos,
                        static_cast<int32_t>(batch));
        }
        tma_load_3d(tile_b + s * kTileElems, &map_b, &full[s], static_cast<int32_t>(f0), pos,
                    static_cast<int32_t>(batch));
    };

    if constexpr (kTma) {
        if (threadIdx.x == 0) {
            for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
            fence_barrier_init();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            if (!kBroadcast) prefetch_tensor_map(&map_a);
            prefetch_tensor_map(&map_b);
            for (int64_t c = 0; c < chunks && c < kStages; ++c) issue(c);
        }
    }

    Acc carry = Acc(0);
    if (initial != nullptr && f_ok) carry = to_acc(initial[batch * features + f]);

    for (int64_t c = 0; c < chunks; ++c) {
        Acc a[kStepsPerWarp];
        Acc b[kStepsPerWarp];
        const int64_t base_t = c * kChunk + warp * kStepsPerWarp;
        bool timed_out = false;
        if constexpr (kTma) {
            const int s = static_cast<int>(c % kStages);
            const uint32_t parity = static_cast<uint32_t>((c / kStages) & 1);
            timed_out = !mbar_wait_bounded(&full[s], parity, status);
            const T *sa = tile_a + s * kTileElems + warp * kStepsPerWarp * kFeatureTile + lane;
            const T *sb = tile_b + s * kTileElems + warp * kStepsPerWarp * kFeatureTile + lane;
#pragma unroll
            for (int j = 0; j < kStepsPerWarp; ++j) {
                const int64_t t = base_t + j;
                if (kBroadcast) {
                    a[j] = t < length ? to_acc(ret_row[t]) : Acc(0);
                } else {
                    a[j] = to_acc(sa[j * kFeatureTile]);
                }
                b[j] = to_acc(sb[j * kFeatureTile]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < kStepsPerWarp; ++j) {
                const int64_t t = base_t + j;
                const bool ok = f_ok && t < length;
                if (kBroadcast) {
                    a[j] = t < length ? to_acc(ret_row[t]) : Acc(0);
                } else {
                    a[j] = ok ? to_acc(ret_row[t * features + f]) : Acc(0);
                }
                b[j] = ok ? to_acc(inc_row[t * features + f]) : Acc(0);
            }
        }

        // Compose this thread's 8 steps into h_out = A * h_in + B.
        Acc A = Acc(1), B = Acc(0);
#pragma unroll
        for (int j = 0; j < kStepsPerWarp; ++j) {
            A = a[j] * A;
            B = a[j] * B + b[j];
        }
        Acc *x = xchg + (c & 1) * (kWarps * 2 * kFeatureTile);
        x[(warp * 2 + 0) * kFeatureTile + lane] = A;
        x[(warp * 2 + 1) * kFeatureTile + lane] = B;
        if (__syncthreads_or(timed_out)) return;

        if constexpr (kTma) {
            if (threadIdx.x == 0 && c + kStages < chunks) issue(c + kStages);
        }

        // Carry-in for this warp, and the carry out of the whole chunk.
        Acc h = carry;
        for (int w = 0; w < warp; ++w) {
            h = x[(w * 2 + 0) * kFeatureTile + lane] * h + x[(w * 2 + 1) * kFeatureTile + lane];
        }
        Acc next = h;
        for (int w = warp; w < kWarps; ++w) {
            next = x[(w * 2 + 0) * kFeatureTile + lane] * next + x[(w * 2 + 1) * kFeatureTile + lane];
        }
#pragma unroll
        for (int j = 0; j < kStepsPerWarp; ++j) {
            h = a[j] * h + b[j];
            const int64_t t = base_t + j;
            if (f_ok && t < length) out_row[t * features + f] = from_acc<T>(h);
        }
        carry = next;
    }
}

// Short sequences (decode steps): one thread per (batch, feature) lane.
template <typename T, bool kBroadcast>
__global__ void scan_forward_short_kernel(const T *__restrict__ retention,
                                          const T *__restrict__ increment,
                                          const T *__restrict__ initial, T *__restrict__ states,
                                          int64_t batch, int64_t length, int64_t features) {
    using Acc = typename Accum<T>::type;
    const int64_t lane = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (lane >= batch * features) return;
    const int64_t b = lane / features;
    const int64_t f = lane - b * features;
    Acc h = initial != nullptr ? to_acc(initial[lane]) : Acc(0);
    for (int64_t t = 0; t < length; ++t) {
        const int64_t offset = (b * length + t) * features + f;
        const Acc a = to_acc(kBroadcast ? retention[b * length + t] : retention[offset]);
        h = a * h + to_acc(increment[offset]);
        states[offset] = from_acc<T>(h);
    }
}

// Reverse-time adjoint: adj_t = g_t + a_{t+1} adj_{t+1}; grad_b_t = adj_t,
// grad_a_t = adj_t * h_{t-1}, grad_h0 = a_0 adj_0 (dense/affine_scan.cu:59-106).
template <typename T, bool kBroadcast>
__global__ void scan_backward_kernel(const T *__restrict__ retention, const T *__restrict__ initial,
                                     const T *__restrict__ states, const T *__restrict__ grad_states,
                                     T *__restrict__ grad_retention, T *__restrict__ grad_increment,
                                     T *__restrict__ grad_initial, int64_t batch, int64_t length,
                                     int64_t features) {
    using Acc = typename Accum<T>::type;
    const int64_t lane = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (lane >= batch * features) return;
    const int64_t b = lane / features;
    const int64_t f = lane - b * features;
    Acc adj = Acc(0);
    for (int64_t t = length - 1; t >= 0; --t) {
        const int64_t offset = (b * length + t) * features + f;
        const Acc a = to_acc(kBroadcast ? retention[b * length + t] : retention[offset]);
        const Acc prev = t == 0 ? (initial != nullptr ? to_acc(initial[lane]) : Acc(0))
                                : to_acc(states[offset - features]);
        adj += to_acc(grad_states[offset]);
        grad_increment[offset] = from_acc<T>(adj);
        grad_retention[offset] = from_acc<T>(adj * prev);
        adj *= a;
    }
    if (grad_initial != nullptr) grad_initial[lane] = from_acc<T>(adj);
}

template <typename T>
size_t scan_smem_bytes(bool tma) {
    using Acc = typename Accum<T>::type;
    const int stages = tma ? stages_for<T>() : 0;
    return static_cast<size_t>(stages) * 2 * kChunk * kFeatureTile * sizeof(T) +
           2 * kWarps * 2 * kFeatureTile * sizeof(Acc) + 8 * sizeof(uint64_t);
}

template <typename T, bool kTma, bool kBroadcast>
int launch_chunked(const T *retention, const T *increment, const T *initial, T *states,
                   int64_t batch, int64_t length, int64_t features, cudaStream_t stream) {
    CUtensorMap map_a{}, map_b{};
    if constexpr (kTma) {
        const uint64_t es = sizeof(T);
        const uint64_t dims[3] = {static_cast<uint64_t>(features), static_cast<uint64_t>(length),
                                  static_cast<uint64_t>(batch)};
        const uint64_t strides[2] = {features * es, length * features * es};
        const uint32_t box[3] = {kFeatureTile, kChunk, 1};
        int rc;
        if (!kBroadcast) {
            rc = encode_tensor_map(&map_a, TensorMapType<T>::value, 3, retention, dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc != KOEMI_OK) return rc;
        }
        rc = encode_tensor_map(&map_b, TensorMapType<T>::value, 3, increment, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc != KOEMI_OK) return rc;
    }
    const size_t smem = scan_smem_bytes<T>(kTma);
    auto kernel = scan_forward_kernel<T, kTma, kBroadcast>;
    if (smem > 48 * 1024) {
        KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)));
    }
    const dim3 grid(static_cast<unsigned>(ceil_div(features, kFeatureTile)),
                    static_cast<unsigned>(batch));
    kernel<<<grid, kThreads, smem, stream>>>(map_a, map_b, retention, increment, initial, states,
                                             length, features, device_status_word());
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

template <typename T>
int scan_forward_typed(const void *retention, const void *increment, const void *initial,
                       void *states, int64_t batch, int64_t length, int64_t features,
                       bool broadcast, cudaStream_t stream) {
    const T *r = static_cast<const T *>(retention);
    const T *i = static_cast<const T *>(increment);
    const T *h0 = static_cast<const T *>(initial);
    T *out = static_cast<T *>(states);
    if (length <= 8 || batch > 65535) {
        const int64_t lanes = batch * features;
        const int threads = 256;
        const unsigned blocks = static_cast<unsigned>(ceil_div(lanes, threads));
        if (broadcast) {
            scan_forward_short_kernel<T, true><<<blocks, threads, 0, stream>>>(r, i, h0, out, batch,
                                                                                length, features);
        } else {
            scan_forward_short_kernel<T, false><<<blocks, threads, 0, stream>>>(r, i, h0, out, batch,
                                                                                 length, features);
        }
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    }
    bool tma = sizeof(T) != 8 && (features * sizeof(T)) % 16 == 0 && aligned(increment, 16) &&
               (broadcast || aligned(retention, 16)) && length < (int64_t(1) << 31) &&
               features < (int64_t(1) << 31);
    if constexpr (sizeof(T) == 8) tma = false;
    if constexpr (sizeof(T) != 8) {
        if (tma) {
            return broadcast ? launch_chunked<T, true, true>(r, i, h0, out, batch, length, features, stream)
                             : launch_chunked<T, true, false>(r, i, h0, out, batch, length, features, stream);
        }
    }
    return broadcast ? launch_chunked<T, false, true>(r, i, h0, out, batch, length, features, stream)
                     : launch_chunked<T, false, false>(r, i, h0, out, batch, length, features, stream);
}

template <typename T>
int scan_backward_typed(const void *retention, const void *initial, const void *states,
                        const void *grad_states, void *grad_retention, void *grad_increment,
                        void *grad_initial, int64_t batch, int64_t length, int64_t features,
                        bool broadcast, cudaStream_t stream) {
    const int64_t lanes = batch * features;
    const int threads = 128;
    const unsigned blocks = static_cast<unsigned>(ceil_div(lanes, threads));
    auto launch = [&](auto kernel) {
        kernel<<<blocks, threads, 0, stream>>>(
            static_cast<const T *>(retention), static_cast<const T *>(initial),
            static_cast<const T *>(states), static_cast<const T *>(grad_states),
            static_cast<T *>(grad_retention), static_cast<T *>(grad_increment),
            static_cast<T *>(grad_initial), batch, length, features);
    };
    if (broadcast) {
        launch(scan_backward_kernel<T, true>);
    } else {
        launch(scan_backward_kernel<T, false>);
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

int check_scan_shapes(int64_t batch, int64_t length, int64_t features) {
    if (batch < 0 || length < 0 || features < 0) {
        return fail(KOEMI_ERR_INVALID, "scan sizes must be non-negative");
    }
    if (batch > 0 && length > 0 && features > 0 &&
        batch > (int64_t(1) << 62) / length / features) {
        return fail(KOEMI_ERR_INVALID, "scan tensor is too large");
    }
    return KOEMI_OK;
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_dense_affine_scan_forward(const void *retention, const void *increment,
                                               const void *initial, void *states, int64_t batch,
                                               int64_t length, int64_t features,
                                               int broadcast_retention, int dtype, void *stream) {
    clear_error();
    int rc = check_scan_shapes(batch, length, features);
    if (rc != KOEMI_OK) return rc;
    if (batch == 0 || length == 0 || features == 0) return KOEMI_OK;
    if (retention == nullptr || increment == nullptr || states == nullptr) {
        return fail(KOEMI_ERR_INVALID, "retention, increment and states must be non-NULL");
    }
    // grid.y carries the batch, so batches above 65535 take the per-lane
    // kernel (scan_forward_typed), which has no such limit.
    const bool bc = broadcast_retention != 0;
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: return scan_forward_typed<float>(retention, increment, initial, states, batch, length, features, bc, s);
        case KOEMI_F16: return scan_forward_typed<__half>(retention, increment, initial, states, batch, length, features, bc, s);
        case KOEMI_BF16: return scan_forward_typed<__nv_bfloat16>(retention, increment, initial, states, batch, length, features, bc, s);
        case KOEMI_F64: return scan_forward_typed<double>(retention, increment, initial, states, batch, length, features, bc, s);
        default: return fail(KOEMI_ERR_INVALID, "unsupported scan dtype %d", dtype);
    }
}

extern "C" int koemi_dense_affine_scan_backward(const void *retention, const void *initial,
                                                const void *states, const void *grad_states,
                                                void *grad_retention, void *grad_increment,
                                                void *grad_initial, int64_t batch, int64_t length,
                                                int64_t features, int broadcast_retention,
                                                int dtype, void *stream) {
    clear_error();
    int rc = check_scan_shapes(batch, length, features);
    if (rc != KOEMI_OK) return rc;
    if (batch == 0 || length == 0 || features == 0) return KOEMI_OK;
    if (retention == nullptr || states == nullptr || grad_states == nullptr ||
        grad_retention == nullptr || grad_increment == nullptr) {
        return fail(KOEMI_ERR_INVALID, "scan backward tensors must be non-NULL");
    }
    const bool bc = broadcast_retention != 0;
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: return scan_backward_typed<float>(retention, initial, states, grad_states, grad_retention, grad_increment, grad_initial, batch, length, features, bc, s);
        case KOEMI_F16: return scan_backward_typed<__half>(retention, initial, states, grad_states, grad_retention, grad_increment, grad_initial, batch, length, features, bc, s);
        case KOEMI_BF16: return scan_backward_typed<__nv_bfloat16>(retention, initial, states, grad_states, grad_retention, grad_increment, grad_initial, batch, length, features, bc, s);
        case KOEMI_F64: return scan_backward_typed<double>(retention, initial, states, grad_states, grad_retention, grad_increment, grad_initial, batch, length, features, bc, s);
        default: return fail(KOEMI_ERR_INVALID, "unsupported scan dtype %d", dtype);
    }
}

// Gate epilogue fused with the padding masks (memory.py:22-26, network.py:308-309).
namespace koemi {
namespace {
__global__ void bounded_gates_kernel(const float *__restrict__ projections,
                                     const uint8_t *__restrict__ valid, float *__restrict__ retention,
                                     float *__restrict__ increment, int64_t rows, int64_t features,
                                     float lo, float hi) {
    const int64_t index = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (index >= rows * features) return;
    const int64_t row = index / features;
    const int64_t f = index - row * features;
    const bool keep = valid == nullptr || valid[row] != 0;
    if (!keep) {
        retention[index] = 1.0f;
        increment[index] = 0.0f;
        return;
    }
    const float pre_a = projections[row * 2 * features + f];
    const float pre_c = projections[row * 2 * features + features + f];
    const float a = lo + (hi - lo) * sigmoidf_(pre_a);
    retention[index] = a;
    increment[index] = (1.0f - a) * tanhf(pre_c);
}
}  // namespace
}  // namespace koemi

extern "C" int koemi_dense_bounded_gates(const float *projections, const uint8_t *valid,
                                         float *retention, float *increment, int64_t rows,
                                         int64_t features, float minimum_retention,
                                         float maximum_retention, void *stream) {
    clear_error();
    if (rows < 0 || features < 0) return fail(KOEMI_ERR_INVALID, "negative gate sizes");
    if (rows == 0 || features == 0) return KOEMI_OK;
    const int64_t total = rows * features;
    bounded_gates_kernel<<<static_cast<unsigned>(ceil_div(total, 256)), 256, 0, as_stream(stream)>>>(
        projections, valid, retention, increment, rows, features, minimum_retention,
        maximum_retention);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}
