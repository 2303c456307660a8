// Expert-parallel exchange over peer memory (NVLink / NVSwitch).
//
// Every rank allocates one exchange buffer with cudaMalloc and shares it with
// the other ranks through CUDA IPC handles (no NVLink multicast objects). The
// dispatch and return of token rows are then plain stores into the owner's or
// the sender's buffer, fused with the pack / unpack of the slabs, and a
// per-exchange epoch flag written with release semantics after the last row.
// Waiting kernels spin on the peers' flags with an iteration limit: when the
// limit runs out they record KOEMI_ERR_TIMEOUT in the device status word and
// return, so a missing peer never hangs the GPU.
//
// The buffer layout and the flag protocol are in peer.cuh.
#include <algorithm>
#include <cstring>

#include "peer.cuh"
#include "vec.cuh"

namespace koemi {
namespace {

constexpr int64_t kMaxPeerRanks = peer::kMaxRanks;
constexpr int64_t kEpochSlot = peer::kEpochSlot;
using peer::Layout;
using peer::layout;
using peer::signal_peers;
using peer::wait_flags;

template <typename T>
__device__ __forceinline__ void copy_row(T *dst, const T *src, int64_t width, bool vector, int lane) {
    if (vector) {
        constexpr int W = 16 / sizeof(T);
        for (int64_t p = lane; p < width / W; p += 32) {
            *reinterpret_cast<uint4 *>(dst + p * W) = load_stream(src + p * W);
        }
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = src[c];
    }
}

struct ExchangeArgs {
    const uint64_t *peers;  // [ranks] base address of every rank's buffer (own included)
    uint8_t *own;
    int64_t rank, ranks, local_experts, capacity, width;
    size_t ids, rows, ret;
    int *status;
};

// Sender: slab row (g, j) goes straight to owner g's recv block `rank`.
template <typename T>
__global__ void ep_dispatch_kernel(ExchangeArgs a, const T *__restrict__ sorted_rows,
                                   const int64_t *__restrict__ sorted_experts, const int64_t *__restrict__ offsets,
                                   bool vector) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint64_t epoch = reinterpret_cast<const volatile uint64_t *>(a.own)[kEpochSlot] + 1;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
         q < a.ranks * a.capacity; q += warps) {
        const int64_t g = q / a.capacity;
        const int64_t j = q - g * a.capacity;
        const int64_t i = offsets[g * a.local_experts] + j;
        const bool live = i < offsets[(g + 1) * a.local_experts];
        uint8_t *peer = reinterpret_cast<uint8_t *>(a.peers[g]);
        const int64_t slot = a.rank * a.capacity + j;
        if (lane == 0) {
            reinterpret_cast<int32_t *>(peer + a.ids)[slot] =
                live ? static_cast<int32_t>(sorted_experts[i] - g * a.local_experts) : -1;
        }
        if (live) copy_row(reinterpret_cast<T *>(peer + a.rows) + slot * a.width, sorted_rows + i * a.width, a.width,
                           vector, lane);
    }
    signal_peers(a.own, a.peers, 0, a.rank, a.ranks, epoch, true);
}

// Sender, fused with the row gather: slab row (g, j) is token row
// sorted_tokens[i] of `context` (converted to the exchange dtype T), stored
// straight into owner g's recv block `rank`. Saves the gathered copy of the
// sorted rows that the plain dispatch reads.
template <typename TI, typename T>
__global__ void ep_dispatch_gather_kernel(ExchangeArgs a, const TI *__restrict__ context,
                                          const int64_t *__restrict__ sorted_tokens,
                                          const int64_t *__restrict__ sorted_experts,
                                          const int64_t *__restrict__ offsets) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint64_t epoch = reinterpret_cast<const volatile uint64_t *>(a.own)[kEpochSlot] + 1;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    constexpr int W = 8;  // 8 elements per packet on both sides (16 B of T = 16-bit, 32 B of fp32)
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
         q < a.ranks * a.capacity; q += warps) {
        const int64_t g = q / a.capacity;
        const int64_t j = q - g * a.capacity;
        const int64_t i = offsets[g * a.local_experts] + j;
        const bool live = i < offsets[(g + 1) * a.local_experts];
        uint8_t *peer = reinterpret_cast<uint8_t *>(a.peers[g]);
        const int64_t slot = a.rank * a.capacity + j;
        if (lane == 0) {
            reinterpret_cast<int32_t *>(peer + a.ids)[slot] =
                live ? static_cast<int32_t>(sorted_experts[i] - g * a.local_experts) : -1;
        }
        if (!live) continue;
        const TI *src = context + sorted_tokens[i] * a.width;
        T *dst = reinterpret_cast<T *>(peer + a.rows) + slot * a.width;
        for (int64_t c = static_cast<int64_t>(lane) * W; c < a.width; c += 32 * W) {
            float v[8];
            if constexpr (sizeof(TI) == 4) {
                const float4 lo = *reinterpret_cast<const float4 *>(src + c);
                const float4 hi = *reinterpret_cast<const float4 *>(src + c + 4);
                v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
                v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
            } else {
                unpack(load_cached(src + c), v, TI());
            }
            *reinterpret_cast<uint4 *>(dst + c) = pack(v, T());
        }
    }
    signal_peers(a.own, a.peers, 0, a.rank, a.ranks, epoch, true);
}

// Sender, fused with the fusion RMSNorm of a decode block: token row t of
// `fused` (fp32 [tokens, width]) is normalised exactly as rms_rows_cached
// does it (x * rsqrt(mean(x^2) + eps) * weight, the same loads and sum
// order) into `context` (fp32, the combine's residual), and for each of its
// top_k pairs that routes to an expert the normalised row, converted to the
// exchange dtype T, goes straight into the owner's recv block `rank` at the
// pair's slot (its sorted index minus the owner's first pair). The ids of
// every slot of this sender's block in every owner (the owner-local expert,
// -1 past the owner's pairs) and the epoch flags follow, as in the gathering
// dispatch. One warp per row; width a multiple of 4 and at most 2048.
template <typename T>
__global__ void ep_norm_dispatch_kernel(ExchangeArgs a, const float *__restrict__ fused,
                                        const float *__restrict__ norm_weight, float *__restrict__ context,
                                        const int64_t *__restrict__ positions,
                                        const int64_t *__restrict__ sorted_experts,
                                        const int64_t *__restrict__ offsets, int64_t tokens, int64_t top_k,
                                        float eps) {
    pdl_trigger();
    pdl_wait();
    constexpr int NV = 16;  // 16-byte fp32 packets per lane: width <= 2048
    const int lane = threadIdx.x & 31;
    const uint64_t epoch = peer::current_epoch(a.own) + 1;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    const int64_t packets = a.width / 4;
    const int64_t valid_pairs = offsets[a.ranks * a.local_experts];
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); t < tokens;
         t += warps) {
        const float *xr = fused + t * a.width;
        float4 v[NV], w[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t p = lane + 32 * i;
            if (p < packets) {
                const uint4 raw = load_stream(xr + p * 4);
                v[i] = *reinterpret_cast<const float4 *>(&raw);
                const uint4 wraw = load_cached(norm_weight + p * 4);
                w[i] = *reinterpret_cast<const float4 *>(&wraw);
            }
        }
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            if (lane + 32 * i < packets) {
                sum = fmaf(v[i].x, v[i].x, sum);
                sum = fmaf(v[i].y, v[i].y, sum);
                sum = fmaf(v[i].z, v[i].z, sum);
                sum = fmaf(v[i].w, v[i].w, sum);
            }
        }
        sum = warp_sum(sum);
        const float inv = rsqrtf(sum / static_cast<float>(a.width) + eps);
        float *cr = context + t * a.width;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int64_t p = lane + 32 * i;
            if (p < packets) {
                v[i] = make_float4(v[i].x * inv * w[i].x, v[i].y * inv * w[i].y, v[i].z * inv * w[i].z,
                                   v[i].w * inv * w[i].w);
                *reinterpret_cast<float4 *>(cr + p * 4) = v[i];
            }
        }
        for (int64_t s = 0; s < top_k; ++s) {
            const int64_t pos = positions[t * top_k + s];
            if (pos < 0 || pos >= valid_pairs) continue;
            int64_t g = a.ranks - 1;
            while (g > 0 && offsets[g * a.local_experts] > pos) --g;
            const int64_t slot = a.rank * a.capacity + pos - offsets[g * a.local_experts];
            uint8_t *peer_buffer = reinterpret_cast<uint8_t *>(a.peers[g]);
            if (lane == 0) {
                reinterpret_cast<int32_t *>(peer_buffer + a.ids)[slot] =
                    static_cast<int32_t>(sorted_experts[pos] - g * a.local_experts);
            }
            T *dst = reinterpret_cast<T *>(peer_buffer + a.rows) + slot * a.width;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int64_t p = lane + 32 * i;
                if (p < packets) {
                    union {
                        T h[4];
                        uint2 u;
                    } out;
                    out.h[0] = from_acc<T>(v[i].x);
                    out.h[1] = from_acc<T>(v[i].y);
                    out.h[2] = from_acc<T>(v[i].z);
                    out.h[3] = from_acc<T>(v[i].w);
                    *reinterpret_cast<uint2 *>(dst + p * 4) = out.u;
                }
            }
        }
    }
    // this sender's dead slots in every owner's block
    const int64_t threads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < a.ranks * a.capacity;
         q += threads) {
        const int64_t g = q / a.capacity;
        const int64_t j = q - g * a.capacity;
        if (j >= offsets[(g + 1) * a.local_experts] - offsets[g * a.local_experts]) {
            reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(a.peers[g]) + a.ids)[a.rank * a.capacity + j] = -1;
        }
    }
    signal_peers(a.own, a.peers, 0, a.rank, a.ranks, epoch, true);
}

// Owner, fused: wait for every sender's rows, then (every CTA redundantly, in
// shared memory) the stable counting sort of the received slots by local
// expert -- slot order [sender][j], dead slots (id -1) last -- and each CTA
// gathers its share of the live rows into expert-major order. CTA 0 writes
// the segment offsets [local + 1], the sorted expert ids (local for dead
// slots) and each slot's sorted position. Replaces the wait kernel, the
// validity mask and the general permutation of the received rows.
constexpr int kOwnerThreads = 512;
constexpr int kOwnerWarps = kOwnerThreads / 32;
constexpr int64_t kOwnerMaxSlots = 4096;
constexpr int64_t kOwnerMaxExperts = 255;
constexpr int32_t kExpertTileRows = 128;  // row tile of the tcgen05 grouped GEMM (umma.cu kBM)

template <typename T>
__global__ __launch_bounds__(kOwnerThreads) void ep_owner_sort_kernel(ExchangeArgs a, T *__restrict__ sorted_rows,
                                                                      int64_t *__restrict__ offsets_out,
                                                                      int64_t *__restrict__ experts_out,
                                                                      int64_t *__restrict__ positions_out,
                                                                      int64_t *__restrict__ slots_out,
                                                                      int32_t *__restrict__ tile_prefix_out,
                                                                      bool vector) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ int32_t shared[];
    // a wait that gives up (status word set) sorts every slot as dead, so the
    // outputs stay well formed: empty segments, no rows
    const bool arrived = wait_flags(a.own, 0, a.ranks, a.status);
    const int n = static_cast<int>(a.ranks * a.capacity);
    const int buckets = static_cast<int>(a.local_experts) + 1;
    int32_t *keys = shared;                       // [n]
    int32_t *order = keys + n;                    // [n] slot at each sorted position
    int32_t *running = order + n;                 // [buckets]
    int32_t *warp_counts = running + buckets;     // [kOwnerWarps][buckets]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int32_t *ids = reinterpret_cast<const int32_t *>(a.own + a.ids);
    for (int b = threadIdx.x; b < buckets; b += kOwnerThreads) running[b] = 0;
    for (int i = threadIdx.x; i < kOwnerWarps * buckets; i += kOwnerThreads) warp_counts[i] = 0;
    __syncthreads();
    for (int q = threadIdx.x; q < n; q += kOwnerThreads) {
        const int32_t id = arrived ? ids[q] : -1;
        const int32_t key = id < 0 || id >= a.local_experts ? static_cast<int32_t>(a.local_experts) : id;
        keys[q] = key;
        atomicAdd(&running[key], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan (at most 256 buckets)
        int32_t carry = 0, tiles = 0;
        for (int b = 0; b < buckets; ++b) {
            const int32_t v = running[b];
            running[b] = carry;
            if (blockIdx.x == 0) {
                offsets_out[b] = carry;
                // the grouped GEMM's tile map: 128-row tiles before each local expert
                if (tile_prefix_out != nullptr && b < a.local_experts) {
                    tile_prefix_out[b] = tiles;
                    tiles += (v + kExpertTileRows - 1) / kExpertTileRows;
                }
            }
            carry += v;
        }
        if (blockIdx.x == 0 && tile_prefix_out != nullptr) tile_prefix_out[a.local_experts] = tiles;
    }
    __syncthreads();
    const unsigned lower = (1u << lane) - 1u;
    for (int base = 0; base < n; base += kOwnerThreads) {
        const int q = base + static_cast<int>(threadIdx.x);
        const bool live = q < n;
        const int32_t key = live ? keys[q] : 0;
        const int digit = live ? key : -1 - lane;
        const unsigned same = __match_any_sync(0xffffffffu, digit);
        const int rank = __popc(same & lower);
        if (live && (same & lower) == 0) warp_counts[warp * buckets + digit] = __popc(same);
        __syncthreads();
        if (live) {
            int32_t before = 0;
            for (int w = 0; w < warp; ++w) before += warp_counts[w * buckets + digit];
            order[running[digit] + before + rank] = q;
        }
        __syncthreads();
        for (int b = threadIdx.x; b < buckets; b += kOwnerThreads) {
            int32_t total = 0;
            for (int w = 0; w < kOwnerWarps; ++w) {
                total += warp_counts[w * buckets + b];
                warp_counts[w * buckets + b] = 0;
            }
            running[b] += total;
        }
        __syncthreads();
    }
    // after the scatter, running[b] is the end of bucket b: the live rows end
    // where the last expert's bucket does
    const int32_t live_rows = running[a.local_experts - 1];
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < n; i += kOwnerThreads) {
            const int32_t q = order[i];
            experts_out[i] = keys[q];
            positions_out[q] = i;
            if (slots_out != nullptr) slots_out[i] = q;
        }
    }
    // rows of sorted positions [0, live_rows): one warp per row, CTAs strided
    const T *recv = reinterpret_cast<const T *>(a.own + a.rows);
    const int64_t warps_total = static_cast<int64_t>(gridDim.x) * kOwnerWarps;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kOwnerWarps + warp; i < live_rows; i += warps_total) {
        copy_row(sorted_rows + i * a.width, recv + static_cast<int64_t>(order[i]) * a.width, a.width, vector, lane);
    }
}

// Owner: wait until every sender's rows of this exchange have landed.
__global__ void ep_wait_dispatch_kernel(const uint8_t *own, int64_t ranks, int *status) {
    pdl_trigger();
    pdl_wait();
    wait_flags(own, 0, ranks, status);
}

// Owner: received row (s, j) with a live id goes back to sender s's ret
// block `rank`, from the local expert outputs at local_positions[(s, j)].
template <typename T>
__global__ void ep_return_kernel(ExchangeArgs a, const T *__restrict__ local_out,
                                 const int64_t *__restrict__ local_positions, bool vector) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint64_t epoch = reinterpret_cast<const volatile uint64_t *>(a.own)[kEpochSlot];
    const int32_t *ids = reinterpret_cast<const int32_t *>(a.own + a.ids);
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
         q < a.ranks * a.capacity; q += warps) {
        if (ids[q] < 0) continue;
        const int64_t s = q / a.capacity;
        const int64_t j = q - s * a.capacity;
        uint8_t *peer = reinterpret_cast<uint8_t *>(a.peers[s]);
        copy_row(reinterpret_cast<T *>(peer + a.ret) + (a.rank * a.capacity + j) * a.width,
                 local_out + local_positions[q] * a.width, a.width, vector, lane);
    }
    signal_peers(a.own, a.peers, 1, a.rank, a.ranks, epoch, false);
}

// Sender: wait for every owner's returns, then unpack into sorted order.
template <typename T>
__global__ void ep_collect_kernel(ExchangeArgs a, const int64_t *__restrict__ sorted_experts,
                                  const int64_t *__restrict__ offsets, T *__restrict__ sorted_out, int64_t pairs,
                                  bool vector) {
    pdl_trigger();
    pdl_wait();
    if (!wait_flags(a.own, 1, a.ranks, a.status)) return;
    const int lane = threadIdx.x & 31;
    const T *ret = reinterpret_cast<const T *>(a.own + a.ret);
    const int64_t valid = offsets[a.ranks * a.local_experts];
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); i < pairs;
         i += warps) {
        T *dst = sorted_out + i * a.width;
        if (i < valid) {
            const int64_t g = sorted_experts[i] / a.local_experts;
            copy_row(dst, ret + (g * a.capacity + i - offsets[g * a.local_experts]) * a.width, a.width, vector, lane);
        } else if (vector) {
            constexpr int W = 16 / sizeof(T);
            for (int64_t p = lane; p < a.width / W; p += 32) *reinterpret_cast<uint4 *>(dst + p * W) = make_uint4(0, 0, 0, 0);
        } else {
            for (int64_t c = lane; c < a.width; c += 32) dst[c] = from_acc<T>(0.0f);
        }
    }
}

int exchange_args(ExchangeArgs *a, const uint64_t *peers, void *own, int64_t rank, int64_t ranks,
                  int64_t local_experts, int64_t capacity, int64_t width, int dtype) {
    if (ranks < 1 || ranks > kMaxPeerRanks || rank < 0 || rank >= ranks) {
        return fail(KOEMI_ERR_INVALID, "peer exchange needs 1 <= ranks <= %lld and 0 <= rank < ranks", (long long)kMaxPeerRanks);
    }
    if (local_experts < 1 || capacity < 1 || width < 1) return fail(KOEMI_ERR_INVALID, "bad exchange sizes");
    const size_t es = dtype_size(dtype);
    if (dtype != KOEMI_F32 && dtype != KOEMI_F16 && dtype != KOEMI_BF16) return fail(KOEMI_ERR_INVALID, "rows must be f32, f16 or bf16");
    if (peers == nullptr || own == nullptr || !aligned(own, 256)) return fail(KOEMI_ERR_INVALID, "exchange buffers must be 256-byte aligned");
    const Layout l = layout(ranks, capacity, width, es);
    *a = ExchangeArgs{peers, static_cast<uint8_t *>(own), rank, ranks, local_experts, capacity, width, l.ids, l.rows, l.ret,
                      device_status_word()};
    return KOEMI_OK;
}

unsigned exchange_blocks(int64_t rows) {
    const int64_t wanted = ceil_div(rows, 8);
    const int64_t cap = static_cast<int64_t>(sm_count()) * 4;
    return static_cast<unsigned>(wanted < 1 ? 1 : (wanted > cap ? cap : wanted));
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" size_t koemi_peer_exchange_bytes(int64_t ranks, int64_t capacity, int64_t width, int dtype) {
    if (ranks < 1 || capacity < 1 || width < 1 || dtype_size(dtype) == 0) return 0;
    return layout(ranks, capacity, width, dtype_size(dtype)).total;
}

extern "C" int koemi_peer_exchange_offsets(int64_t ranks, int64_t capacity, int64_t width, int dtype,
                                           size_t *ids_offset, size_t *rows_offset) {
    clear_error();
    if (ranks < 1 || capacity < 1 || width < 1 || dtype_size(dtype) == 0 || ids_offset == nullptr || rows_offset == nullptr) {
        return fail(KOEMI_ERR_INVALID, "bad exchange layout arguments");
    }
    const Layout l = layout(ranks, capacity, width, dtype_size(dtype));
    *ids_offset = l.ids;
    *rows_offset = l.rows;
    return KOEMI_OK;
}

extern "C" int koemi_peer_buffer_alloc(size_t bytes, void **ptr, void *handle_out) {
    clear_error();
    if (ptr == nullptr || handle_out == nullptr || bytes == 0) return fail(KOEMI_ERR_INVALID, "bad peer buffer arguments");
    void *p = nullptr;
    KOEMI_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t handle;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&handle, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(KOEMI_ERR_CUDA, "peer buffer: %s", cudaGetErrorString(e));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) <= KOEMI_PEER_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &handle, sizeof(handle));
    *ptr = p;
    return KOEMI_OK;
}

extern "C" int koemi_peer_buffer_open(const void *handle, void **ptr) {
    clear_error();
    if (handle == nullptr || ptr == nullptr) return fail(KOEMI_ERR_INVALID, "bad peer handle arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    KOEMI_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return KOEMI_OK;
}

extern "C" int koemi_peer_buffer_close(void *ptr) {
    clear_error();
    KOEMI_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return KOEMI_OK;
}

extern "C" int koemi_peer_buffer_free(void *ptr) {
    clear_error();
    KOEMI_CUDA_TRY(cudaFree(ptr));
    return KOEMI_OK;
}

extern "C" int koemi_ep_dispatch(const void *sorted_rows, const int64_t *sorted_experts, const int64_t *segment_offsets,
                                 const uint64_t *peers, void *own, int64_t pairs, int64_t width, int64_t rank,
                                 int64_t ranks, int64_t local_experts, int64_t capacity, int dtype, void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    if (capacity < pairs) return fail(KOEMI_ERR_INVALID, "capacity %lld is below the %lld pairs one owner may receive", (long long)capacity, (long long)pairs);
    const bool vector = (width * static_cast<int64_t>(dtype_size(dtype))) % 16 == 0 && aligned(sorted_rows, 16);
    const unsigned blocks = exchange_blocks(ranks * capacity);
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: KOEMI_CUDA_TRY(launch_pdl(ep_dispatch_kernel<float>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const float *>(sorted_rows), sorted_experts, segment_offsets, vector)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(ep_dispatch_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const __half *>(sorted_rows), sorted_experts, segment_offsets, vector)); break;
        default: KOEMI_CUDA_TRY(launch_pdl(ep_dispatch_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const __nv_bfloat16 *>(sorted_rows), sorted_experts, segment_offsets, vector)); break;
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_wait_dispatch(const void *own, int64_t ranks, void *stream) {
    clear_error();
    if (own == nullptr || ranks < 1 || ranks > kMaxPeerRanks) return fail(KOEMI_ERR_INVALID, "bad exchange wait arguments");
    KOEMI_CUDA_TRY(launch_pdl(ep_wait_dispatch_kernel, dim3(1), dim3(32), 0, as_stream(stream), dim3(1, 1, 1), static_cast<const uint8_t *>(own), ranks, device_status_word()));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_return(const void *local_out, const int64_t *local_positions, const uint64_t *peers, void *own,
                               int64_t width, int64_t rank, int64_t ranks, int64_t local_experts, int64_t capacity,
                               int dtype, void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    const bool vector = (width * static_cast<int64_t>(dtype_size(dtype))) % 16 == 0 && aligned(local_out, 16);
    const unsigned blocks = exchange_blocks(ranks * capacity);
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: KOEMI_CUDA_TRY(launch_pdl(ep_return_kernel<float>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const float *>(local_out), local_positions, vector)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(ep_return_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const __half *>(local_out), local_positions, vector)); break;
        default: KOEMI_CUDA_TRY(launch_pdl(ep_return_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, static_cast<const __nv_bfloat16 *>(local_out), local_positions, vector)); break;
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_collect(const int64_t *sorted_experts, const int64_t *segment_offsets, void *sorted_out,
                                const uint64_t *peers, void *own, int64_t pairs, int64_t width, int64_t rank,
                                int64_t ranks, int64_t local_experts, int64_t capacity, int dtype, void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    if (pairs == 0) return KOEMI_OK;
    const bool vector = (width * static_cast<int64_t>(dtype_size(dtype))) % 16 == 0 && aligned(sorted_out, 16);
    const unsigned blocks = exchange_blocks(pairs);
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: KOEMI_CUDA_TRY(launch_pdl(ep_collect_kernel<float>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, sorted_experts, segment_offsets, static_cast<float *>(sorted_out), pairs, vector)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(ep_collect_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, sorted_experts, segment_offsets, static_cast<__half *>(sorted_out), pairs, vector)); break;
        default: KOEMI_CUDA_TRY(launch_pdl(ep_collect_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, sorted_experts, segment_offsets, static_cast<__nv_bfloat16 *>(sorted_out), pairs, vector)); break;
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_dispatch_gather(const void *context, int context_dtype, const int64_t *sorted_tokens,
                                        const int64_t *sorted_experts, const int64_t *segment_offsets,
                                        const uint64_t *peers, void *own, int64_t pairs, int64_t width, int64_t rank,
                                        int64_t ranks, int64_t local_experts, int64_t capacity, int dtype,
                                        void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    if (capacity < pairs) return fail(KOEMI_ERR_INVALID, "capacity %lld is below the %lld pairs one owner may receive", (long long)capacity, (long long)pairs);
    if (dtype == KOEMI_F32 || width % 8 != 0 || !aligned(context, 16) || context == nullptr || sorted_tokens == nullptr) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the gathering dispatch takes 16-bit exchange rows, width a multiple of 8 and 16-byte aligned context");
    }
    const unsigned blocks = exchange_blocks(ranks * capacity);
    cudaStream_t s = as_stream(stream);
#define KOEMI_DISPATCH_GATHER(TI, T) \
    KOEMI_CUDA_TRY(launch_pdl(ep_dispatch_gather_kernel<TI, T>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a, \
                              static_cast<const TI *>(context), sorted_tokens, sorted_experts, segment_offsets))
    if (context_dtype == KOEMI_F32 && dtype == KOEMI_BF16) KOEMI_DISPATCH_GATHER(float, __nv_bfloat16);
    else if (context_dtype == KOEMI_F32 && dtype == KOEMI_F16) KOEMI_DISPATCH_GATHER(float, __half);
    else if (context_dtype == KOEMI_BF16 && dtype == KOEMI_BF16) KOEMI_DISPATCH_GATHER(__nv_bfloat16, __nv_bfloat16);
    else if (context_dtype == KOEMI_F16 && dtype == KOEMI_F16) KOEMI_DISPATCH_GATHER(__half, __half);
    else return fail(KOEMI_ERR_INVALID, "context dtype must be f32 or the exchange dtype");
#undef KOEMI_DISPATCH_GATHER
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_norm_dispatch(const float *fused, const float *norm_weight, float eps, float *context,
                                      const int64_t *pair_positions, const int64_t *sorted_experts,
                                      const int64_t *segment_offsets, int64_t tokens, int64_t top_k,
                                      const uint64_t *peers, void *own, int64_t width, int64_t rank, int64_t ranks,
                                      int64_t local_experts, int64_t capacity, int dtype, void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    if (tokens < 0 || top_k < 1) return fail(KOEMI_ERR_INVALID, "bad token count or top_k");
    if (capacity < tokens * top_k) {
        return fail(KOEMI_ERR_INVALID, "capacity %lld is below the %lld pairs one owner may receive",
                    (long long)capacity, (long long)(tokens * top_k));
    }
    if ((dtype != KOEMI_BF16 && dtype != KOEMI_F16) || width % 4 != 0 || width > 2048 || !aligned(fused, 16) ||
        !aligned(norm_weight, 16) || !aligned(context, 16) || pair_positions == nullptr || sorted_experts == nullptr ||
        segment_offsets == nullptr) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the normalising dispatch takes 16-bit exchange rows, width a multiple of 4 "
                                           "up to 2048 and 16-byte aligned rows");
    }
    const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, ceil_div(tokens, 8)));
    cudaStream_t s = as_stream(stream);
    if (dtype == KOEMI_BF16) {
        KOEMI_CUDA_TRY(launch_pdl(ep_norm_dispatch_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a,
                                  fused, norm_weight, context, pair_positions, sorted_experts, segment_offsets, tokens,
                                  top_k, eps));
    } else {
        KOEMI_CUDA_TRY(launch_pdl(ep_norm_dispatch_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), a,
                                  fused, norm_weight, context, pair_positions, sorted_experts, segment_offsets, tokens,
                                  top_k, eps));
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_ep_owner_sort(const uint64_t *peers, void *own, int64_t width, int64_t rank, int64_t ranks,
                                   int64_t local_experts, int64_t capacity, int dtype, void *sorted_rows,
                                   int64_t *segment_offsets, int64_t *sorted_experts, int64_t *positions,
                                   int64_t *slots, int32_t *tile_prefix, void *stream) {
    clear_error();
    ExchangeArgs a;
    int rc = exchange_args(&a, peers, own, rank, ranks, local_experts, capacity, width, dtype);
    if (rc != KOEMI_OK) return rc;
    const int64_t n = ranks * capacity;
    if (n > kOwnerMaxSlots || local_experts > kOwnerMaxExperts) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the owner sort takes at most %lld slots and %lld local experts",
                    (long long)kOwnerMaxSlots, (long long)kOwnerMaxExperts);
    }
    if (sorted_rows == nullptr || segment_offsets == nullptr || sorted_experts == nullptr || positions == nullptr) {
        return fail(KOEMI_ERR_INVALID, "owner sort outputs must be non-NULL");
    }
    const bool vector = (width * static_cast<int64_t>(dtype_size(dtype))) % 16 == 0 && aligned(sorted_rows, 16);
    const int64_t buckets = local_experts + 1;
    const size_t smem = static_cast<size_t>(2 * n + buckets * (kOwnerWarps + 1)) * sizeof(int32_t);
    const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(64, ceil_div(n, 64))));
    cudaStream_t s = as_stream(stream);
    auto go = [&](auto kernel, auto *typed) -> int {
        if (smem > 48 * 1024) {
            KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        }
        KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(blocks), dim3(kOwnerThreads), smem, s, dim3(1, 1, 1), a, typed,
                                  segment_offsets, sorted_experts, positions, slots, tile_prefix, vector));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    switch (dtype) {
        case KOEMI_F32: return go(ep_owner_sort_kernel<float>, static_cast<float *>(sorted_rows));
        case KOEMI_F16: return go(ep_owner_sort_kernel<__half>, static_cast<__half *>(sorted_rows));
        default: return go(ep_owner_sort_kernel<__nv_bfloat16>, static_cast<__nv_bfloat16 *>(sorted_rows));
    }
}
