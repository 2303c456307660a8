// Dense front: affine recurrent scan h_t = a_t * h_{t-1} + b_t.
//
// Layout: retention/increment/states are [batch, length, features] row-major
// (features contiguous), fp32 state. Three kernels:
//   - scan_segment_kernel (with a caller workspace): the sequence is cut into
//     segments scanned by separate CTAs that pass carries by decoupled
//     look-back (described at the kernel); thousands of CTAs at prefill sizes.
//   - scan_forward_kernel (no workspace): one CTA owns 32 features of one
//     batch row and walks the whole sequence in chunks of 64 positions staged
//     by TMA (3D tensor map, box {32 features, 64 positions, 1}) through a
//     multi-stage mbarrier pipeline. Inside a chunk, warp w owns positions
//     [8w, 8w + 8) and lane l owns feature l: each thread composes its 8
//     affine maps into one (A, B) pair, the per-warp pairs are exchanged
//     through shared memory to form each warp's carry-in from the running
//     state, and the thread replays its 8 steps to produce h_t.
//   - scan_forward_short_kernel: T <= 8 (decode steps), one thread per lane.
// Reference behaviour: dense/affine_scan.cu:18-56 (sequential per lane) and
// model/scan.py:17-30 (log-step doubling); all compute the same recurrence.
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

// Segmented scan with decoupled look-back. The sequence is cut into segments
// of kSegment positions; a tile is (segment, batch row, 64 features) and one
// CTA scans one tile, so config-sized problems launch thousands of CTAs
// instead of one serial walker per 32 features. Each CTA:
//   1. takes a ticket from a global counter (tickets are handed out in launch
//      order, segment-major, so every predecessor tile already runs) and
//      loads its a/b rows with one 3D TMA box per warp (warp w owns rows
//      [w P, w P + P), P = kSegment / 4; lane l owns features 2l, 2l + 1);
//   2. composes each warp's P steps into one affine map, then the 4 warp
//      maps into the tile map (A, B);
//   3. publishes (A, B), walks back over the predecessor tiles of the same
//      (batch, feature) chain -- composing their maps until it meets a
//      published end state -- and publishes its own end state A h_in + B;
//   4. replays its rows from h_in, writes h_t over b_t in shared memory and
//      stores the rows with one TMA store per warp.
// Published values carry their own validity: the host fills the workspace
// with 0xFF bytes, a float whose bits are all ones is "not yet written", and
// a writer never stores that pattern (any NaN is stored as the canonical
// 0x7FFFFFFF). Each 4-byte store is single-copy atomic, so a reader checks
// every component it loads and needs no flag, fence or acquire. The walk
// loads the records of up to 8 predecessors at once, one L2 round trip per
// window. HBM traffic is a, b read once and h written once; the look-back
// moves 768 B per tile. Every wait is bounded.
constexpr int kSegFeatures = 64;
constexpr int kSegWarps = 4;
constexpr int kSegThreads = kSegWarps * 32;

template <typename T>
constexpr int segment_length() {
    return sizeof(T) == 2 ? 128 : 64;  // 32 KB of a + b per tile either way: six CTAs per SM
}

struct ScanWorkspace {
    // [0, 256): ticket counter (starts at 0xFFFFFFFF, so the first ticket is
    // the wrapped increment 0); then per tile, lane-major: maps
    // {A(2l), A(2l+1), B(2l), B(2l+1)} x 32 lanes (512 B) and end states
    // {H(2l), H(2l+1)} x 32 lanes (256 B). All of it is filled with 0xFF.
    static constexpr size_t kHead = 256;
    static constexpr size_t kTileBytes = 3 * kSegFeatures * 4;
    __host__ __device__ static size_t bytes(int64_t tiles) { return kHead + tiles * kTileBytes; }
};

constexpr uint32_t kUnwritten = 0xFFFFFFFFu;

__device__ __forceinline__ float publishable(float v) {
    return __float_as_uint(v) == kUnwritten ? __uint_as_float(0x7FFFFFFFu) : v;
}
__device__ __forceinline__ bool written(float v) { return __float_as_uint(v) != kUnwritten; }

__device__ __forceinline__ float4 ld_relaxed_f4(const float *p) {
    float4 v;
    asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_f4(float *p, float4 v) {
    asm volatile("st.relaxed.gpu.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_relaxed_f2(float *p, float2 v) {
    asm volatile("st.relaxed.gpu.global.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(v.x), "f"(v.y) : "memory");
}

__device__ __forceinline__ float2 ld_relaxed_f2(const float *p) {
    float2 v;
    asm volatile("ld.relaxed.gpu.global.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int32_t c0, int32_t c1,
                                             int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_drain() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Two adjacent features of one row, as fp32.
__device__ __forceinline__ float2 load_pair(const __nv_bfloat16 *p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
}
__device__ __forceinline__ float2 load_pair(const __half *p) {
    return __half22float2(*reinterpret_cast<const __half2 *>(p));
}
__device__ __forceinline__ float2 load_pair(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ void store_pair(__nv_bfloat16 *p, float x, float y) {
    *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(x, y);
}
__device__ __forceinline__ void store_pair(__half *p, float x, float y) {
    *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(x, y);
}
__device__ __forceinline__ void store_pair(float *p, float x, float y) {
    *reinterpret_cast<float2 *>(p) = make_float2(x, y);
}

template <typename T>
size_t segment_smem_bytes() {
    constexpr int kSegment = segment_length<T>();
    return 2 * size_t(kSegment) * kSegFeatures * sizeof(T)     // a, b (h over b)
           + 2 * kSegWarps * kSegFeatures * sizeof(float)      // warp maps
           + kSegFeatures * sizeof(float)                      // h_in
           + kSegment * sizeof(float)                          // broadcast a
           + kSegWarps * sizeof(uint64_t) + 16;                // barriers, ticket
}

template <typename T, bool kBroadcast>
__global__ __launch_bounds__(kSegThreads, 6) void scan_segment_kernel(
    const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
    const __grid_constant__ CUtensorMap map_h, const T *__restrict__ retention, const T *__restrict__ initial,
    int64_t length, int64_t features, int64_t chains, int64_t feature_tiles, unsigned char *workspace,
    int64_t tiles, int *status) {
    constexpr int kSegment = segment_length<T>();
    constexpr int kRows = kSegment / kSegWarps;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    T *tile_a = reinterpret_cast<T *>(smem_raw);
    T *tile_b = tile_a + kSegment * kSegFeatures;
    float *warp_a = reinterpret_cast<float *>(tile_b + kSegment * kSegFeatures);
    float *warp_b = warp_a + kSegWarps * kSegFeatures;
    float *h_in = warp_b + kSegWarps * kSegFeatures;
    float *bcast_a = h_in + kSegFeatures;
    uint64_t *full = reinterpret_cast<uint64_t *>(bcast_a + kSegment);
    uint32_t *shared_ticket = reinterpret_cast<uint32_t *>(full + kSegWarps);

    uint32_t *counter = reinterpret_cast<uint32_t *>(workspace);
    float *records = reinterpret_cast<float *>(workspace + ScanWorkspace::kHead);
    constexpr int kRecord = 3 * kSegFeatures;  // floats per tile

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        *shared_ticket = atomicAdd(counter, 1u) + 1u;
        for (int w = 0; w < kSegWarps; ++w) mbar_init(&full[w], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t ticket = *shared_ticket;
    const int64_t segment = ticket / chains;
    const int64_t chain = ticket - segment * chains;
    const int64_t batch = chain / feature_tiles;
    const int32_t f0 = static_cast<int32_t>((chain - batch * feature_tiles) * kSegFeatures);
    const int32_t t0 = static_cast<int32_t>(segment * kSegment);

    if (threadIdx.x == 0) {
        constexpr uint32_t kWarpBytes = (kBroadcast ? 1u : 2u) * kRows * kSegFeatures * sizeof(T);
        for (int w = 0; w < kSegWarps; ++w) {
            mbar_arrive_expect_tx(&full[w], kWarpBytes);
            const int64_t offset = int64_t(w) * kRows * kSegFeatures;
            if (!kBroadcast) {
                tma_load_3d(tile_a + offset, &map_a, &full[w], f0, t0 + w * kRows, static_cast<int32_t>(batch));
            }
            tma_load_3d(tile_b + offset, &map_b, &full[w], f0, t0 + w * kRows, static_cast<int32_t>(batch));
        }
    }
    if constexpr (kBroadcast) {
        for (int i = threadIdx.x; i < kSegment; i += kSegThreads) {
            const int64_t t = int64_t(t0) + i;
            bcast_a[i] = t < length ? to_acc(retention[batch * length + t]) : 0.0f;
        }
        __syncthreads();
    }

    // 2. This warp's rows composed into one map per feature.
    bool ok = mbar_wait_bounded(&full[warp], 0, status);
    const int col = 2 * lane;
    float ax = 1.f, ay = 1.f, bx = 0.f, by = 0.f;
    if (ok) {
#pragma unroll 8
        for (int j = 0; j < kRows; ++j) {
            const int row = warp * kRows + j;
            const float2 a = kBroadcast ? make_float2(bcast_a[row], bcast_a[row])
                                        : load_pair(tile_a + row * kSegFeatures + col);
            const float2 b = load_pair(tile_b + row * kSegFeatures + col);
            ax *= a.x;
            ay *= a.y;
            bx = fmaf(a.x, bx, b.x);
            by = fmaf(a.y, by, b.y);
        }
    }
    warp_a[warp * kSegFeatures + col] = ax;
    warp_a[warp * kSegFeatures + col + 1] = ay;
    warp_b[warp * kSegFeatures + col] = bx;
    warp_b[warp * kSegFeatures + col + 1] = by;
    if (__syncthreads_or(!ok)) {
        // A load gave up: publish an end state (zeros) so successors do not
        // wait, give this warp's copies one more bounded wait, then leave.
        if (warp == 0) st_relaxed_f2(records + ticket * kRecord + 2 * kSegFeatures + col, make_float2(0.f, 0.f));
        if (!ok) mbar_wait_bounded(&full[warp], 0, nullptr);
        return;
    }

    // 3. Tile map, look-back and publication (warp 0).
    if (warp == 0) {
        float TAx = 1.f, TAy = 1.f, TBx = 0.f, TBy = 0.f;
#pragma unroll
        for (int w = 0; w < kSegWarps; ++w) {
            const float wax = warp_a[w * kSegFeatures + col], way = warp_a[w * kSegFeatures + col + 1];
            TAx *= wax;
            TAy *= way;
            TBx = fmaf(wax, TBx, warp_b[w * kSegFeatures + col]);
            TBy = fmaf(way, TBy, warp_b[w * kSegFeatures + col + 1]);
        }
        float *record = records + ticket * kRecord;
        float hx = 0.f, hy = 0.f;
        if (segment == 0) {
            const int64_t f = int64_t(f0) + col;
            if (initial != nullptr) {
                if (f < features) hx = to_acc(initial[batch * features + f]);
                if (f + 1 < features) hy = to_acc(initial[batch * features + f + 1]);
            }
        } else {
            st_relaxed_f4(record + 4 * lane, make_float4(publishable(TAx), publishable(TAy), publishable(TBx),
                                                        publishable(TBy)));
            // h_in = M_A * h_end(p) + M_B while walking p back along the chain;
            // a window loads the records of up to kWindow predecessors at once.
            constexpr int kWindow = 8;
            float MAx = 1.f, MAy = 1.f, MBx = 0.f, MBy = 0.f;
            int64_t p = ticket - chains;
            bool done = false;
            uint32_t spins = 0;
            while (!done) {
                float4 maps[kWindow];
                float2 ends[kWindow];
#pragma unroll
                for (int i = 0; i < kWindow; ++i) {
                    const int64_t q = p - i * chains;
                    if (q >= 0) {
                        const float *r = records + q * kRecord;
                        ends[i] = ld_relaxed_f2(r + 2 * kSegFeatures + col);
                        maps[i] = ld_relaxed_f4(r + 4 * lane);
                    }
                }
                int advanced = 0;
#pragma unroll
                for (int i = 0; i < kWindow; ++i) {
                    if (done || advanced != i || p - i * chains < 0) continue;
                    if (written(ends[i].x) && written(ends[i].y)) {
                        hx = fmaf(MAx, ends[i].x, MBx);
                        hy = fmaf(MAy, ends[i].y, MBy);
                        done = true;
                    } else if (written(maps[i].x) && written(maps[i].y) && written(maps[i].z) &&
                               written(maps[i].w)) {
                        MBx = fmaf(MAx, maps[i].z, MBx);
                        MBy = fmaf(MAy, maps[i].w, MBy);
                        MAx *= maps[i].x;
                        MAy *= maps[i].y;
                        advanced = i + 1;
                    }
                }
                if (done) break;
                if (advanced > 0) {
                    p -= advanced * chains;
                    spins = 0;
                } else if (++spins >= (1u << 20)) {  // each try is an L2 round trip: about a second in all
                    atomicExch(status, KOEMI_ERR_TIMEOUT);
                    break;
                }
            }
        }
        st_relaxed_f2(record + 2 * kSegFeatures + col,
                      make_float2(publishable(fmaf(TAx, hx, TBx)), publishable(fmaf(TAy, hy, TBy))));
        h_in[col] = hx;
        h_in[col + 1] = hy;
    }
    __syncthreads();

    // 4. Replay from this warp's carry-in; h_t overwrites b_t; TMA store.
    float hx = h_in[col], hy = h_in[col + 1];
    for (int w = 0; w < warp; ++w) {
        hx = fmaf(warp_a[w * kSegFeatures + col], hx, warp_b[w * kSegFeatures + col]);
        hy = fmaf(warp_a[w * kSegFeatures + col + 1], hy, warp_b[w * kSegFeatures + col + 1]);
    }
#pragma unroll 8
    for (int j = 0; j < kRows; ++j) {
        const int row = warp * kRows + j;
        const float2 a = kBroadcast ? make_float2(bcast_a[row], bcast_a[row])
                                    : load_pair(tile_a + row * kSegFeatures + col);
        T *slot = tile_b + row * kSegFeatures + col;
        const float2 b = load_pair(slot);
        hx = fmaf(a.x, hx, b.x);
        hy = fmaf(a.y, hy, b.y);
        store_pair(slot, hx, hy);
    }
    fence_proxy_async();
    __syncwarp();
    // Rows past the sequence end are zero fill: a box that starts beyond the
    // end is not stored; a ragged box is clipped by the tensor map bounds.
    if (lane == 0 && int64_t(t0) + warp * kRows < length) {
        tma_store_3d(&map_h, tile_b + int64_t(warp) * kRows * kSegFeatures, f0, t0 + warp * kRows,
                     static_cast<int32_t>(batch));
        tma_store_drain();
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
int64_t segment_tiles(int64_t batch, int64_t length, int64_t features) {
    return batch * ceil_div(features, kSegFeatures) * ceil_div(length, segment_length<T>());
}

template <typename T, bool kBroadcast>
int launch_segmented(const T *retention, const T *increment, const T *initial, T *states, int64_t batch,
                     int64_t length, int64_t features, void *workspace, cudaStream_t stream) {
    constexpr int kRows = segment_length<T>() / kSegWarps;
    const int64_t feature_tiles = ceil_div(features, kSegFeatures);
    const int64_t chains = batch * feature_tiles;
    const int64_t tiles = segment_tiles<T>(batch, length, features);
    const uint64_t es = sizeof(T);
    const uint64_t dims[3] = {static_cast<uint64_t>(features), static_cast<uint64_t>(length),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {features * es, length * features * es};
    const uint32_t box[3] = {kSegFeatures, kRows, 1};
    CUtensorMap map_a{}, map_b{}, map_h{};
    int rc;
    if (!kBroadcast) {
        rc = encode_tensor_map(&map_a, TensorMapType<T>::value, 3, retention, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc != KOEMI_OK) return rc;
    }
    rc = encode_tensor_map(&map_b, TensorMapType<T>::value, 3, increment, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != KOEMI_OK) return rc;
    rc = encode_tensor_map(&map_h, TensorMapType<T>::value, 3, states, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != KOEMI_OK) return rc;
    KOEMI_CUDA_TRY(cudaMemsetAsync(workspace, 0xFF, ScanWorkspace::bytes(tiles), stream));
    const size_t smem = segment_smem_bytes<T>();
    auto kernel = scan_segment_kernel<T, kBroadcast>;
    KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
    kernel<<<static_cast<unsigned>(tiles), kSegThreads, smem, stream>>>(
        map_a, map_b, map_h, retention, initial, length, features, chains, feature_tiles,
        static_cast<unsigned char *>(workspace), tiles, device_status_word());
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

// Whether the segmented kernel takes this call: 16-bit or fp32 rows that TMA
// can address (16-byte aligned bases and row pitch), a sequence longer than a
// decode step, and a caller workspace of koemi_dense_affine_scan_workspace().
template <typename T>
bool segmented_eligible(const void *retention, const void *increment, const void *states, int64_t batch,
                        int64_t length, int64_t features, bool broadcast, size_t workspace_bytes) {
    if (sizeof(T) == 8 || length <= 8) return false;
    if ((features * sizeof(T)) % 16 != 0 || !aligned(increment, 16) || !aligned(states, 16)) return false;
    if (!broadcast && !aligned(retention, 16)) return false;
    if (length >= (int64_t(1) << 31) || features >= (int64_t(1) << 31) || batch >= (int64_t(1) << 31)) {
        return false;
    }
    const int64_t tiles = segment_tiles<T>(batch, length, features);
    if (tiles >= (int64_t(1) << 31)) return false;
    return workspace_bytes >= ScanWorkspace::bytes(tiles);
}

template <typename T>
int scan_forward_typed(const void *retention, const void *increment, const void *initial,
                       void *states, int64_t batch, int64_t length, int64_t features,
                       bool broadcast, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    const T *r = static_cast<const T *>(retention);
    const T *i = static_cast<const T *>(increment);
    const T *h0 = static_cast<const T *>(initial);
    T *out = static_cast<T *>(states);
    if constexpr (sizeof(T) != 8) {
        if (workspace != nullptr &&
            segmented_eligible<T>(retention, increment, states, batch, length, features, broadcast,
                                  workspace_bytes)) {
            return broadcast
                       ? launch_segmented<T, true>(r, i, h0, out, batch, length, features, workspace, stream)
                       : launch_segmented<T, false>(r, i, h0, out, batch, length, features, workspace, stream);
        }
    }
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

extern "C" size_t koemi_dense_affine_scan_workspace(int64_t batch, int64_t length, int64_t features,
                                                    int dtype) {
    if (batch <= 0 || length <= 8 || features <= 0) return 0;
    int64_t tiles;
    switch (dtype) {
        case KOEMI_F32: tiles = segment_tiles<float>(batch, length, features); break;
        case KOEMI_F16:
        case KOEMI_BF16: tiles = segment_tiles<__half>(batch, length, features); break;
        default: return 0;
    }
    return tiles >= (int64_t(1) << 31) ? 0 : ScanWorkspace::bytes(tiles);
}

extern "C" int koemi_dense_affine_scan_forward(const void *retention, const void *increment,
                                               const void *initial, void *states, int64_t batch,
                                               int64_t length, int64_t features,
                                               int broadcast_retention, int dtype, void *workspace,
                                               size_t workspace_bytes, void *stream) {
    clear_error();
    int rc = check_scan_shapes(batch, length, features);
    if (rc != KOEMI_OK) return rc;
    if (batch == 0 || length == 0 || features == 0) return KOEMI_OK;
    if (retention == nullptr || increment == nullptr || states == nullptr) {
        return fail(KOEMI_ERR_INVALID, "retention, increment and states must be non-NULL");
    }
    // grid.y carries the batch in the chunked kernel, so batches above 65535
    // without a workspace take the per-lane kernel (scan_forward_typed).
    const bool bc = broadcast_retention != 0;
    cudaStream_t s = as_stream(stream);
    void *ws = workspace;
    const size_t wb = workspace_bytes;
    switch (dtype) {
        case KOEMI_F32: return scan_forward_typed<float>(retention, increment, initial, states, batch, length, features, bc, ws, wb, s);
        case KOEMI_F16: return scan_forward_typed<__half>(retention, increment, initial, states, batch, length, features, bc, ws, wb, s);
        case KOEMI_BF16: return scan_forward_typed<__nv_bfloat16>(retention, increment, initial, states, batch, length, features, bc, ws, wb, s);
        case KOEMI_F64: return scan_forward_typed<double>(retention, increment, initial, states, batch, length, features, bc, ws, wb, s);
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
// Four features per thread (16-byte loads and stores), grid (feature
// chunks, row blocks): the window path's [rows, 2 F] projections stream
// through once.
__global__ __launch_bounds__(256) void bounded_gates_vec_kernel(const float *__restrict__ projections,
                                                                const uint8_t *__restrict__ valid,
                                                                float *__restrict__ retention,
                                                                float *__restrict__ increment, int64_t rows,
                                                                int64_t features, float lo, float hi) {
    const int64_t f = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (f >= features) return;
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        float4 a = make_float4(1.0f, 1.0f, 1.0f, 1.0f), inc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (valid == nullptr || valid[row] != 0) {
            const float4 pa = __ldg(reinterpret_cast<const float4 *>(projections + row * 2 * features + f));
            const float4 pc = __ldg(reinterpret_cast<const float4 *>(projections + row * 2 * features + features + f));
            a = make_float4(lo + (hi - lo) * sigmoidf_(pa.x), lo + (hi - lo) * sigmoidf_(pa.y),
                            lo + (hi - lo) * sigmoidf_(pa.z), lo + (hi - lo) * sigmoidf_(pa.w));
            inc = make_float4((1.0f - a.x) * tanhf(pc.x), (1.0f - a.y) * tanhf(pc.y), (1.0f - a.z) * tanhf(pc.z),
                              (1.0f - a.w) * tanhf(pc.w));
        }
        *reinterpret_cast<float4 *>(retention + row * features + f) = a;
        *reinterpret_cast<float4 *>(increment + row * features + f) = inc;
    }
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
    if (features % 4 == 0 && aligned(projections, 16) && aligned(retention, 16) && aligned(increment, 16)) {
        const unsigned chunks = static_cast<unsigned>(ceil_div(features / 4, 256));
        const unsigned row_blocks = static_cast<unsigned>(rows < 65535 ? rows : 65535);
        bounded_gates_vec_kernel<<<dim3(chunks, row_blocks), 256, 0, as_stream(stream)>>>(
            projections, valid, retention, increment, rows, features, minimum_retention, maximum_retention);
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    }
    const int64_t total = rows * features;
    bounded_gates_kernel<<<static_cast<unsigned>(ceil_div(total, 256)), 256, 0, as_stream(stream)>>>(
        projections, valid, retention, increment, rows, features, minimum_retention,
        maximum_retention);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}
