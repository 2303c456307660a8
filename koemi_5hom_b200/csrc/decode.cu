// Decode-step kernels: one token per stream, state updated in place.
//
// The window path (model/network.py) rebuilds every ring with cat/slice each
// step, like the reference (memory.py:385-403,431-475). At decode the rings
// are circular instead: the local ring's oldest slot is one device-side head
// shared by all streams (every stream writes one entry per step), and each
// salient ring keeps its own head and count (entries are written only when a
// token is admitted). Reads are order-independent softmax sums, so they see
// exactly the reference's rings; the logical (oldest-first) order is restored
// only when the state is exported.
//
//  koemi_dense_decode_step      gate epilogue + padding masks + scan step
//                               (memory.py:22-26, network.py:307-310)
//  koemi_think_ring_decode_step local and salient reads, novelty, then the
//                               ring writes and admission (memory.py:307-361,
//                               405-455; network.py:327-358)
//  koemi_assoc_decode_step      feature softmaxes, confidence-weighted read of
//                               the rank-one memory and its decayed write
//                               (memory.py:82-95,248-255,279-287)
#include <cmath>

#include <type_traits>

#include "common.cuh"
#include "vec.cuh"

namespace koemi {
namespace {

// -------------------------------------------------------------- gates+scan
template <typename TP>
__global__ void decode_gates_kernel(const float *__restrict__ pre, const uint8_t *__restrict__ valid,
                                    float *__restrict__ working, TP *__restrict__ prior, TP *__restrict__ h_out,
                                    int64_t h_stride, TP *__restrict__ h_copy, int64_t batch, int64_t features,
                                    float lo, float hi) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= batch * features) return;
    const int64_t row = i / features;
    const int64_t f = i - row * features;
    const bool ok = valid == nullptr || valid[row] != 0;
    float a = 1.0f, b = 0.0f;
    if (ok) {
        a = lo + (hi - lo) * sigmoidf_(pre[row * 2 * features + f]);
        b = (1.0f - a) * tanhf(pre[row * 2 * features + features + f]);
    }
    const float previous = working[i];
    if (prior != nullptr) prior[i] = from_acc<TP>(previous);
    const float h = a * previous + b;
    working[i] = h;
    if (h_out != nullptr) h_out[row * h_stride + f] = from_acc<TP>(h);
    if (h_copy != nullptr) h_copy[i] = from_acc<TP>(h);
}

// ---------------------------------------------------------------- rings
constexpr int kRingThreads = 256;
constexpr int kRingWarps = kRingThreads / 32;

struct RingArgs {
    const float *queries;
    int64_t query_stride;
    const float *entries;  // [B, 2d]: key | value of the new entry (unmasked, fp32)
    int64_t entry_stride;
    const uint8_t *valid;
    const float *surprise;
    float threshold;
    void *local_keys;      // ring element type TR
    void *local_values;
    uint8_t *local_valid;
    const int64_t *local_head;
    void *salient_keys;
    void *salient_values;
    uint8_t *salient_valid;
    int32_t *salient_head;
    int32_t *salient_count;
    void *local_out;
    void *salient_out;
    int64_t out_stride;
    float *novelty_out;
    uint8_t *admission_out;
    int64_t batch;
    int64_t width;
    int64_t local_slots;
    int64_t salient_slots;
};

__device__ __forceinline__ float block_reduce(float v, float *scratch, bool take_max) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = take_max ? warp_max(v) : warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = scratch[0];
    for (int w = 1; w < kRingWarps; ++w) r = take_max ? fmaxf(r, scratch[w]) : r + scratch[w];
    return r;
}

// 16-byte packets of ring rows: 4 fp32 or 8 bf16 elements.
template <typename TR>
struct RingPacket;
template <>
struct RingPacket<float> {
    static constexpr int kWidth = 4;
    __device__ static void load(const float *p, float (&v)[4]) {
        const float4 x = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    }
    __device__ static void store(float *p, const float (&v)[4]) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <>
struct RingPacket<__nv_bfloat16> {
    static constexpr int kWidth = 8;
    __device__ static void load(const __nv_bfloat16 *p, float (&v)[8]) {
        const uint4 x = __ldg(reinterpret_cast<const uint4 *>(p));
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    __device__ static void store(__nv_bfloat16 *p, const float (&v)[8]) {
        uint4 x;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&x);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4 *>(p) = x;
    }
};

// blockIdx.y == 0: local ring, 1: salient ring. Shared memory: q[width],
// scores[slots], cosines[slots], reduction scratch.
template <typename TR, typename TO>
__global__ __launch_bounds__(kRingThreads) void ring_decode_kernel(RingArgs a) {
    pdl_trigger();
    pdl_wait();
    using P = RingPacket<TR>;
    constexpr int W = P::kWidth;
    extern __shared__ float shared[];
    const bool local = blockIdx.y == 0;
    const int64_t b = blockIdx.x;
    const int64_t d = a.width;
    const int64_t slots = local ? a.local_slots : a.salient_slots;
    float *q = shared;
    float *score = q + d;
    float *cosine = score + slots;
    float *scratch = cosine + slots;
    __shared__ int32_t write_slot;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *query = a.queries + b * a.query_stride;
    float qq = 0.0f;
    if ((reinterpret_cast<uintptr_t>(query) & 15) == 0) {  // d % 4 == 0 (the host checks it)
        for (int64_t c = threadIdx.x; c < d / 4; c += kRingThreads) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(query) + c);
            reinterpret_cast<float4 *>(q)[c] = v;
            qq += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int64_t c = threadIdx.x; c < d; c += kRingThreads) {
            const float v = query[c];
            q[c] = v;
            qq += v * v;
        }
    }
    const float q_norm = sqrtf(block_reduce(qq, scratch, false));
    TR *keys = static_cast<TR *>(local ? a.local_keys : a.salient_keys) + b * slots * d;
    TR *values = static_cast<TR *>(local ? a.local_values : a.salient_values) + b * slots * d;
    const uint8_t *flags = (local ? a.local_valid : a.salient_valid) + b * slots;
    const float scale = rsqrtf(static_cast<float>(d));
    const int64_t packets = d / W;  // the host requires width % W == 0

    // pass 1: one warp per slot, dot(q, k) and |k|^2 over 16-byte packets
    for (int64_t s = warp; s < slots; s += kRingWarps) {
        if (!flags[s]) {
            if (lane == 0) {
                score[s] = -INFINITY;
                cosine[s] = -INFINITY;
            }
            continue;
        }
        const TR *row = keys + s * d;
        float dot = 0.0f, kk = 0.0f;
#pragma unroll 8
        for (int64_t c = lane; c < packets; c += 32) {
            float k[W], qv[W];
            P::load(row + c * W, k);
#pragma unroll
            for (int e = 0; e < W; e += 4) {  // the query packet as 16-byte shared loads (q is 16-byte aligned)
                *reinterpret_cast<float4 *>(qv + e) = *reinterpret_cast<const float4 *>(q + c * W + e);
            }
#pragma unroll
            for (int e = 0; e < W; ++e) {
                dot = fmaf(k[e], qv[e], dot);
                kk = fmaf(k[e], k[e], kk);
            }
        }
        dot = warp_sum(dot);
        kk = warp_sum(kk);
        if (lane == 0) {
            score[s] = dot * scale;
            cosine[s] = dot / (fmaxf(sqrtf(kk), 1e-12f) * fmaxf(q_norm, 1e-12f));
        }
    }
    __syncthreads();
    float m = -INFINITY, best_cos = -INFINITY;
    for (int64_t s = threadIdx.x; s < slots; s += kRingThreads) {
        m = fmaxf(m, score[s]);
        best_cos = fmaxf(best_cos, cosine[s]);
    }
    m = block_reduce(m, scratch, true);
    best_cos = block_reduce(best_cos, scratch, true);
    const bool any = m != -INFINITY;
    float total = 0.0f;
    for (int64_t s = threadIdx.x; s < slots; s += kRingThreads) {
        const float w = any && score[s] != -INFINITY ? expf(score[s] - m) : 0.0f;
        score[s] = w;
        total += w;
    }
    total = block_reduce(total, scratch, false);
    const float inv_total = any ? 1.0f / total : 0.0f;

    // the slots with a nonzero weight, ascending (warp ballots; the cosine
    // array is free once best_cos is reduced)
    int32_t *live = reinterpret_cast<int32_t *>(cosine);
    __shared__ int32_t live_count;
    if (warp == 0) {
        int32_t base = 0;
        for (int64_t s0 = 0; s0 < slots; s0 += 32) {
            const int64_t s = s0 + lane;
            const bool nonzero = s < slots && score[s] != 0.0f;
            const unsigned mask = __ballot_sync(0xffffffffu, nonzero);
            if (nonzero) live[base + __popc(mask & ((1u << lane) - 1u))] = static_cast<int32_t>(s);
            base += __popc(mask);
        }
        if (lane == 0) live_count = base;
    }
    __syncthreads();
    const int32_t n_live = live_count;

    // pass 2: each thread owns packets of columns and sums the weighted values
    // of the live slots in ascending order, kValueUnroll loads in flight
    constexpr int kValueUnroll = 8;
    TO *out = static_cast<TO *>(local ? a.local_out : a.salient_out) + b * a.out_stride;
    for (int64_t c = threadIdx.x; c < packets; c += kRingThreads) {
        float acc[W];
#pragma unroll
        for (int e = 0; e < W; ++e) acc[e] = 0.0f;
        int32_t i = 0;
        for (; i + kValueUnroll <= n_live; i += kValueUnroll) {
            float v[kValueUnroll][W], w[kValueUnroll];
#pragma unroll
            for (int u = 0; u < kValueUnroll; ++u) {
                const int32_t slot = live[i + u];
                w[u] = score[slot];
                P::load(values + static_cast<int64_t>(slot) * d + c * W, v[u]);
            }
#pragma unroll
            for (int u = 0; u < kValueUnroll; ++u) {
#pragma unroll
                for (int e = 0; e < W; ++e) acc[e] = fmaf(w[u], v[u][e], acc[e]);
            }
        }
        for (; i < n_live; ++i) {
            const int32_t slot = live[i];
            const float w = score[slot];
            float v[W];
            P::load(values + static_cast<int64_t>(slot) * d + c * W, v);
#pragma unroll
            for (int e = 0; e < W; ++e) acc[e] = fmaf(w, v[e], acc[e]);
        }
#pragma unroll
        for (int e = 0; e < W; ++e) out[c * W + e] = from_acc<TO>(acc[e] * inv_total);
    }
    const bool token_valid = a.valid == nullptr || a.valid[b] != 0;
    if (local && threadIdx.x == 0 && a.novelty_out != nullptr) {
        a.novelty_out[b] = any ? fminf(fmaxf(1.0f - best_cos, 0.0f), 1.0f) : 1.0f;
    }

    // writes, after every read of the slot being replaced
    if (threadIdx.x == 0) {
        if (local) {
            write_slot = static_cast<int32_t>(*a.local_head);
        } else {
            const bool admitted = token_valid && a.surprise[b] > a.threshold;
            if (a.admission_out != nullptr) a.admission_out[b] = admitted;
            write_slot = -1;
            if (admitted) {
                const int32_t head = a.salient_head[b];
                const int32_t count = a.salient_count[b];
                if (count < slots) {
                    write_slot = static_cast<int32_t>((head + count) % slots);
                    a.salient_count[b] = count + 1;
                } else {
                    write_slot = head;  // the ring is full: the oldest admitted entry leaves
                    a.salient_head[b] = static_cast<int32_t>((head + 1) % slots);
                }
            }
        }
    }
    __syncthreads();
    const int32_t slot = write_slot;
    if (slot < 0) return;
    TR *key_dst = keys + slot * d;
    TR *value_dst = values + slot * d;
    const float *entry = a.entries + b * a.entry_stride;
    for (int64_t c = threadIdx.x; c < packets; c += kRingThreads) {
        float k[W], v[W];
#pragma unroll
        for (int e = 0; e < W; ++e) {
            k[e] = token_valid ? entry[c * W + e] : 0.0f;
            v[e] = token_valid ? entry[d + c * W + e] : 0.0f;
        }
        P::store(key_dst + c * W, k);
        P::store(value_dst + c * W, v);
    }
    if (threadIdx.x == 0) (local ? a.local_valid : a.salient_valid)[b * slots + slot] = local ? token_valid : 1;
}

// The same step with each (stream, ring) split over a thread-block cluster of
// gridDim.z CTAs, for batches too small to fill the GPU with one CTA per
// ring: CTA p scores slots [p S / P, (p + 1) S / P) and sums their weighted
// values into a partial row; the softmax maximum, the best cosine, the
// weight totals and the partial rows are combined across the cluster through
// distributed shared memory (in CTA order, so the result is deterministic);
// CTA p writes output columns [p d / P, (p + 1) d / P). The ring write and the
// admission bookkeeping are done by the cluster's first CTA after every CTA
// has read the ring.
__device__ __forceinline__ float ld_dsmem_f32(const float *local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename TR, typename TO>
__global__ __launch_bounds__(kRingThreads) void ring_decode_split_kernel(RingArgs a) {
    pdl_trigger();
    pdl_wait();
    using P = RingPacket<TR>;
    constexpr int W = P::kWidth;
    extern __shared__ float shared[];
    const bool local = blockIdx.y == 0;
    const int64_t b = blockIdx.x;
    const int64_t d = a.width;
    const int64_t slots = local ? a.local_slots : a.salient_slots;
    const uint32_t parts = gridDim.z;
    const uint32_t part = blockIdx.z;  // == rank in the cluster (cluster dims (1, 1, parts))
    const int64_t slot_begin = slots * part / parts;
    const int64_t slot_end = slots * (part + 1) / parts;
    const int64_t own = slot_end - slot_begin;
    float *q = shared;                 // [d]
    float *partial = q + d;            // [d] this CTA's weighted value sums
    float *score = partial + d;        // [own]
    float *cosine = score + own;       // [own]
    float *scratch = cosine + own;     // [kRingWarps]
    __shared__ float cl_max, cl_cos, cl_total;
    __shared__ int32_t write_slot;
    __shared__ int32_t live_count;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *query = a.queries + b * a.query_stride;
    float qq = 0.0f;
    if ((reinterpret_cast<uintptr_t>(query) & 15) == 0) {  // d % 4 == 0 (the host checks it)
        for (int64_t c = threadIdx.x; c < d / 4; c += kRingThreads) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(query) + c);
            reinterpret_cast<float4 *>(q)[c] = v;
            qq += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int64_t c = threadIdx.x; c < d; c += kRingThreads) {
            const float v = query[c];
            q[c] = v;
            qq += v * v;
        }
    }
    const float q_norm = sqrtf(block_reduce(qq, scratch, false));
    TR *keys = static_cast<TR *>(local ? a.local_keys : a.salient_keys) + b * slots * d;
    TR *values = static_cast<TR *>(local ? a.local_values : a.salient_values) + b * slots * d;
    const uint8_t *flags = (local ? a.local_valid : a.salient_valid) + b * slots;
    const float scale = rsqrtf(static_cast<float>(d));
    const int64_t packets = d / W;

    for (int64_t i = warp; i < own; i += kRingWarps) {
        const int64_t s = slot_begin + i;
        if (!flags[s]) {
            if (lane == 0) {
                score[i] = -INFINITY;
                cosine[i] = -INFINITY;
            }
            continue;
        }
        const TR *row = keys + s * d;
        float dot = 0.0f, kk = 0.0f;
#pragma unroll 8
        for (int64_t c = lane; c < packets; c += 32) {
            float k[W], qv[W];
            P::load(row + c * W, k);
#pragma unroll
            for (int e = 0; e < W; e += 4) {  // the query packet as 16-byte shared loads (q is 16-byte aligned)
                *reinterpret_cast<float4 *>(qv + e) = *reinterpret_cast<const float4 *>(q + c * W + e);
            }
#pragma unroll
            for (int e = 0; e < W; ++e) {
                dot = fmaf(k[e], qv[e], dot);
                kk = fmaf(k[e], k[e], kk);
            }
        }
        dot = warp_sum(dot);
        kk = warp_sum(kk);
        if (lane == 0) {
            score[i] = dot * scale;
            cosine[i] = dot / (fmaxf(sqrtf(kk), 1e-12f) * fmaxf(q_norm, 1e-12f));
        }
    }
    __syncthreads();
    float m = -INFINITY, best = -INFINITY;
    for (int64_t i = threadIdx.x; i < own; i += kRingThreads) {
        m = fmaxf(m, score[i]);
        best = fmaxf(best, cosine[i]);
    }
    m = block_reduce(m, scratch, true);
    best = block_reduce(best, scratch, true);
    if (threadIdx.x == 0) {
        cl_max = m;
        cl_cos = best;
    }
    cluster_barrier();  // 1: every CTA's maximum and best cosine are visible
    m = -INFINITY;
    best = -INFINITY;
    for (uint32_t r = 0; r < parts; ++r) {
        m = fmaxf(m, ld_dsmem_f32(&cl_max, r));
        best = fmaxf(best, ld_dsmem_f32(&cl_cos, r));
    }
    const bool any = m != -INFINITY;
    float total = 0.0f;
    for (int64_t i = threadIdx.x; i < own; i += kRingThreads) {
        const float w = any && score[i] != -INFINITY ? expf(score[i] - m) : 0.0f;
        score[i] = w;
        total += w;
    }
    total = block_reduce(total, scratch, false);
    if (threadIdx.x == 0) cl_total = total;
    int32_t *live = reinterpret_cast<int32_t *>(cosine);
    if (warp == 0) {
        int32_t base = 0;
        for (int64_t i0 = 0; i0 < own; i0 += 32) {
            const int64_t i = i0 + lane;
            const bool nonzero = i < own && score[i] != 0.0f;
            const unsigned mask = __ballot_sync(0xffffffffu, nonzero);
            if (nonzero) live[base + __popc(mask & ((1u << lane) - 1u))] = static_cast<int32_t>(i);
            base += __popc(mask);
        }
        if (lane == 0) live_count = base;
    }
    __syncthreads();
    const int32_t n_live = live_count;
    constexpr int kValueUnroll = 8;
    for (int64_t c = threadIdx.x; c < packets; c += kRingThreads) {
        float acc[W];
#pragma unroll
        for (int e = 0; e < W; ++e) acc[e] = 0.0f;
        int32_t i = 0;
        for (; i + kValueUnroll <= n_live; i += kValueUnroll) {
            float v[kValueUnroll][W], w[kValueUnroll];
#pragma unroll
            for (int u = 0; u < kValueUnroll; ++u) {
                const int32_t li = live[i + u];
                w[u] = score[li];
                P::load(values + (slot_begin + li) * d + c * W, v[u]);
            }
#pragma unroll
            for (int u = 0; u < kValueUnroll; ++u) {
#pragma unroll
                for (int e = 0; e < W; ++e) acc[e] = fmaf(w[u], v[u][e], acc[e]);
            }
        }
        for (; i < n_live; ++i) {
            const int32_t li = live[i];
            const float w = score[li];
            float v[W];
            P::load(values + (slot_begin + li) * d + c * W, v);
#pragma unroll
            for (int e = 0; e < W; ++e) acc[e] = fmaf(w, v[e], acc[e]);
        }
#pragma unroll
        for (int e = 0; e < W; ++e) partial[c * W + e] = acc[e];
    }
    cluster_barrier();  // 2: partial rows and totals are visible; every ring read is done
    float all_total = 0.0f;
    for (uint32_t r = 0; r < parts; ++r) all_total += ld_dsmem_f32(&cl_total, r);
    const float inv_total = any ? 1.0f / all_total : 0.0f;
    TO *out = static_cast<TO *>(local ? a.local_out : a.salient_out) + b * a.out_stride;
    const int64_t col_begin = d * part / parts, col_end = d * (part + 1) / parts;
    for (int64_t c = col_begin + threadIdx.x; c < col_end; c += kRingThreads) {
        float sum = 0.0f;
        for (uint32_t r = 0; r < parts; ++r) sum += ld_dsmem_f32(partial + c, r);
        out[c] = from_acc<TO>(sum * inv_total);
    }
    const bool token_valid = a.valid == nullptr || a.valid[b] != 0;
    if (part == 0) {
        if (local && threadIdx.x == 0 && a.novelty_out != nullptr) {
            a.novelty_out[b] = any ? fminf(fmaxf(1.0f - best, 0.0f), 1.0f) : 1.0f;
        }
        if (threadIdx.x == 0) {
            if (local) {
                write_slot = static_cast<int32_t>(*a.local_head);
            } else {
                const bool admitted = token_valid && a.surprise[b] > a.threshold;
                if (a.admission_out != nullptr) a.admission_out[b] = admitted;
                write_slot = -1;
                if (admitted) {
                    const int32_t head = a.salient_head[b];
                    const int32_t count = a.salient_count[b];
                    if (count < slots) {
                        write_slot = static_cast<int32_t>((head + count) % slots);
                        a.salient_count[b] = count + 1;
                    } else {
                        write_slot = head;
                        a.salient_head[b] = static_cast<int32_t>((head + 1) % slots);
                    }
                }
            }
        }
        __syncthreads();
        const int32_t slot = write_slot;
        if (slot >= 0) {
            TR *key_dst = keys + slot * d;
            TR *value_dst = values + slot * d;
            const float *entry = a.entries + b * a.entry_stride;
            for (int64_t c = threadIdx.x; c < packets; c += kRingThreads) {
                float k[W], v[W];
#pragma unroll
                for (int e = 0; e < W; ++e) {
                    k[e] = token_valid ? entry[c * W + e] : 0.0f;
                    v[e] = token_valid ? entry[d + c * W + e] : 0.0f;
                }
                P::store(key_dst + c * W, k);
                P::store(value_dst + c * W, v);
            }
            if (threadIdx.x == 0) {
                (local ? a.local_valid : a.salient_valid)[b * slots + slot] = local ? token_valid : 1;
            }
        }
    }
    cluster_barrier();  // 3: no CTA leaves while another still reads its shared memory
}

// ----------------------------------------------------------- associative
constexpr int kAssocThreads = 512;

// Feature logits of the key (which = 0) and query (which = 1) rows of one
// stream: W [m, d] (type TW) times the row rounded to TW (the numerics of a
// TW x TW tensor-core projection with fp32 accumulation), plus bias. One warp
// per (which, feature) task; d % 8 == 0 and 16-byte aligned weight rows use
// 8-wide packets, 8-byte aligned fp32 projection rows.
template <typename TW>
__device__ void assoc_feature_logits(const float *__restrict__ proj, const TW *__restrict__ weight,
                                     const TW *__restrict__ bias, float *__restrict__ logits, int64_t d,
                                     int64_t m, bool vector) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t task = warp; task < 2 * m; task += kAssocThreads / 32) {
        const int64_t which = task / m, j = task - which * m;
        const float *x = proj + which * d;
        const TW *w = weight + j * d;
        float acc = 0.0f;
        if (vector) {
#pragma unroll 8
            for (int64_t c = lane * 8; c < d; c += 256) {
                float wv[8];
                if constexpr (std::is_same_v<TW, float>) {
                    const float4 lo = __ldg(reinterpret_cast<const float4 *>(w + c));
                    const float4 hi = __ldg(reinterpret_cast<const float4 *>(w + c + 4));
                    wv[0] = lo.x; wv[1] = lo.y; wv[2] = lo.z; wv[3] = lo.w;
                    wv[4] = hi.x; wv[5] = hi.y; wv[6] = hi.z; wv[7] = hi.w;
                } else {
                    unpack(__ldg(reinterpret_cast<const uint4 *>(w + c)), wv, TW{});
                }
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float2 xv = *reinterpret_cast<const float2 *>(x + c + e);
                    acc = fmaf(to_acc(from_acc<TW>(xv.x)), wv[e], acc);
                    acc = fmaf(to_acc(from_acc<TW>(xv.y)), wv[e + 1], acc);
                }
            }
        } else {
            for (int64_t c = lane; c < d; c += 32) acc = fmaf(to_acc(from_acc<TW>(x[c])), to_acc(w[c]), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) logits[task] = acc + (bias != nullptr ? to_acc(bias[j]) : 0.0f);
    }
}

// The same logits with the key and query rows staged in shared memory first
// (rounded to TW) and each warp's weight packets loaded eight at a time
// before any is used, so a feature costs one L2 round trip per 2048 columns
// instead of one per 256. Warp w takes features w, w + 16, ... for both rows
// (they share the weight row). Per-lane summation order is that of
// assoc_feature_logits, so the results are identical. Needs d % 8 == 0,
// 16-byte aligned weight rows and 8-byte aligned projection rows.
template <typename TW>
__device__ void assoc_feature_logits_staged(const float *__restrict__ proj, const TW *__restrict__ weight,
                                            const TW *__restrict__ bias, float *__restrict__ logits,
                                            float *__restrict__ xs, int64_t d, int64_t m) {
    for (int64_t c = 2 * static_cast<int64_t>(threadIdx.x); c < 2 * d; c += 2 * kAssocThreads) {
        const float2 v = *reinterpret_cast<const float2 *>(proj + c);
        xs[c] = to_acc(from_acc<TW>(v.x));
        xs[c + 1] = to_acc(from_acc<TW>(v.y));
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kGroup = 8;
    constexpr int kWords = std::is_same_v<TW, float> ? 2 : 1;  // 16-byte words per 8 weights
    for (int64_t j = warp; j < m; j += kAssocThreads / 32) {
        const TW *w = weight + j * d;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int64_t g0 = 0; g0 < d; g0 += 256 * kGroup) {
            uint4 raw[kGroup][kWords];
#pragma unroll
            for (int i = 0; i < kGroup; ++i) {
                const int64_t c = g0 + lane * 8 + 256 * i;
                if (c < d) {
#pragma unroll
                    for (int h = 0; h < kWords; ++h) raw[i][h] = __ldg(reinterpret_cast<const uint4 *>(w + c) + h);
                }
            }
#pragma unroll
            for (int i = 0; i < kGroup; ++i) {
                const int64_t c = g0 + lane * 8 + 256 * i;
                if (c >= d) continue;
                float wv[8];
                if constexpr (std::is_same_v<TW, float>) {
                    unpack(raw[i][0], *reinterpret_cast<float(*)[4]>(wv), float{});
                    unpack(raw[i][1], *reinterpret_cast<float(*)[4]>(wv + 4), float{});
                } else {
                    unpack(raw[i][0], wv, TW{});
                }
                // the staged rows read as 16-byte packets (c is a multiple of
                // 8 and d of 8): two loads per row instead of eight
                // bank-conflicted scalar ones; the FMAs keep their order
                float xk[8], xq[8];
                *reinterpret_cast<float4 *>(xk) = reinterpret_cast<const float4 *>(xs + c)[0];
                *reinterpret_cast<float4 *>(xk + 4) = reinterpret_cast<const float4 *>(xs + c)[1];
                *reinterpret_cast<float4 *>(xq) = reinterpret_cast<const float4 *>(xs + d + c)[0];
                *reinterpret_cast<float4 *>(xq + 4) = reinterpret_cast<const float4 *>(xs + d + c)[1];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    acc0 = fmaf(xk[e], wv[e], acc0);
                    acc1 = fmaf(xq[e], wv[e], acc1);
                }
            }
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        if (lane == 0) {
            const float bj = bias != nullptr ? to_acc(bias[j]) : 0.0f;
            logits[j] = acc0 + bj;
            logits[m + j] = acc1 + bj;
        }
    }
}

// gridDim.y CTAs per stream (one thread-block cluster) split the d memory
// rows; each recomputes the features. The memory row i (m features) is read
// as m/4 float4 packets by m/4 adjacent threads, which combine their partial
// dot products with the query features by shuffles; the decayed write goes
// back in place. The normaliser is updated by the cluster's first CTA after
// a cluster barrier, once every CTA has read it. feature_logits ([2, batch,
// m]) may be NULL, in which case the logits come from feature_weight /
// feature_bias in the kernel.
template <typename TO, typename TW>
__global__ __launch_bounds__(kAssocThreads) void assoc_decode_kernel(
    const float *__restrict__ projections, int64_t proj_stride, const float *__restrict__ feature_logits,
    const TW *__restrict__ feature_weight, const TW *__restrict__ feature_bias, bool vector_features,
    bool stage_features, const float *__restrict__ surprise, const uint8_t *__restrict__ valid,
    float *__restrict__ basis,
    float *__restrict__ normalizer, TO *__restrict__ read_out, int64_t read_stride, int64_t batch, int64_t d,
    int64_t m) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float shared[];
    float *f = shared;       // [m] write features
    float *qf = shared + m;  // [m] query features
    float *own_logits = shared + 2 * m;  // [2, m] when computed here
    float *staged_rows = shared + 4 * m;  // [2, d] when staging (stage_features)
    __shared__ float s_decay, s_write, s_den;
    const int64_t b = blockIdx.x;
    const float *proj = projections + b * proj_stride;
    if (feature_logits == nullptr) {
        if (stage_features) {
            assoc_feature_logits_staged(proj, feature_weight, feature_bias, own_logits, staged_rows, d, m);
        } else {
            assoc_feature_logits(proj, feature_weight, feature_bias, own_logits, d, m, vector_features);
        }
        __syncthreads();
    }
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        for (int which = 0; which < 2; ++which) {
            const float *logits = feature_logits != nullptr ? feature_logits + (which * batch + b) * m
                                                            : own_logits + which * m;
            float mx = -INFINITY;
            for (int64_t j = lane; j < m; j += 32) mx = fmaxf(mx, logits[j]);
            mx = warp_max(mx);
            float sum = 0.0f;
            for (int64_t j = lane; j < m; j += 32) sum += expf(logits[j] - mx);
            sum = warp_sum(sum);
            float *dst = which == 0 ? f : qf;
            for (int64_t j = lane; j < m; j += 32) dst[j] = expf(logits[j] - mx) / sum;
        }
        __syncwarp();
        // den = normaliser . query features, one feature per lane (a serial
        // loop of dependent-latency loads in one thread would dominate here)
        float den = 0.0f;
        for (int64_t j = lane; j < m; j += 32) den += normalizer[b * m + j] * qf[j];
        den = warp_sum(den);
        if (lane == 0) {
            const bool ok = valid == nullptr || valid[b] != 0;
            const float lo = 1.0f / 4096.0f, hi = 1.0f - 1.0f / 4096.0f;
            const float decay = lo + (hi - lo) * sigmoidf_(proj[3 * d]);
            const float s = surprise != nullptr ? fminf(fmaxf(surprise[b], 0.0f), 1.0f) : 0.0f;
            const float write = sigmoidf_(proj[3 * d + 1]) * (0.25f + 0.75f * s);
            s_decay = ok ? decay : 1.0f;
            s_write = ok ? write : 0.0f;
            s_den = den;
        }
    }
    __syncthreads();
    const float decay = s_decay, write = s_write, den = s_den;
    const float reg = den + 1.0f / 256.0f;
    const float confidence = den / reg;
    float *rows = basis + b * d * m;
    const int64_t row_begin = d * blockIdx.y / gridDim.y;
    const int64_t row_end = d * (blockIdx.y + 1) / gridDim.y;
    if (m % 4 == 0 && m <= 128 && (kAssocThreads % (m / 4)) == 0 && 32 % (m / 4) == 0) {
        const int parts = static_cast<int>(m / 4);
        const int part = static_cast<int>(threadIdx.x) % parts;
        const int64_t rows_per_pass = kAssocThreads / parts;
        const float4 qv = reinterpret_cast<const float4 *>(qf)[part];
        const float4 fv = reinterpret_cast<const float4 *>(f)[part];
        // uniform trip count: every lane reaches the shuffles; kPasses rows
        // per thread are loaded before any is used, to keep loads in flight
        constexpr int kPasses = 4;
        for (int64_t base = row_begin; base < row_end; base += kPasses * rows_per_pass) {
            float4 x[kPasses];
            float value[kPasses];
#pragma unroll
            for (int u = 0; u < kPasses; ++u) {
                const int64_t i = base + u * rows_per_pass + threadIdx.x / parts;
                const bool live = i < row_end;
                x[u] = live ? *(reinterpret_cast<const float4 *>(rows + i * m) + part) : make_float4(0.f, 0.f, 0.f, 0.f);
                value[u] = live ? proj[2 * d + i] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kPasses; ++u) {
                const int64_t i = base + u * rows_per_pass + threadIdx.x / parts;
                float num = x[u].x * qv.x + x[u].y * qv.y + x[u].z * qv.z + x[u].w * qv.w;
                for (int o = 1; o < parts; o <<= 1) num += __shfl_xor_sync(0xffffffffu, num, o);
                if (i >= row_end) continue;
                const float v = write * tanhf(value[u]);
                float4 y;
                y.x = decay * x[u].x + v * fv.x;
                y.y = decay * x[u].y + v * fv.y;
                y.z = decay * x[u].z + v * fv.z;
                y.w = decay * x[u].w + v * fv.w;
                *(reinterpret_cast<float4 *>(rows + i * m) + part) = y;
                if (part == 0) read_out[b * read_stride + i] = from_acc<TO>(confidence * num / reg);
            }
        }
    } else {
        for (int64_t i = row_begin + threadIdx.x; i < row_end; i += kAssocThreads) {
            float *row = rows + i * m;
            const float v = tanhf(proj[2 * d + i]);
            float num = 0.0f;
            for (int64_t j = 0; j < m; ++j) {
                const float x = row[j];
                num += x * qf[j];
                row[j] = decay * x + write * v * f[j];
            }
            read_out[b * read_stride + i] = from_acc<TO>(confidence * num / reg);
        }
    }
    // every CTA of the stream has read the normaliser (den) before this
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (blockIdx.y == 0 && threadIdx.x < m) {
        const int64_t j = threadIdx.x;
        normalizer[b * m + j] = decay * normalizer[b * m + j] + write * f[j];
    }
}

// The same step for kM = 16 features with the key/query rows staged (the
// config-5 shape), latency-ordered: every global load that does not depend
// on another -- this warp's feature-weight row, the normaliser, the decay /
// write / surprise / validity scalars, the first pass of basis rows and the
// staged key/query rows -- is issued at entry, so a CTA waits for one memory
// round trip before it computes instead of one per phase. Arithmetic and its
// order are those of assoc_decode_kernel (bit-identical results).
template <typename TO, typename TW, int kM>
__global__ __launch_bounds__(kAssocThreads, 2) void assoc_decode_prefetch_kernel(
    const float *__restrict__ projections, int64_t proj_stride, const TW *__restrict__ feature_weight,
    const TW *__restrict__ feature_bias, const float *__restrict__ surprise, const uint8_t *__restrict__ valid,
    float *__restrict__ basis, float *__restrict__ normalizer, TO *__restrict__ read_out, int64_t read_stride,
    int64_t d) {
    static_assert(kM % 4 == 0 && kM <= kAssocThreads / 32 && 32 % (kM / 4) == 0, "feature count");
    pdl_trigger();
    pdl_wait();
    extern __shared__ float shared[];
    float *f = shared;                   // [m] write features
    float *qf = shared + kM;             // [m] query features
    float *own_logits = shared + 2 * kM; // [2, m]
    float *xs = shared + 4 * kM;         // [2, d] staged key | query rows, rounded to TW
    __shared__ float s_decay, s_write, s_den;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.x;
    const float *proj = projections + b * proj_stride;
    float *rows = basis + b * d * kM;
    const int64_t row_begin = d * blockIdx.y / gridDim.y;
    const int64_t row_end = d * (blockIdx.y + 1) / gridDim.y;
    constexpr int kParts = kM / 4;
    constexpr int kPasses = 4;
    constexpr int64_t kRowsPerPass = kAssocThreads / kParts;
    const int part = static_cast<int>(threadIdx.x) % kParts;

    // ---- every independent load, issued before any is used
    float pre_decay = 0.0f, pre_write = 0.0f, s_value = 0.0f;
    bool ok = true;
    if (threadIdx.x == 0) {
        pre_decay = proj[3 * d];
        pre_write = proj[3 * d + 1];
        s_value = surprise != nullptr ? surprise[b] : 0.0f;
        ok = valid == nullptr || valid[b] != 0;
    }
    const float nrm = threadIdx.x < kM ? normalizer[b * kM + threadIdx.x] : 0.0f;
    constexpr int kGroup = 8;
    constexpr int kWords = std::is_same_v<TW, float> ? 2 : 1;
    uint4 wraw[kGroup][kWords];
    const TW *wrow = feature_weight + static_cast<int64_t>(warp < kM ? warp : 0) * d;
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
        const int64_t c = lane * 8 + 256 * i;
        if (warp < kM && c < d) {
#pragma unroll
            for (int h = 0; h < kWords; ++h) wraw[i][h] = __ldg(reinterpret_cast<const uint4 *>(wrow + c) + h);
        }
    }
    float4 x0[kPasses];
    float value0[kPasses];
#pragma unroll
    for (int u = 0; u < kPasses; ++u) {
        const int64_t i = row_begin + u * kRowsPerPass + threadIdx.x / kParts;
        const bool live = i < row_end;
        x0[u] = live ? *(reinterpret_cast<const float4 *>(rows + i * kM) + part) : make_float4(0.f, 0.f, 0.f, 0.f);
        value0[u] = live ? proj[2 * d + i] : 0.0f;
    }
    for (int64_t c = 2 * static_cast<int64_t>(threadIdx.x); c < 2 * d; c += 2 * kAssocThreads) {
        const float2 v = *reinterpret_cast<const float2 *>(proj + c);
        xs[c] = to_acc(from_acc<TW>(v.x));
        xs[c + 1] = to_acc(from_acc<TW>(v.y));
    }
    __syncthreads();

    // ---- feature logits: warp j, both rows, summed as assoc_feature_logits_staged does
    if (warp < kM) {
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int64_t g0 = 0; g0 < d; g0 += 256 * kGroup) {
            if (g0 > 0) {  // rows wider than 2048: later groups load here
#pragma unroll
                for (int i = 0; i < kGroup; ++i) {
                    const int64_t c = g0 + lane * 8 + 256 * i;
                    if (c < d) {
#pragma unroll
                        for (int h = 0; h < kWords; ++h) wraw[i][h] = __ldg(reinterpret_cast<const uint4 *>(wrow + c) + h);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kGroup; ++i) {
                const int64_t c = g0 + lane * 8 + 256 * i;
                if (c >= d) continue;
                float wv[8];
                if constexpr (std::is_same_v<TW, float>) {
                    unpack(wraw[i][0], *reinterpret_cast<float(*)[4]>(wv), float{});
                    unpack(wraw[i][1], *reinterpret_cast<float(*)[4]>(wv + 4), float{});
                } else {
                    unpack(wraw[i][0], wv, TW{});
                }
                // the staged rows read as 16-byte packets (c is a multiple of
                // 8 and d of 8): two loads per row instead of eight
                // bank-conflicted scalar ones; the FMAs keep their order
                float xk[8], xq[8];
                *reinterpret_cast<float4 *>(xk) = reinterpret_cast<const float4 *>(xs + c)[0];
                *reinterpret_cast<float4 *>(xk + 4) = reinterpret_cast<const float4 *>(xs + c)[1];
                *reinterpret_cast<float4 *>(xq) = reinterpret_cast<const float4 *>(xs + d + c)[0];
                *reinterpret_cast<float4 *>(xq + 4) = reinterpret_cast<const float4 *>(xs + d + c)[1];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    acc0 = fmaf(xk[e], wv[e], acc0);
                    acc1 = fmaf(xq[e], wv[e], acc1);
                }
            }
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        if (lane == 0) {
            const float bj = feature_bias != nullptr ? to_acc(feature_bias[warp]) : 0.0f;
            own_logits[warp] = acc0 + bj;
            own_logits[kM + warp] = acc1 + bj;
        }
    }
    __syncthreads();

    // ---- feature softmaxes, the normaliser read and the gates (warp 0)
    if (warp == 0) {
        for (int which = 0; which < 2; ++which) {
            const float *logits = own_logits + which * kM;
            float mx = -INFINITY;
            for (int j = lane; j < kM; j += 32) mx = fmaxf(mx, logits[j]);
            mx = warp_max(mx);
            float sum = 0.0f;
            for (int j = lane; j < kM; j += 32) sum += expf(logits[j] - mx);
            sum = warp_sum(sum);
            float *dst = which == 0 ? f : qf;
            for (int j = lane; j < kM; j += 32) dst[j] = expf(logits[j] - mx) / sum;
        }
        __syncwarp();
        float den = lane < kM ? nrm * qf[lane] : 0.0f;
        den = warp_sum(den);
        if (lane == 0) {
            const float lo = 1.0f / 4096.0f, hi = 1.0f - 1.0f / 4096.0f;
            const float decay = lo + (hi - lo) * sigmoidf_(pre_decay);
            const float sv = surprise != nullptr ? fminf(fmaxf(s_value, 0.0f), 1.0f) : 0.0f;
            const float write = sigmoidf_(pre_write) * (0.25f + 0.75f * sv);
            s_decay = ok ? decay : 1.0f;
            s_write = ok ? write : 0.0f;
            s_den = den;
        }
    }
    __syncthreads();
    const float decay = s_decay, write = s_write, den = s_den;
    const float reg = den + 1.0f / 256.0f;
    const float confidence = den / reg;
    const float4 qv = reinterpret_cast<const float4 *>(qf)[part];
    const float4 fv = reinterpret_cast<const float4 *>(f)[part];
    for (int64_t base = row_begin; base < row_end; base += kPasses * kRowsPerPass) {
        float4 x[kPasses];
        float value[kPasses];
#pragma unroll
        for (int u = 0; u < kPasses; ++u) {
            if (base == row_begin) {
                x[u] = x0[u];
                value[u] = value0[u];
            } else {
                const int64_t i = base + u * kRowsPerPass + threadIdx.x / kParts;
                const bool live = i < row_end;
                x[u] = live ? *(reinterpret_cast<const float4 *>(rows + i * kM) + part) : make_float4(0.f, 0.f, 0.f, 0.f);
                value[u] = live ? proj[2 * d + i] : 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < kPasses; ++u) {
            const int64_t i = base + u * kRowsPerPass + threadIdx.x / kParts;
            float num = x[u].x * qv.x + x[u].y * qv.y + x[u].z * qv.z + x[u].w * qv.w;
            for (int o = 1; o < kParts; o <<= 1) num += __shfl_xor_sync(0xffffffffu, num, o);
            if (i >= row_end) continue;
            const float v = write * tanhf(value[u]);
            float4 y;
            y.x = decay * x[u].x + v * fv.x;
            y.y = decay * x[u].y + v * fv.y;
            y.z = decay * x[u].z + v * fv.z;
            y.w = decay * x[u].w + v * fv.w;
            *(reinterpret_cast<float4 *>(rows + i * kM) + part) = y;
            if (part == 0) read_out[b * read_stride + i] = from_acc<TO>(confidence * num / reg);
        }
    }
    // every CTA of the stream has read the normaliser (den) before this
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (blockIdx.y == 0 && threadIdx.x < kM) {
        normalizer[b * kM + threadIdx.x] = decay * nrm + write * f[threadIdx.x];
    }
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_dense_decode_step(const float *projections, const uint8_t *valid, float *working,
                                       void *prior_out, void *h_out, int64_t h_stride, void *h_copy, int64_t batch,
                                       int64_t features, float minimum_retention, float maximum_retention,
                                       int prior_dtype, void *stream) {
    clear_error();
    if (batch < 0 || features < 0) return fail(KOEMI_ERR_INVALID, "negative decode sizes");
    if (batch == 0 || features == 0) return KOEMI_OK;
    const int64_t total = batch * features;
    const unsigned blocks = static_cast<unsigned>(ceil_div(total, 256));
    cudaStream_t s = as_stream(stream);
    switch (prior_dtype) {
        case KOEMI_F32: KOEMI_CUDA_TRY(launch_pdl(decode_gates_kernel<float>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), projections, valid, working, static_cast<float *>(prior_out), static_cast<float *>(h_out), h_stride, static_cast<float *>(h_copy), batch, features, minimum_retention, maximum_retention)); break;
        case KOEMI_BF16: KOEMI_CUDA_TRY(launch_pdl(decode_gates_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), projections, valid, working, static_cast<__nv_bfloat16 *>(prior_out), static_cast<__nv_bfloat16 *>(h_out), h_stride, static_cast<__nv_bfloat16 *>(h_copy), batch, features, minimum_retention, maximum_retention)); break;
        case KOEMI_F16: KOEMI_CUDA_TRY(launch_pdl(decode_gates_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), projections, valid, working, static_cast<__half *>(prior_out), static_cast<__half *>(h_out), h_stride, static_cast<__half *>(h_copy), batch, features, minimum_retention, maximum_retention)); break;
        default: return fail(KOEMI_ERR_INVALID, "prior dtype must be f32, f16 or bf16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_think_ring_decode_step(
    const float *queries, int64_t query_stride, const float *entries, int64_t entry_stride, const uint8_t *valid,
    const float *surprise, float threshold, void *local_keys, void *local_values, uint8_t *local_valid,
    const int64_t *local_head, void *salient_keys, void *salient_values, uint8_t *salient_valid,
    int32_t *salient_head, int32_t *salient_count, void *local_out, void *salient_out, int64_t out_stride,
    float *novelty_out, uint8_t *admission_out, int64_t batch, int64_t width, int64_t local_slots,
    int64_t salient_slots, int ring_dtype, int out_dtype, void *stream) {
    clear_error();
    if (batch < 0 || width < 0 || local_slots < 1 || salient_slots < 1) return fail(KOEMI_ERR_INVALID, "bad ring sizes");
    if (batch == 0) return KOEMI_OK;
    if (ring_dtype != KOEMI_F32 && ring_dtype != KOEMI_BF16) return fail(KOEMI_ERR_INVALID, "rings must be f32 or bf16");
    const int64_t packet = ring_dtype == KOEMI_F32 ? 4 : 8;
    if (width % packet != 0 || !aligned(local_keys, 16) || !aligned(salient_keys, 16) || !aligned(local_values, 16) ||
        !aligned(salient_values, 16)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "ring decode needs 16-byte aligned ring rows (width %% %lld == 0)", (long long)packet);
    }
    if (batch > 2147483647) return fail(KOEMI_ERR_INVALID, "too many streams");
    RingArgs args{queries, query_stride, entries, entry_stride, valid, surprise, threshold, local_keys, local_values,
                  local_valid, local_head, salient_keys, salient_values, salient_valid, salient_head, salient_count,
                  local_out, salient_out, out_stride, novelty_out, admission_out, batch, width, local_slots,
                  salient_slots};
    const int64_t slots = local_slots > salient_slots ? local_slots : salient_slots;
    const size_t smem = (static_cast<size_t>(width) + 2 * slots + kRingWarps) * sizeof(float);
    if (smem > 200 * 1024) return fail(KOEMI_ERR_UNSUPPORTED, "ring decode shared memory too large");
    const dim3 grid(static_cast<unsigned>(batch), 2);
    cudaStream_t s = as_stream(stream);
    // few streams: split every ring over a cluster of CTAs (>= 16 slots each)
    int64_t parts = 2 * static_cast<int64_t>(sm_count()) / batch;  // about two CTAs per SM over both rings
    const int64_t min_slots = local_slots < salient_slots ? local_slots : salient_slots;
    parts = parts > 8 ? 8 : parts;
    while (parts > 1 && min_slots / parts < 16) --parts;
    if (parts >= 2) {
        const int64_t own = (slots + parts - 1) / parts;
        const size_t split_smem = (2 * static_cast<size_t>(width) + 2 * own + kRingWarps) * sizeof(float);
        auto run_split = [&](auto kernel) -> int {
            if (split_smem > 48 * 1024) {
                KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(split_smem)));
            }
            KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(static_cast<unsigned>(batch), 2, static_cast<unsigned>(parts)),
                                      dim3(kRingThreads), split_smem, s, dim3(1, 1, static_cast<unsigned>(parts)), args));
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        };
        const bool bf16_ring = ring_dtype == KOEMI_BF16;
        switch (out_dtype) {
            case KOEMI_F32: return bf16_ring ? run_split(ring_decode_split_kernel<__nv_bfloat16, float>) : run_split(ring_decode_split_kernel<float, float>);
            case KOEMI_BF16: return bf16_ring ? run_split(ring_decode_split_kernel<__nv_bfloat16, __nv_bfloat16>) : run_split(ring_decode_split_kernel<float, __nv_bfloat16>);
            case KOEMI_F16: return bf16_ring ? run_split(ring_decode_split_kernel<__nv_bfloat16, __half>) : run_split(ring_decode_split_kernel<float, __half>);
            default: return fail(KOEMI_ERR_INVALID, "ring outputs must be f32, f16 or bf16");
        }
    }
    auto run = [&](auto kernel) -> int {
        if (smem > 48 * 1024) {
            KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        }
        KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(grid), dim3(kRingThreads), smem, s, dim3(1, 1, 1), args));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    const bool bf16_ring = ring_dtype == KOEMI_BF16;
    switch (out_dtype) {
        case KOEMI_F32: return bf16_ring ? run(ring_decode_kernel<__nv_bfloat16, float>) : run(ring_decode_kernel<float, float>);
        case KOEMI_BF16: return bf16_ring ? run(ring_decode_kernel<__nv_bfloat16, __nv_bfloat16>) : run(ring_decode_kernel<float, __nv_bfloat16>);
        case KOEMI_F16: return bf16_ring ? run(ring_decode_kernel<__nv_bfloat16, __half>) : run(ring_decode_kernel<float, __half>);
        default: return fail(KOEMI_ERR_INVALID, "ring outputs must be f32, f16 or bf16");
    }
}

extern "C" int koemi_assoc_decode_step(const float *projections, int64_t proj_stride, const float *feature_logits,
                                       const void *feature_weight, const void *feature_bias, int weight_dtype,
                                       const float *surprise, const uint8_t *valid, float *basis, float *normalizer,
                                       void *read_out, int64_t read_stride, int64_t batch, int64_t width,
                                       int64_t features, int out_dtype, void *stream) {
    clear_error();
    if (batch < 0 || width < 0 || features < 1 || features > kAssocThreads) return fail(KOEMI_ERR_INVALID, "bad associative sizes");
    if (batch == 0) return KOEMI_OK;
    if (feature_logits == nullptr && feature_weight == nullptr) {
        return fail(KOEMI_ERR_INVALID, "either feature_logits or feature_weight must be given");
    }
    if (features % 4 == 0 && !aligned(basis, 16)) return fail(KOEMI_ERR_UNSUPPORTED, "basis must be 16-byte aligned");
    const bool vector = width % 8 == 0 && aligned(feature_weight, 16) && aligned(projections, 8) && proj_stride % 2 == 0;
    // key and query rows staged in shared memory for the fused feature
    // projection when they fit in 32 KB
    const bool stage = vector && feature_logits == nullptr && width <= 4096;
    const size_t smem = (4 * static_cast<size_t>(features) + (stage ? 2 * static_cast<size_t>(width) : 0)) * sizeof(float);
    // few streams: split each stream's rows over a cluster of up to 8 CTAs so
    // the grid covers the SMs (at least 64 rows per CTA)
    int64_t parts = 2 * static_cast<int64_t>(sm_count()) / batch;
    parts = parts < 1 ? 1 : (parts > 8 ? 8 : parts);
    while (parts > 1 && width / parts < 64) --parts;
    cudaStream_t s = as_stream(stream);
    auto run = [&](auto *out_type, auto *weight_type) -> int {
        using TO = std::remove_pointer_t<decltype(out_type)>;
        using TW = std::remove_pointer_t<decltype(weight_type)>;
        if (stage && features == 16) {  // the config-5 shape: latency-ordered kernel
            KOEMI_CUDA_TRY(launch_pdl(assoc_decode_prefetch_kernel<TO, TW, 16>,
                                      dim3(static_cast<unsigned>(batch), static_cast<unsigned>(parts)),
                                      dim3(kAssocThreads), smem, s, dim3(1, static_cast<unsigned>(parts), 1), projections,
                                      proj_stride, static_cast<const TW *>(feature_weight),
                                      static_cast<const TW *>(feature_bias), surprise, valid, basis, normalizer,
                                      static_cast<TO *>(read_out), read_stride, width));
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        }
        KOEMI_CUDA_TRY(launch_pdl(assoc_decode_kernel<TO, TW>, dim3(static_cast<unsigned>(batch), static_cast<unsigned>(parts)),
                                  dim3(kAssocThreads), smem, s, dim3(1, static_cast<unsigned>(parts), 1), projections,
                                  proj_stride, feature_logits, static_cast<const TW *>(feature_weight),
                                  static_cast<const TW *>(feature_bias), vector, stage, surprise, valid, basis, normalizer,
                                  static_cast<TO *>(read_out), read_stride, batch, width, features));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    auto with_weight = [&](auto *out_type) -> int {
        switch (feature_logits != nullptr ? KOEMI_F32 : weight_dtype) {
            case KOEMI_F32: return run(out_type, static_cast<float *>(nullptr));
            case KOEMI_BF16: return run(out_type, static_cast<__nv_bfloat16 *>(nullptr));
            case KOEMI_F16: return run(out_type, static_cast<__half *>(nullptr));
            default: return fail(KOEMI_ERR_INVALID, "feature weights must be f32, f16 or bf16");
        }
    };
    switch (out_dtype) {
        case KOEMI_F32: return with_weight(static_cast<float *>(nullptr));
        case KOEMI_BF16: return with_weight(static_cast<__nv_bfloat16 *>(nullptr));
        case KOEMI_F16: return with_weight(static_cast<__half *>(nullptr));
        default: return fail(KOEMI_ERR_INVALID, "associative read output must be f32, f16 or bf16");
    }
}
