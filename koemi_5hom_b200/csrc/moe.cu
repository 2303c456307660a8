// MoE front: routing, stable permutation into expert segments, gather and
// deterministic combines. All index work is integer and bit-exact.
//
// Permutation = stable counting sort of pair keys (expert id, or E for an
// invalid pair). Pass 1 counts keys per (block of 1024 pairs, bucket); one CTA
// turns the counts into bucket-major exclusive offsets; pass 2 recomputes each
// block's keys and scatters every pair to offset[bucket][block] + its rank
// among equal keys inside the block (warp match-any ranks plus per-warp
// prefix counts), which is exactly the order of a stable argsort. Keys with
// more than 11 bits (E >= 2048) run the same counting sort once per 11-bit
// digit, least significant digit first (an LSD radix sort).
// Reference: moe/moe_kernels.cu:45-145 (route, pair keys, CUB 64-bit radix
// sort, histogram, scan, gathers) and model/experts.py:171-216,261-289.
#include <type_traits>

#include "peer.cuh"
#include "vec.cuh"

namespace koemi {
namespace {

// ------------------------------------------------------------------ routing

__device__ __forceinline__ uint64_t content_hash(uint64_t token, uint64_t previous) {
    // Same arithmetic as content_dispatch_hash (experts.py:30-38): 64-bit
    // products masked to 32 bits, two multiply-xorshift rounds.
    uint64_t value = (token * 1000003ull + previous * 97409ull) & 0xFFFFFFFFull;
    value ^= value >> 16;
    value = (value * 0x45D9F3Bull) & 0xFFFFFFFFull;
    value ^= value >> 16;
    value = (value * 0x45D9F3Bull) & 0xFFFFFFFFull;
    return value ^ (value >> 16);
}

template <typename Index>
__global__ void route_topk_kernel(const Index *__restrict__ tokens, const Index *__restrict__ previous,
                                  const uint8_t *__restrict__ valid, int64_t *__restrict__ out,
                                  int64_t count, int64_t experts, int64_t top_k) {
    pdl_trigger();
    pdl_wait();
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= count) return;
    const bool ok = valid == nullptr || valid[t] != 0;
    const uint64_t hash = content_hash(static_cast<uint64_t>(static_cast<int64_t>(tokens[t])),
                                       static_cast<uint64_t>(static_cast<int64_t>(previous[t])));
    for (int64_t s = 0; s < top_k; ++s) {
        // int64 sum as in assign_top_k (experts.py:287-288): no 2^32 wrap.
        const uint64_t slot_hash = hash + static_cast<uint64_t>(s) * 0x9E3779B9ull;
        out[t * top_k + s] = ok ? static_cast<int64_t>(slot_hash % static_cast<uint64_t>(experts)) : -1;
    }
}

// One warp per token: fp32 softmax over E logits, top-k chosen on the logits
// (monotone in the probability) with the lowest expert id winning ties.
__global__ void learned_topk_kernel(const float *__restrict__ logits, const uint8_t *__restrict__ valid,
                                    int64_t *__restrict__ assignments, float *__restrict__ weights,
                                    float *__restrict__ probabilities, int64_t tokens, int64_t experts,
                                    int64_t top_k, int renormalize) {
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    const bool ok = valid == nullptr || valid[t] != 0;
    const float *row = logits + t * experts;
    float m = -INFINITY;
    for (int64_t e = lane; e < experts; e += 32) m = fmaxf(m, row[e]);
    m = warp_max(m);
    float sum = 0.0f;
    for (int64_t e = lane; e < experts; e += 32) sum += expf(row[e] - m);
    sum = warp_sum(sum);
    if (probabilities != nullptr) {
        for (int64_t e = lane; e < experts; e += 32) {
            probabilities[t * experts + e] = ok ? expf(row[e] - m) / sum : 0.0f;
        }
    }
    float chosen_sum = 0.0f;
    float last_value = INFINITY;
    int64_t last_index = -1;
    for (int64_t k = 0; k < top_k; ++k) {
        // Next candidate: largest logit strictly "after" (last_value, last_index)
        // in the order (value desc, index asc).
        float best = -INFINITY;
        int64_t best_index = INT64_MAX;
        for (int64_t e = lane; e < experts; e += 32) {
            const float v = row[e];
            const bool after = (v < last_value) || (v == last_value && e > last_index);
            if (after && (v > best || (v == best && e < best_index))) {
                best = v;
                best_index = e;
            }
        }
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, offset);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, best_index, offset);
            if (ov > best || (ov == best && oi < best_index)) {
                best = ov;
                best_index = oi;
            }
        }
        last_value = best;
        last_index = best_index;
        const float p = expf(best - m) / sum;
        chosen_sum += p;
        if (lane == 0) {
            assignments[t * top_k + k] = ok ? best_index : -1;
            weights[t * top_k + k] = ok ? p : 0.0f;
        }
    }
    if (renormalize && ok && lane == 0 && chosen_sum > 0.0f) {
        for (int64_t k = 0; k < top_k; ++k) weights[t * top_k + k] /= chosen_sum;
    }
}

// --------------------------------------------------------------- permutation

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kPairsPerThread = 4;
constexpr int kPairsPerBlock = kSortThreads * kPairsPerThread;
constexpr int kDigitBits = 11;
constexpr int kMaxBuckets = 1 << kDigitBits;

// Key of pair p: its expert when valid (first occurrence in the token's
// slots, experts.py:261-267), else E.
template <typename Index>
__device__ __forceinline__ int32_t pair_key(const Index *assignments, const uint8_t *valid,
                                            int64_t pair, int64_t top_k, int64_t experts) {
    const int64_t token = pair / top_k;
    const int64_t slot = pair - token * top_k;
    const int64_t e = static_cast<int64_t>(assignments[pair]);
    bool ok = (valid == nullptr || valid[token] != 0) && e >= 0 && e < experts;
    for (int64_t s = 0; s < slot && ok; ++s) ok = static_cast<int64_t>(assignments[token * top_k + s]) != e;
    return ok ? static_cast<int32_t>(e) : static_cast<int32_t>(experts);
}

// counts[bucket * blocks + block] = number of keys of `block` in `bucket`.
__global__ __launch_bounds__(kSortThreads) void digit_count_kernel(const int32_t *__restrict__ keys, int64_t pairs,
                                                                   int shift, int buckets,
                                                                   int32_t *__restrict__ counts) {
    extern __shared__ int32_t hist[];
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) hist[b] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPairsPerBlock;
    for (int r = 0; r < kPairsPerThread; ++r) {
        const int64_t p = base + r * kSortThreads + threadIdx.x;
        if (p < pairs) atomicAdd(&hist[(keys[p] >> shift) & (buckets - 1)], 1);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) {
        counts[static_cast<int64_t>(b) * gridDim.x + blockIdx.x] = hist[b];
    }
}

// The first pass's count fused with building the keys: each thread makes the
// keys of the pairs it counts (the same pair-to-thread mapping as
// digit_count_kernel) and stores them with their pair index for the scatter.
template <typename Index>
__global__ __launch_bounds__(kSortThreads) void keys_count_kernel(const Index *__restrict__ assignments,
                                                                  const uint8_t *__restrict__ valid,
                                                                  int32_t *__restrict__ keys,
                                                                  int32_t *__restrict__ values, int64_t pairs,
                                                                  int64_t top_k, int64_t experts, int buckets,
                                                                  int32_t *__restrict__ counts) {
    extern __shared__ int32_t hist[];
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) hist[b] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPairsPerBlock;
    for (int r = 0; r < kPairsPerThread; ++r) {
        const int64_t p = base + r * kSortThreads + threadIdx.x;
        if (p < pairs) {
            const int32_t key = pair_key(assignments, valid, p, top_k, experts);
            keys[p] = key;
            values[p] = static_cast<int32_t>(p);
            atomicAdd(&hist[key & (buckets - 1)], 1);
        }
    }
    __syncthreads();
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) {
        counts[static_cast<int64_t>(b) * gridDim.x + blockIdx.x] = hist[b];
    }
}

// Exclusive scan of the bucket-major counts array in place (one CTA, 16
// consecutive counts per thread per round: two rounds for the config-4
// permutation's 32768 counts). Each round's 16384 counts move between global
// and shared memory with coalesced accesses (element i of the round at
// i + i / 16 in shared memory, so each thread's 16 consecutive counts sit in
// distinct banks across a warp); the scan itself reads and writes shared
// memory. With `offsets` it also writes offsets[e] = data[e * stride] for
// e < offsets_count: after a single-pass sort's scan that is the number of
// keys below bucket e, i.e. the segment offsets.
constexpr int kScanPerThread = 16;
constexpr int kScanThreads = 1024;
constexpr int kScanRound = kScanThreads * kScanPerThread;
constexpr size_t kScanSmemBytes = static_cast<size_t>(kScanRound + kScanRound / kScanPerThread) * sizeof(int32_t);
__device__ __forceinline__ int scan_slot(int i) { return i + i / kScanPerThread; }

__global__ __launch_bounds__(kScanThreads) void exclusive_scan_kernel(int32_t *__restrict__ data, int64_t n,
                                                                      int64_t *__restrict__ offsets, int64_t stride,
                                                                      int64_t offsets_count) {
    extern __shared__ int32_t staged[];  // [kScanRound + kScanRound / 16]
    __shared__ int32_t warp_totals[32];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int64_t base = 0; base < n; base += kScanRound) {
#pragma unroll
        for (int j = 0; j < kScanPerThread; ++j) {
            const int i = j * kScanThreads + static_cast<int>(threadIdx.x);
            staged[scan_slot(i)] = base + i < n ? data[base + i] : 0;
        }
        __syncthreads();
        const int first = static_cast<int>(threadIdx.x) * kScanPerThread;
        int32_t v[kScanPerThread];
        int32_t sum = 0;
#pragma unroll
        for (int j = 0; j < kScanPerThread; ++j) {
            v[j] = staged[scan_slot(first + j)];
            sum += v[j];
        }
        int32_t inclusive = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t other = __shfl_up_sync(0xffffffffu, inclusive, o);
            if (lane >= o) inclusive += other;
        }
        if (lane == 31) warp_totals[warp] = inclusive;
        __syncthreads();
        if (warp == 0) {
            int32_t t = warp_totals[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t other = __shfl_up_sync(0xffffffffu, t, o);
                if (lane >= o) t += other;
            }
            warp_totals[lane] = t;
        }
        __syncthreads();
        int32_t running = carry + (warp == 0 ? 0 : warp_totals[warp - 1]) + inclusive - sum;
#pragma unroll
        for (int j = 0; j < kScanPerThread; ++j) {
            staged[scan_slot(first + j)] = running;
            running += v[j];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kScanPerThread; ++j) {
            const int i = j * kScanThreads + static_cast<int>(threadIdx.x);
            if (base + i < n) data[base + i] = staged[scan_slot(i)];
        }
        if (threadIdx.x == 0) carry += warp_totals[31];
        __syncthreads();
    }
    if (offsets != nullptr) {
        for (int64_t e = threadIdx.x; e < offsets_count; e += kScanThreads) offsets[e] = data[e * stride];
    }
}

// Scatter with the block's stable ranks. Round r handles pairs
// base + r*256 + tid, so (round, warp, lane) order equals pair order.
// With `final_positions` (the last pass, when nothing later needs the sorted
// key and value arrays) the pass writes the finishing outputs instead:
// sorted_rows[position] = pair / top_k, sorted_experts[position] = key and
// final_positions[pair] = position (either of the first two may be NULL).
__global__ __launch_bounds__(kSortThreads) void digit_scatter_kernel(
    const int32_t *__restrict__ keys_in, const int32_t *__restrict__ values_in, int64_t pairs, int shift,
    int buckets, const int32_t *__restrict__ offsets, int32_t *__restrict__ keys_out,
    int32_t *__restrict__ values_out, int64_t top_k, int64_t *__restrict__ sorted_rows,
    int64_t *__restrict__ sorted_experts, int64_t *__restrict__ final_positions) {
    extern __shared__ int32_t shared[];
    int32_t *running = shared;                   // [buckets]
    int32_t *warp_counts = shared + buckets;     // [kSortWarps][buckets]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) {
        running[b] = offsets[static_cast<int64_t>(b) * gridDim.x + blockIdx.x];
    }
    for (int i = threadIdx.x; i < kSortWarps * buckets; i += kSortThreads) warp_counts[i] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPairsPerBlock;
    const unsigned lower = (1u << lane) - 1u;
    for (int r = 0; r < kPairsPerThread; ++r) {
        const int64_t p = base + r * kSortThreads + threadIdx.x;
        const bool live = p < pairs;
        const int32_t key = live ? keys_in[p] : 0;
        const int digit = live ? (key >> shift) & (buckets - 1) : -1 - lane;  // unique when dead
        const unsigned same = __match_any_sync(0xffffffffu, digit);
        const int rank = __popc(same & lower);
        const bool leader = (same & lower) == 0;
        if (live && leader) warp_counts[warp * buckets + digit] = __popc(same);
        __syncthreads();
        int32_t before = 0;
        if (live) {
            for (int w = 0; w < warp; ++w) before += warp_counts[w * buckets + digit];
            const int32_t position = running[digit] + before + rank;
            if (final_positions != nullptr) {
                const int32_t pair = values_in[p];
                if (sorted_rows != nullptr) sorted_rows[position] = pair / top_k;
                if (sorted_experts != nullptr) sorted_experts[position] = key;
                final_positions[pair] = position;
            } else {
                keys_out[position] = key;
                values_out[position] = values_in[p];
            }
        }
        __syncthreads();
        for (int b = threadIdx.x; b < buckets; b += kSortThreads) {
            int32_t total = 0;
            for (int w = 0; w < kSortWarps; ++w) {
                total += warp_counts[w * buckets + b];
                warp_counts[w * buckets + b] = 0;
            }
            running[b] += total;
        }
        __syncthreads();
    }
}

// The whole permutation in one CTA for decode-sized inputs (pairs <=
// kSmallPairs, experts < kSmallBuckets): keys, bucket histogram, exclusive
// scan (= segment offsets), the same stable round-based scatter as
// digit_scatter_kernel, and the finishing outputs. The result equals the
// multi-kernel radix path (a stable counting sort has one answer).
constexpr int kSmallThreads = 1024;
constexpr int kSmallWarps = kSmallThreads / 32;
constexpr int64_t kSmallPairs = 4096;
constexpr int64_t kSmallBuckets = 256;

template <typename Index>
__global__ __launch_bounds__(kSmallThreads) void small_permute_kernel(
    const Index *__restrict__ assignments, const uint8_t *__restrict__ valid, int64_t pairs, int64_t top_k,
    int64_t experts, int64_t *__restrict__ segment_offsets, int64_t *__restrict__ sorted_rows,
    int64_t *__restrict__ sorted_experts, int64_t *__restrict__ pair_positions,
    int32_t *__restrict__ sorted_pairs_out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ int32_t shared[];
    const int buckets = static_cast<int>(experts) + 1;  // keys in [0, experts]; experts = dropped
    const int n = static_cast<int>(pairs);
    int32_t *keys = shared;                          // [pairs]
    int32_t *sorted_keys = keys + n;                 // [pairs]
    int32_t *sorted_pairs = sorted_keys + n;         // [pairs]
    int32_t *running = sorted_pairs + n;             // [buckets]
    int32_t *warp_counts = running + buckets;        // [kSmallWarps][buckets]
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int b = threadIdx.x; b < buckets; b += kSmallThreads) running[b] = 0;
    for (int i = threadIdx.x; i < kSmallWarps * buckets; i += kSmallThreads) warp_counts[i] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < n; p += kSmallThreads) {
        const int32_t key = pair_key(assignments, valid, p, top_k, experts);
        keys[p] = key;
        atomicAdd(&running[key], 1);
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the histogram; segment_offsets[e] = first index with key >= e
        int32_t carry = 0;
        for (int b0 = 0; b0 < buckets; b0 += 32) {
            const int b = b0 + lane;
            const int32_t v = b < buckets ? running[b] : 0;
            int32_t inclusive = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t other = __shfl_up_sync(0xffffffffu, inclusive, o);
                if (lane >= o) inclusive += other;
            }
            if (b < buckets) {
                running[b] = carry + inclusive - v;
                segment_offsets[b] = carry + inclusive - v;
            }
            carry += __shfl_sync(0xffffffffu, inclusive, 31);
        }
    }
    __syncthreads();
    const unsigned lower = (1u << lane) - 1u;
    for (int base = 0; base < n; base += kSmallThreads) {
        const int p = base + static_cast<int>(threadIdx.x);
        const bool live = p < n;
        const int32_t key = live ? keys[p] : 0;
        const int digit = live ? key : -1 - lane;  // unique when dead
        const unsigned same = __match_any_sync(0xffffffffu, digit);
        const int rank = __popc(same & lower);
        if (live && (same & lower) == 0) warp_counts[warp * buckets + digit] = __popc(same);
        __syncthreads();
        if (live) {
            int32_t before = 0;
            for (int w = 0; w < warp; ++w) before += warp_counts[w * buckets + digit];
            const int32_t position = running[digit] + before + rank;
            sorted_keys[position] = key;
            sorted_pairs[position] = p;
        }
        __syncthreads();
        for (int b = threadIdx.x; b < buckets; b += kSmallThreads) {
            int32_t total = 0;
            for (int w = 0; w < kSmallWarps; ++w) {
                total += warp_counts[w * buckets + b];
                warp_counts[w * buckets + b] = 0;
            }
            running[b] += total;
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < n; i += kSmallThreads) {
        const int32_t pair = sorted_pairs[i];
        sorted_pairs_out[i] = pair;
        if (sorted_rows != nullptr) sorted_rows[i] = pair / top_k;
        if (sorted_experts != nullptr) sorted_experts[i] = sorted_keys[i];
        if (pair_positions != nullptr) pair_positions[pair] = i;
    }
}

// segment_offsets[e] = first sorted index whose key >= e (keys are sorted).
__global__ void segment_offsets_kernel(const int32_t *__restrict__ sorted_keys, int64_t pairs,
                                       int64_t experts, int64_t *__restrict__ offsets) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e > experts) return;
    int64_t lo = 0, hi = pairs;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (sorted_keys[mid] < e) lo = mid + 1; else hi = mid;
    }
    offsets[e] = lo;
}

__global__ void finish_permutation_kernel(const int32_t *__restrict__ sorted_keys,
                                          const int32_t *__restrict__ sorted_pairs, int64_t pairs,
                                          int64_t top_k, int64_t *__restrict__ sorted_rows,
                                          int64_t *__restrict__ sorted_experts,
                                          int64_t *__restrict__ pair_positions) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int64_t pair = sorted_pairs[i];
    if (sorted_rows != nullptr) sorted_rows[i] = pair / top_k;
    if (sorted_experts != nullptr) sorted_experts[i] = sorted_keys[i];
    if (pair_positions != nullptr) pair_positions[pair] = i;
}

// One warp per sorted row: copy the token's context row, zero past the
// valid count (moe_kernels.cu:122-145).
template <typename T>
__global__ void gather_rows_kernel(const T *__restrict__ context, const int32_t *__restrict__ sorted_pairs,
                                   const int64_t *__restrict__ valid_count, T *__restrict__ out,
                                   int64_t pairs, int64_t width, int64_t top_k, bool vector) {
    const int lane = threadIdx.x & 31;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (i >= pairs) return;
    const bool live = i < *valid_count;
    const int64_t row = sorted_pairs[i] / top_k;
    T *dst = out + i * width;
    const T *src = context + row * width;
    if (vector) {
        constexpr int W = 16 / sizeof(T);
        const int64_t packets = width / W;
        for (int64_t p = lane; p < packets; p += 32) {
            const uint4 v = live ? load_stream(src + p * W) : make_uint4(0, 0, 0, 0);
            store_stream(dst + p * W, v);
        }
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = live ? src[c] : from_acc<T>(0.0f);
    }
}

// Token-major form of the row gather, used when the pair positions are
// known: one warp per token reads its row once and writes it to the sorted
// position of each of its top_k pairs (zeros for pairs past the valid count),
// so a row routed to k experts is read once instead of k times.
template <typename T>
__global__ void scatter_rows_kernel(const T *__restrict__ context, const int64_t *__restrict__ pair_positions,
                                    const int64_t *__restrict__ valid_count, T *__restrict__ out, int64_t tokens,
                                    int64_t width, int64_t top_k, bool vector) {
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    const int64_t valid = *valid_count;
    bool any_live = false;
    for (int64_t k = 0; k < top_k; ++k) any_live |= pair_positions[t * top_k + k] < valid;
    const T *src = context + t * width;
    if (vector) {
        constexpr int W = 16 / sizeof(T);
        const int64_t packets = width / W;
        for (int64_t p = lane; p < packets; p += 32) {
            const uint4 v = any_live ? load_stream(src + p * W) : make_uint4(0, 0, 0, 0);
            for (int64_t k = 0; k < top_k; ++k) {
                const int64_t pos = pair_positions[t * top_k + k];
                store_stream(out + pos * width + p * W, pos < valid ? v : make_uint4(0, 0, 0, 0));
            }
        }
    } else {
        for (int64_t c = lane; c < width; c += 32) {
            const T v = any_live ? src[c] : from_acc<T>(0.0f);
            for (int64_t k = 0; k < top_k; ++k) {
                const int64_t pos = pair_positions[t * top_k + k];
                out[pos * width + c] = pos < valid ? v : from_acc<T>(0.0f);
            }
        }
    }
}

// --------------------------------------------------------------- combines

// slot lists per token: count[row] (atomic), slots[row * cap + j].
__global__ void collect_rows_kernel(const int64_t *__restrict__ sorted_rows,
                                    const int64_t *__restrict__ segment_offsets, int64_t experts,
                                    int64_t tokens, int32_t *__restrict__ counts,
                                    int32_t *__restrict__ slots, int64_t cap) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= segment_offsets[experts]) return;
    const int64_t row = sorted_rows[i];
    if (row < 0 || row >= tokens) return;
    const int32_t j = atomicAdd(&counts[row], 1);
    if (j < cap) slots[row * cap + j] = static_cast<int32_t>(i);
}

template <typename T>
__global__ void combine_rows_kernel(const T *__restrict__ y, const int32_t *__restrict__ counts,
                                    int32_t *__restrict__ slots, int64_t cap, T *__restrict__ out,
                                    int64_t tokens, int64_t width, float inv_k) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= tokens) return;
    int n = counts[row];
    if (n > cap) n = static_cast<int>(cap);
    int32_t *list = slots + row * cap;
    if (lane == 0) {  // ascending sorted-index order, independent of atomic order
        for (int a = 1; a < n; ++a) {
            const int32_t v = list[a];
            int b = a - 1;
            while (b >= 0 && list[b] > v) {
                list[b + 1] = list[b];
                --b;
            }
            list[b + 1] = v;
        }
    }
    __syncwarp();
    for (int64_t c = lane; c < width; c += 32) {
        float acc = 0.0f;
        for (int j = 0; j < n; ++j) acc += to_acc(y[static_cast<int64_t>(list[j]) * width + c]) * inv_k;
        out[row * width + c] = from_acc<T>(acc);
    }
}

// Fused expert combine + residual + RMSNorm (experts.py:136-142,
// router.py:70-73,96-97): one warp per token row, fp32 context.
template <typename T>
__global__ void combine_residual_rmsnorm_kernel(const float *__restrict__ context, const T *__restrict__ y,
                                                const int64_t *__restrict__ positions,
                                                const int64_t *__restrict__ segment_offsets,
                                                const float *__restrict__ weights,
                                                const uint8_t *__restrict__ valid,
                                                const float *__restrict__ norm_weight, float *__restrict__ out,
                                                int64_t tokens, int64_t width, int64_t top_k,
                                                int64_t experts, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= tokens) return;
    const float *cr = context + row * width;
    float *orow = out + row * width;
    if (valid != nullptr && valid[row] == 0) {
        for (int64_t c = lane; c < width; c += 32) orow[c] = cr[c];
        return;
    }
    const int64_t valid_pairs = segment_offsets[experts];
    const float inv_k = 1.0f / static_cast<float>(top_k);
    float sum = 0.0f;
    // pass 1: u = context + sum_slot scale * y, stored to out, sum of squares
    for (int64_t c = lane; c < width; c += 32) {
        float update = 0.0f;
        for (int64_t s = 0; s < top_k; ++s) {
            const int64_t pos = positions[row * top_k + s];
            if (pos < 0 || pos >= valid_pairs) continue;
            const float scale = weights != nullptr ? weights[row * top_k + s] : inv_k;
            update += to_acc(y[pos * width + c]) * scale;
        }
        const float u = cr[c] + update;
        orow[c] = u;
        sum = fmaf(u, u, sum);
    }
    sum = warp_sum(sum);
    const float inv = rsqrtf(sum / static_cast<float>(width) + eps);
    for (int64_t c = lane; c < width; c += 32) orow[c] = orow[c] * inv * norm_weight[c];
}

// Vectorised form of the above for widths that are a multiple of 4 and
// 16-byte aligned rows, k <= 8: one warp per row, float4 context, the row's
// k expert rows read once, the residual sum kept in `out` between passes.
template <typename T>
__global__ void combine_residual_rmsnorm_vec_kernel(const float *__restrict__ context, const T *__restrict__ y,
                                                    const int64_t *__restrict__ positions,
                                                    const int64_t *__restrict__ segment_offsets,
                                                    const float *__restrict__ weights,
                                                    const uint8_t *__restrict__ valid,
                                                    const float *__restrict__ norm_weight, float *__restrict__ out,
                                                    int64_t tokens, int64_t width, int64_t top_k, int64_t experts,
                                                    float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= tokens) return;
    const float4 *cr = reinterpret_cast<const float4 *>(context + row * width);
    float4 *orow = reinterpret_cast<float4 *>(out + row * width);
    const int64_t quads = width / 4;
    if (valid != nullptr && valid[row] == 0) {
        for (int64_t c = lane; c < quads; c += 32) orow[c] = cr[c];
        return;
    }
    const int64_t valid_pairs = segment_offsets[experts];
    const T *src[8];
    float scale[8];
    int live = 0;
    for (int64_t s = 0; s < top_k; ++s) {
        const int64_t pos = positions[row * top_k + s];
        if (pos < 0 || pos >= valid_pairs) continue;
        src[live] = y + pos * width;
        scale[live] = weights != nullptr ? weights[row * top_k + s] : 1.0f / static_cast<float>(top_k);
        ++live;
    }
    float sum = 0.0f;
    for (int64_t c = lane; c < quads; c += 32) {
        float4 u = cr[c];
        for (int s = 0; s < live; ++s) {
            const T *p = src[s] + c * 4;
            u.x += to_acc(p[0]) * scale[s];
            u.y += to_acc(p[1]) * scale[s];
            u.z += to_acc(p[2]) * scale[s];
            u.w += to_acc(p[3]) * scale[s];
        }
        orow[c] = u;
        sum += u.x * u.x + u.y * u.y + u.z * u.z + u.w * u.w;
    }
    sum = warp_sum(sum);
    const float inv = rsqrtf(sum / static_cast<float>(width) + eps);
    const float4 *wq = reinterpret_cast<const float4 *>(norm_weight);
    for (int64_t c = lane; c < quads; c += 32) {
        float4 u = orow[c];
        const float4 w = wq[c];
        u.x *= inv * w.x;
        u.y *= inv * w.y;
        u.z *= inv * w.z;
        u.w *= inv * w.w;
        orow[c] = u;
    }
}

// ------------------------------------------------------ expert parallelism
// Rank g owns experts [g * local_experts, (g + 1) * local_experts), so the
// expert-major sorted pairs are already grouped by owner. The dispatch slab
// holds `capacity` rows per owner: slab row g * capacity + j is sorted row
// segment_offsets[g * local_experts] + j while j is below that owner's count.

// One warp per slab row: copy the sorted row (16-byte packets when `vector`)
// and record its owner-local expert, -1 for padding rows.
template <typename T>
__global__ void ep_pack_kernel(const T *__restrict__ sorted_rows, const int64_t *__restrict__ sorted_experts,
                               const int64_t *__restrict__ offsets, T *__restrict__ slab,
                               int32_t *__restrict__ slab_experts, int64_t ranks, int64_t local_experts,
                               int64_t capacity, int64_t width, bool vector) {
    const int lane = threadIdx.x & 31;
    const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (q >= ranks * capacity) return;
    const int64_t g = q / capacity;
    const int64_t i = offsets[g * local_experts] + (q - g * capacity);
    const bool live = i < offsets[(g + 1) * local_experts];
    if (lane == 0) slab_experts[q] = live ? static_cast<int32_t>(sorted_experts[i] - g * local_experts) : -1;
    if (!live) return;
    const T *src = sorted_rows + i * width;
    T *dst = slab + q * width;
    if (vector) {
        constexpr int W = 16 / sizeof(T);
        for (int64_t p = lane; p < width / W; p += 32) store_stream(dst + p * W, load_stream(src + p * W));
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = src[c];
    }
}

// One warp per sorted row: take the row's result back from its owner's
// returned slab rows; rows past the valid pairs are zero.
template <typename T>
__global__ void ep_unpack_kernel(const T *__restrict__ slab, const int64_t *__restrict__ sorted_experts,
                                 const int64_t *__restrict__ offsets, T *__restrict__ sorted_out, int64_t pairs,
                                 int64_t ranks, int64_t local_experts, int64_t capacity, int64_t width,
                                 bool vector) {
    const int lane = threadIdx.x & 31;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (i >= pairs) return;
    T *dst = sorted_out + i * width;
    const bool live = i < offsets[ranks * local_experts];
    const T *src = nullptr;
    if (live) {
        const int64_t g = sorted_experts[i] / local_experts;
        src = slab + (g * capacity + i - offsets[g * local_experts]) * width;
    }
    if (vector) {
        constexpr int W = 16 / sizeof(T);
        for (int64_t p = lane; p < width / W; p += 32) {
            store_stream(dst + p * W, live ? load_stream(src + p * W) : make_uint4(0, 0, 0, 0));
        }
    } else {
        for (int64_t c = lane; c < width; c += 32) dst[c] = live ? src[c] : from_acc<T>(0.0f);
    }
}

// Four consecutive expert outputs as fp32 (8-byte aligned).
template <typename T>
__device__ __forceinline__ float4 load_quad(const T *p) {
    if constexpr (std::is_same<T, float>::value) {
        const float2 lo = __ldg(reinterpret_cast<const float2 *>(p));
        const float2 hi = __ldg(reinterpret_cast<const float2 *>(p + 2));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
        union {
            uint2 u;
            T h[4];
        } in;
        in.u = __ldg(reinterpret_cast<const uint2 *>(p));
        return make_float4(to_acc(in.h[0]), to_acc(in.h[1]), to_acc(in.h[2]), to_acc(in.h[3]));
    }
}

// Four fp32 values stored as TO (16 bytes of fp32 or 8 bytes of a 16-bit type).
template <typename TO>
__device__ __forceinline__ void store_quad(TO *dst, float4 v) {
    if constexpr (std::is_same<TO, float>::value) {
        *reinterpret_cast<float4 *>(dst) = v;
    } else {
        union {
            TO h[4];
            uint2 u;
        } out;
        out.h[0] = from_acc<TO>(v.x);
        out.h[1] = from_acc<TO>(v.y);
        out.h[2] = from_acc<TO>(v.z);
        out.h[3] = from_acc<TO>(v.w);
        *reinterpret_cast<uint2 *>(dst) = out.u;
    }
}

// Expert outputs still in the exchange buffer (expert-parallel decode): pair
// p's row was returned by the owner g whose segments hold p, at slot
// p - segment_offsets[g * local_experts] of g's block of ret_rows. own ==
// nullptr: the rows are y[p] as usual.
struct ReturnedRows {
    const uint8_t *own;
    size_t ret;
    int64_t capacity, local_experts, ranks;
    int *status;
};

// The vector combine with the row held in registers (NQ quads per lane):
// every load of a row is issued before its values are used, and the output
// is written once. With `next_norm`, the stored row is instead the next
// block's normalised input RMSNorm(x) * next_norm of the combined row x.
// With returned rows, the CTA first waits (bounded) for every owner's return
// flag and reads the rows where the owners stored them.
template <typename T, int NQ, typename TO>
__global__ void combine_residual_rmsnorm_cached_kernel(const ReturnedRows returned, const float *__restrict__ context, const T *__restrict__ y,
                                                       const int64_t *__restrict__ positions,
                                                       const int64_t *__restrict__ segment_offsets,
                                                       const float *__restrict__ weights,
                                                       const uint8_t *__restrict__ valid,
                                                       const float *__restrict__ norm_weight,
                                                       const float *__restrict__ next_norm, TO *__restrict__ out,
                                                       int64_t tokens, int64_t width, int64_t top_k, int64_t experts,
                                                       float eps) {
    pdl_trigger();
    pdl_wait();
    // a wait that gives up (status word set) combines no expert rows
    const bool arrived = returned.own == nullptr || peer::wait_flags(returned.own, 1, returned.ranks, returned.status);
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= tokens) return;
    const float4 *cr = reinterpret_cast<const float4 *>(context + row * width);
    TO *orow = out + row * width;
    const int64_t quads = width / 4;
    float4 u[NQ];
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
        const int64_t c = lane + 32 * i;
        u[i] = c < quads ? __ldg(cr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool combine = valid == nullptr || valid[row] != 0;
    if (combine) {
        const int64_t valid_pairs = segment_offsets[experts];
        for (int64_t s = 0; s < top_k; ++s) {
            const int64_t pos = positions[row * top_k + s];
            if (pos < 0 || pos >= valid_pairs || !arrived) continue;
            const T *src = y + pos * width;
            if (returned.own != nullptr) {
                int64_t g = returned.ranks - 1;
                while (g > 0 && segment_offsets[g * returned.local_experts] > pos) --g;
                src = reinterpret_cast<const T *>(returned.own + returned.ret) +
                      (g * returned.capacity + pos - segment_offsets[g * returned.local_experts]) * width;
            }
            const float scale = weights != nullptr ? weights[row * top_k + s] : 1.0f / static_cast<float>(top_k);
            float4 e[NQ];
#pragma unroll
            for (int i = 0; i < NQ; ++i) {
                const int64_t c = lane + 32 * i;
                e[i] = c < quads ? load_quad(src + c * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < NQ; ++i) {
                u[i].x += e[i].x * scale;
                u[i].y += e[i].y * scale;
                u[i].z += e[i].z * scale;
                u[i].w += e[i].w * scale;
            }
        }
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < NQ; ++i) sum += u[i].x * u[i].x + u[i].y * u[i].y + u[i].z * u[i].z + u[i].w * u[i].w;
        sum = warp_sum(sum);
        const float inv = rsqrtf(sum / static_cast<float>(width) + eps);
        const float4 *wq = reinterpret_cast<const float4 *>(norm_weight);
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
            const int64_t c = lane + 32 * i;
            const float4 w = c < quads ? __ldg(wq + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            u[i] = make_float4(u[i].x * (inv * w.x), u[i].y * (inv * w.y), u[i].z * (inv * w.z), u[i].w * (inv * w.w));
        }
    }
    if (next_norm != nullptr) {  // the input norm of the next block, as rms_rows_cached computes it
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
            sum = fmaf(u[i].x, u[i].x, sum);
            sum = fmaf(u[i].y, u[i].y, sum);
            sum = fmaf(u[i].z, u[i].z, sum);
            sum = fmaf(u[i].w, u[i].w, sum);
        }
        sum = warp_sum(sum);
        const float inv = rsqrtf(sum / static_cast<float>(width) + eps);
        const float4 *nq = reinterpret_cast<const float4 *>(next_norm);
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
            const int64_t c = lane + 32 * i;
            const float4 w = c < quads ? __ldg(nq + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            u[i] = make_float4(u[i].x * inv * w.x, u[i].y * inv * w.y, u[i].z * inv * w.z, u[i].w * inv * w.w);
        }
    }
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
        const int64_t c = lane + 32 * i;
        if (c < quads) store_quad(orow + c * 4, u[i]);
    }
}

// Workspace layout of the permutation.
struct PermuteLayout {
    int64_t blocks;
    int buckets;
    int passes;
    size_t keys_a, values_a, keys_b, values_b, counts, total;
};

PermuteLayout permute_layout(int64_t pairs, int64_t experts) {
    PermuteLayout l{};
    l.blocks = pairs > 0 ? ceil_div(pairs, kPairsPerBlock) : 1;
    int bits = 1;
    while ((int64_t(1) << bits) < experts + 1) ++bits;
    l.passes = (bits + kDigitBits - 1) / kDigitBits;
    l.buckets = l.passes == 1 ? (1 << bits) : kMaxBuckets;
    auto align = [](size_t v) { return (v + 255) & ~size_t(255); };
    size_t offset = 0;
    l.keys_a = offset; offset = align(offset + pairs * sizeof(int32_t));
    l.values_a = offset; offset = align(offset + pairs * sizeof(int32_t));
    l.keys_b = offset; offset = align(offset + pairs * sizeof(int32_t));
    l.values_b = offset; offset = align(offset + pairs * sizeof(int32_t));
    l.counts = offset; offset = align(offset + static_cast<size_t>(l.blocks) * l.buckets * sizeof(int32_t));
    l.total = offset;
    return l;
}

}  // namespace
}  // namespace koemi

using namespace koemi;

extern "C" int koemi_moe_route_topk(const void *token_ids, const void *previous_token_ids,
                                    const uint8_t *valid, int64_t *assignments, int64_t tokens,
                                    int64_t expert_count, int64_t top_k, int index_dtype,
                                    void *stream) {
    clear_error();
    if (tokens < 0) return fail(KOEMI_ERR_INVALID, "tokens must be non-negative");
    if (expert_count < 1 || expert_count > (1 << 20)) return fail(KOEMI_ERR_INVALID, "expert_count must be in [1, 2^20]");
    if (top_k < 1 || top_k > 256 || top_k > expert_count) return fail(KOEMI_ERR_INVALID, "top_k must be in [1, min(256, expert_count)]");
    if (tokens == 0) return KOEMI_OK;
    const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, 256));
    cudaStream_t s = as_stream(stream);
    if (index_dtype == KOEMI_I64) {
        KOEMI_CUDA_TRY(launch_pdl(route_topk_kernel<int64_t>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), static_cast<const int64_t *>(token_ids),
            static_cast<const int64_t *>(previous_token_ids), valid, assignments, tokens, expert_count, top_k));
    } else if (index_dtype == KOEMI_I32) {
        KOEMI_CUDA_TRY(launch_pdl(route_topk_kernel<int32_t>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), static_cast<const int32_t *>(token_ids),
            static_cast<const int32_t *>(previous_token_ids), valid, assignments, tokens, expert_count, top_k));
    } else {
        return fail(KOEMI_ERR_INVALID, "token ids must be int32 or int64");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_moe_learned_topk(const float *gate_logits, const uint8_t *valid,
                                      int64_t *assignments, float *weights, float *probabilities,
                                      int64_t tokens, int64_t expert_count, int64_t top_k,
                                      int renormalize, void *stream) {
    clear_error();
    if (tokens < 0) return fail(KOEMI_ERR_INVALID, "tokens must be non-negative");
    if (expert_count < 1 || top_k < 1 || top_k > expert_count) return fail(KOEMI_ERR_INVALID, "top_k must be in [1, expert_count]");
    if (tokens == 0) return KOEMI_OK;
    const int warps = 8;
    learned_topk_kernel<<<static_cast<unsigned>(ceil_div(tokens, warps)), warps * 32, 0, as_stream(stream)>>>(
        gate_logits, valid, assignments, weights, probabilities, tokens, expert_count, top_k, renormalize);
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" size_t koemi_moe_permute_workspace(int64_t tokens, int64_t top_k, int64_t expert_count) {
    if (tokens < 0 || top_k < 1 || expert_count < 1) return 0;
    return permute_layout(tokens * top_k, expert_count).total;
}

extern "C" int koemi_moe_permute_topk(const void *context, const void *assignments,
                                      const uint8_t *valid, void *sorted_context,
                                      int64_t *sorted_rows, int64_t *sorted_experts,
                                      int64_t *segment_offsets, int64_t *pair_positions,
                                      int64_t tokens, int64_t width, int64_t top_k,
                                      int64_t expert_count, int context_dtype,
                                      int assignment_dtype, void *workspace,
                                      size_t workspace_bytes, void *stream) {
    clear_error();
    if (tokens < 0 || width < 0) return fail(KOEMI_ERR_INVALID, "tokens and width must be non-negative");
    if (expert_count < 1 || expert_count > (1 << 20)) return fail(KOEMI_ERR_INVALID, "expert_count must be in [1, 2^20]");
    if (top_k < 1 || top_k > 256) return fail(KOEMI_ERR_INVALID, "top_k must be in [1, 256]");
    if (tokens * top_k >= (int64_t(1) << 31)) return fail(KOEMI_ERR_UNSUPPORTED, "more than 2^31 pairs");
    if (segment_offsets == nullptr) return fail(KOEMI_ERR_INVALID, "segment_offsets must be non-NULL");
    const int64_t pairs = tokens * top_k;
    const PermuteLayout l = permute_layout(pairs, expert_count);
    if (workspace_bytes < l.total) return fail(KOEMI_ERR_WORKSPACE, "permute needs %zu workspace bytes", l.total);
    cudaStream_t s = as_stream(stream);
    if (pairs == 0) {
        KOEMI_CUDA_TRY(cudaMemsetAsync(segment_offsets, 0, (expert_count + 1) * sizeof(int64_t), s));
        return KOEMI_OK;
    }
    char *ws = static_cast<char *>(workspace);
    int32_t *keys_a = reinterpret_cast<int32_t *>(ws + l.keys_a);
    int32_t *values_a = reinterpret_cast<int32_t *>(ws + l.values_a);
    int32_t *keys_b = reinterpret_cast<int32_t *>(ws + l.keys_b);
    int32_t *values_b = reinterpret_cast<int32_t *>(ws + l.values_b);
    int32_t *counts = reinterpret_cast<int32_t *>(ws + l.counts);
    if (assignment_dtype != KOEMI_I64 && assignment_dtype != KOEMI_I32) {
        return fail(KOEMI_ERR_INVALID, "assignments must be int32 or int64");
    }
    const bool wide_index = assignment_dtype == KOEMI_I64;
    if (pairs <= kSmallPairs && expert_count < kSmallBuckets) {
        const int buckets = static_cast<int>(expert_count) + 1;
        const size_t smem = (3 * static_cast<size_t>(pairs) + static_cast<size_t>(buckets) * (kSmallWarps + 1)) *
                            sizeof(int32_t);
        auto launch = [&](auto kernel, const auto *typed) -> int {
            if (smem > 48 * 1024) {
                KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(smem)));
            }
            KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(1), dim3(kSmallThreads), smem, s, dim3(1, 1, 1), typed, valid, pairs, top_k, expert_count, segment_offsets,
                                                  sorted_rows, sorted_experts, pair_positions, values_a));
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        };
        const int rc = wide_index ? launch(small_permute_kernel<int64_t>, static_cast<const int64_t *>(assignments))
                                  : launch(small_permute_kernel<int32_t>, static_cast<const int32_t *>(assignments));
        if (rc != KOEMI_OK) return rc;
    } else {
        const unsigned pair_blocks = static_cast<unsigned>(ceil_div(pairs, 256));
        const size_t count_smem = static_cast<size_t>(l.buckets) * sizeof(int32_t);
        const size_t scatter_smem = static_cast<size_t>(l.buckets) * (kSortWarps + 1) * sizeof(int32_t);
        if (scatter_smem > 48 * 1024) {
            KOEMI_CUDA_TRY(cudaFuncSetAttribute(digit_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(scatter_smem)));
        }
        KOEMI_CUDA_TRY(cudaFuncSetAttribute(exclusive_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(kScanSmemBytes)));
        for (int pass = 0; pass < l.passes; ++pass) {
            const int shift = pass * kDigitBits;
            if (pass > 0) {
                digit_count_kernel<<<static_cast<unsigned>(l.blocks), kSortThreads, count_smem, s>>>(keys_a, pairs, shift, l.buckets, counts);
            } else if (wide_index) {  // the keys are built by the first count
                keys_count_kernel<int64_t><<<static_cast<unsigned>(l.blocks), kSortThreads, count_smem, s>>>(
                    static_cast<const int64_t *>(assignments), valid, keys_a, values_a, pairs, top_k, expert_count,
                    l.buckets, counts);
            } else {
                keys_count_kernel<int32_t><<<static_cast<unsigned>(l.blocks), kSortThreads, count_smem, s>>>(
                    static_cast<const int32_t *>(assignments), valid, keys_a, values_a, pairs, top_k, expert_count,
                    l.buckets, counts);
            }
            KOEMI_LAUNCH_CHECK();
            // a single pass's scan also yields the segment offsets (every key in its own bucket)
            const bool last_single = l.passes == 1;
            exclusive_scan_kernel<<<1, kScanThreads, kScanSmemBytes, s>>>(
                counts, l.blocks * l.buckets, last_single ? segment_offsets : nullptr, l.blocks, expert_count + 1);
            KOEMI_LAUNCH_CHECK();
            // a single pass that also produces the pair positions writes the
            // finishing outputs itself (the rows then move token-major)
            const bool fused_finish = last_single && pair_positions != nullptr;
            digit_scatter_kernel<<<static_cast<unsigned>(l.blocks), kSortThreads, scatter_smem, s>>>(
                keys_a, values_a, pairs, shift, l.buckets, counts, keys_b, values_b, top_k,
                fused_finish ? sorted_rows : nullptr, fused_finish ? sorted_experts : nullptr,
                fused_finish ? pair_positions : nullptr);
            KOEMI_LAUNCH_CHECK();
            int32_t *t = keys_a; keys_a = keys_b; keys_b = t;
            t = values_a; values_a = values_b; values_b = t;
        }
        if (l.passes > 1) {
            segment_offsets_kernel<<<static_cast<unsigned>(ceil_div(expert_count + 1, 256)), 256, 0, s>>>(keys_a, pairs, expert_count, segment_offsets);
            KOEMI_LAUNCH_CHECK();
        }
        if (!(l.passes == 1 && pair_positions != nullptr)) {
            finish_permutation_kernel<<<pair_blocks, 256, 0, s>>>(keys_a, values_a, pairs, top_k, sorted_rows, sorted_experts, pair_positions);
            KOEMI_LAUNCH_CHECK();
        }
    }
    if (sorted_context != nullptr && width > 0 && pair_positions != nullptr) {
        const size_t es = dtype_size(context_dtype);
        const bool vector = (width * es) % 16 == 0 && aligned(context, 16) && aligned(sorted_context, 16);
        const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, 8));
        const int64_t *valid_count = segment_offsets + expert_count;
        switch (context_dtype) {
            case KOEMI_F32: scatter_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float *>(context), pair_positions, valid_count, static_cast<float *>(sorted_context), tokens, width, top_k, vector); break;
            case KOEMI_F16: scatter_rows_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(context), pair_positions, valid_count, static_cast<__half *>(sorted_context), tokens, width, top_k, vector); break;
            case KOEMI_BF16: scatter_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(context), pair_positions, valid_count, static_cast<__nv_bfloat16 *>(sorted_context), tokens, width, top_k, vector); break;
            default: return fail(KOEMI_ERR_INVALID, "context must be f32, f16 or bf16");
        }
        KOEMI_LAUNCH_CHECK();
    } else if (sorted_context != nullptr && width > 0) {
        const size_t es = dtype_size(context_dtype);
        const bool vector = (width * es) % 16 == 0 && aligned(context, 16) && aligned(sorted_context, 16);
        const unsigned blocks = static_cast<unsigned>(ceil_div(pairs, 8));
        const int64_t *valid_count = segment_offsets + expert_count;
        switch (context_dtype) {
            case KOEMI_F32: gather_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float *>(context), values_a, valid_count, static_cast<float *>(sorted_context), pairs, width, top_k, vector); break;
            case KOEMI_F16: gather_rows_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(context), values_a, valid_count, static_cast<__half *>(sorted_context), pairs, width, top_k, vector); break;
            case KOEMI_BF16: gather_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(context), values_a, valid_count, static_cast<__nv_bfloat16 *>(sorted_context), pairs, width, top_k, vector); break;
            default: return fail(KOEMI_ERR_INVALID, "context must be f32, f16 or bf16");
        }
        KOEMI_LAUNCH_CHECK();
    }
    return KOEMI_OK;
}

extern "C" size_t koemi_moe_combine_workspace(int64_t tokens, int64_t pairs, int64_t top_k) {
    (void)pairs;
    if (tokens <= 0 || top_k <= 0) return 256;
    const size_t counts = ((static_cast<size_t>(tokens) * 4) + 255) & ~size_t(255);
    return counts + static_cast<size_t>(tokens) * top_k * 4;
}

extern "C" int koemi_moe_combine_topk(const void *expert_outputs, const int64_t *sorted_rows,
                                      const int64_t *segment_offsets, void *out, int64_t pairs,
                                      int64_t width, int64_t tokens, int64_t top_k,
                                      int64_t expert_count, int dtype, void *workspace,
                                      size_t workspace_bytes, void *stream) {
    clear_error();
    if (tokens < 0 || width < 0 || pairs < 0) return fail(KOEMI_ERR_INVALID, "sizes must be non-negative");
    if (top_k < 1 || expert_count < 0) return fail(KOEMI_ERR_INVALID, "top_k must be positive");
    if (tokens == 0 || width == 0) return KOEMI_OK;
    if (workspace_bytes < koemi_moe_combine_workspace(tokens, pairs, top_k)) {
        return fail(KOEMI_ERR_WORKSPACE, "combine needs %zu workspace bytes", koemi_moe_combine_workspace(tokens, pairs, top_k));
    }
    cudaStream_t s = as_stream(stream);
    int32_t *counts = static_cast<int32_t *>(workspace);
    int32_t *slots = reinterpret_cast<int32_t *>(static_cast<char *>(workspace) + (((static_cast<size_t>(tokens) * 4) + 255) & ~size_t(255)));
    KOEMI_CUDA_TRY(cudaMemsetAsync(counts, 0, tokens * sizeof(int32_t), s));
    if (pairs > 0) {
        collect_rows_kernel<<<static_cast<unsigned>(ceil_div(pairs, 256)), 256, 0, s>>>(sorted_rows, segment_offsets, expert_count, tokens, counts, slots, top_k);
        KOEMI_LAUNCH_CHECK();
    }
    const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, 8));
    const float inv_k = 1.0f / static_cast<float>(top_k);
    switch (dtype) {
        case KOEMI_F32: combine_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float *>(expert_outputs), counts, slots, top_k, static_cast<float *>(out), tokens, width, inv_k); break;
        case KOEMI_F16: combine_rows_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(expert_outputs), counts, slots, top_k, static_cast<__half *>(out), tokens, width, inv_k); break;
        case KOEMI_BF16: combine_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(expert_outputs), counts, slots, top_k, static_cast<__nv_bfloat16 *>(out), tokens, width, inv_k); break;
        default: return fail(KOEMI_ERR_INVALID, "expert outputs must be f32, f16 or bf16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_moe_combine_residual_rmsnorm(const float *context, const void *expert_out,
                                                  const int64_t *pair_positions,
                                                  const int64_t *segment_offsets,
                                                  const float *weights, const uint8_t *valid,
                                                  const float *norm_weight, float *out,
                                                  int64_t tokens, int64_t width, int64_t top_k,
                                                  int64_t expert_count, float eps, int dtype,
                                                  void *stream) {
    clear_error();
    if (tokens < 0 || width < 0 || top_k < 1) return fail(KOEMI_ERR_INVALID, "bad combine sizes");
    if (tokens == 0 || width == 0) return KOEMI_OK;
    const int rows_per_block = tokens >= static_cast<int64_t>(sm_count()) * 32 ? 8 : 2;
    const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, rows_per_block));
    const int threads = rows_per_block * 32;
    cudaStream_t s = as_stream(stream);
    const bool vector = width % 4 == 0 && top_k <= 8 && aligned(context, 16) && aligned(out, 16) &&
                        aligned(norm_weight, 16) && aligned(expert_out, 8);
    const int64_t quads_per_lane = ceil_div(width / 4, 32);
    if (vector && quads_per_lane <= 16) {
        const ReturnedRows returned{};
        auto run = [&](auto kernel, const auto *typed) -> int {
            KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(blocks), dim3(threads), 0, s, dim3(1, 1, 1), returned, context, typed, pair_positions, segment_offsets, weights, valid,
                                              norm_weight, nullptr, out, tokens, width, top_k, expert_count, eps));
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        };
        auto by_width = [&](const auto *typed) -> int {
            using T = std::remove_cv_t<std::remove_pointer_t<decltype(typed)>>;
            if (quads_per_lane <= 4) return run(combine_residual_rmsnorm_cached_kernel<T, 4, float>, typed);
            if (quads_per_lane <= 8) return run(combine_residual_rmsnorm_cached_kernel<T, 8, float>, typed);
            return run(combine_residual_rmsnorm_cached_kernel<T, 16, float>, typed);
        };
        switch (dtype) {
            case KOEMI_F32: return by_width(static_cast<const float *>(expert_out));
            case KOEMI_F16: return by_width(static_cast<const __half *>(expert_out));
            case KOEMI_BF16: return by_width(static_cast<const __nv_bfloat16 *>(expert_out));
            default: return fail(KOEMI_ERR_INVALID, "expert outputs must be f32, f16 or bf16");
        }
    }
    if (vector) {
        switch (dtype) {
            case KOEMI_F32: combine_residual_rmsnorm_vec_kernel<float><<<blocks, threads, 0, s>>>(context, static_cast<const float *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
            case KOEMI_F16: combine_residual_rmsnorm_vec_kernel<__half><<<blocks, threads, 0, s>>>(context, static_cast<const __half *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
            case KOEMI_BF16: combine_residual_rmsnorm_vec_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(context, static_cast<const __nv_bfloat16 *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
            default: return fail(KOEMI_ERR_INVALID, "expert outputs must be f32, f16 or bf16");
        }
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    }
    switch (dtype) {
        case KOEMI_F32: combine_residual_rmsnorm_kernel<float><<<blocks, threads, 0, s>>>(context, static_cast<const float *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
        case KOEMI_F16: combine_residual_rmsnorm_kernel<__half><<<blocks, threads, 0, s>>>(context, static_cast<const __half *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
        case KOEMI_BF16: combine_residual_rmsnorm_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(context, static_cast<const __nv_bfloat16 *>(expert_out), pair_positions, segment_offsets, weights, valid, norm_weight, out, tokens, width, top_k, expert_count, eps); break;
        default: return fail(KOEMI_ERR_INVALID, "expert outputs must be f32, f16 or bf16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free permutation: the same stable permutation as
// koemi_moe_permute_topk, with its scratch in a fixed device array instead of
// a caller workspace, for callers that cannot allocate device memory.
#include <mutex>

namespace {
constexpr size_t kStaticPermuteScratchBytes = size_t(2) << 20;  // 2 MiB on every device that loads the library
constexpr int kStaticScratchDevices = 64;

// A cached address is only valid in the context it was looked up in: after
// cudaDeviceReset, or when a host drives the device through another context,
// the array lives at a different address. Each cache entry therefore carries
// the driver's unique id of its context (cuCtxGetId, resolved through the
// runtime's driver entry point, so the library still needs no -lcuda).
struct StaticScratchEntry {
    unsigned long long context_id;
    void *address;
};
std::mutex g_static_scratch_mutex;
StaticScratchEntry g_static_scratch[kStaticScratchDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
std::once_flag g_ctx_entry_once;

// Unique id of the calling thread's current context; 0 when there is none yet.
int current_context_id(unsigned long long *id) {
    std::call_once(g_ctx_entry_once, [] {
        void *entry = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &entry, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess) {
            g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(entry);
        }
        entry = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &entry, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess) {
            g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(entry);
        }
    });
    if (g_ctx_get_current == nullptr || g_ctx_get_id == nullptr) {
        return fail(KOEMI_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are unavailable from the driver");
    }
    CUcontext context = nullptr;
    if (g_ctx_get_current(&context) != CUDA_SUCCESS) return fail(KOEMI_ERR_CUDA, "cuCtxGetCurrent failed");
    *id = 0;
    if (context != nullptr && g_ctx_get_id(context, id) != CUDA_SUCCESS) {
        return fail(KOEMI_ERR_CUDA, "cuCtxGetId failed");
    }
    return KOEMI_OK;
}
}  // namespace

static __device__ __align__(256) unsigned char koemi_permute_static_scratch[kStaticPermuteScratchBytes];

namespace {
// Device address of the scratch array in the current device's current
// context. The lookup (cudaGetSymbolAddress with that device current) runs
// on the first call in a context and again whenever the context changed;
// later calls in the same context reuse the cached address.
int static_permute_scratch(void **out) {
    int device = 0;
    KOEMI_CUDA_TRY(cudaGetDevice(&device));
    if (device < 0 || device >= kStaticScratchDevices) {
        return fail(KOEMI_ERR_UNSUPPORTED, "device %d is beyond the static-scratch device table", device);
    }
    unsigned long long context_id = 0;
    int rc = current_context_id(&context_id);
    if (rc != KOEMI_OK) return rc;
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    StaticScratchEntry &entry = g_static_scratch[device];
    if (context_id == 0 || entry.address == nullptr || entry.context_id != context_id) {
        void *address = nullptr;
        KOEMI_CUDA_TRY(cudaGetSymbolAddress(&address, koemi_permute_static_scratch));
        rc = current_context_id(&context_id);  // the lookup may have created the primary context
        if (rc != KOEMI_OK) return rc;
        entry.context_id = context_id;
        entry.address = address;
    }
    *out = entry.address;
    return KOEMI_OK;
}
}  // namespace

extern "C" int koemi_moe_permute_topk_static(const void *context, const void *assignments, const uint8_t *valid,
                                             void *sorted_context, int64_t *sorted_rows, int64_t *sorted_experts,
                                             int64_t *segment_offsets, int64_t *pair_positions, int64_t tokens,
                                             int64_t width, int64_t top_k, int64_t expert_count, int context_dtype,
                                             int assignment_dtype, void *stream) {
    clear_error();
    if (tokens < 0 || top_k < 1 || top_k > 256 || expert_count < 1 || expert_count > (1 << 20)) {
        return fail(KOEMI_ERR_INVALID, "need tokens >= 0, top_k in [1, 256] and expert_count in [1, 2^20]");
    }
    const size_t need = koemi_moe_permute_workspace(tokens, top_k, expert_count);
    if (need > kStaticPermuteScratchBytes) {
        return fail(KOEMI_ERR_UNSUPPORTED,
                    "allocation-free permute: %lld tokens x top_k %lld over %lld experts needs %zu scratch bytes "
                    "(koemi_moe_permute_workspace), more than the fixed %zu-byte array; 65536 token-expert pairs "
                    "always fit at any expert count, more fit with fewer experts; use koemi_moe_permute_topk with "
                    "a workspace", (long long)tokens, (long long)top_k, (long long)expert_count, need,
                    kStaticPermuteScratchBytes);
    }
    void *scratch = nullptr;
    const int rc = static_permute_scratch(&scratch);
    if (rc != KOEMI_OK) return rc;
    // Nothing in the scratch has to start at zero: every count, key and
    // index the permutation reads is written earlier in the same call.
    return koemi_moe_permute_topk(context, assignments, valid, sorted_context, sorted_rows, sorted_experts,
                                  segment_offsets, pair_positions, tokens, width, top_k, expert_count, context_dtype,
                                  assignment_dtype, scratch, kStaticPermuteScratchBytes, stream);
}

// ---------------------------------------------------------------------------
// Expert-parallel dispatch and return slabs.

extern "C" int koemi_moe_ep_pack(const void *sorted_rows, const int64_t *sorted_experts,
                                 const int64_t *segment_offsets, void *slab, int32_t *slab_experts,
                                 int64_t pairs, int64_t width, int64_t ranks, int64_t local_experts,
                                 int64_t capacity, int dtype, void *stream) {
    clear_error();
    if (pairs < 0 || width < 1 || ranks < 1 || local_experts < 1) return fail(KOEMI_ERR_INVALID, "bad expert-parallel sizes");
    if (capacity < pairs) return fail(KOEMI_ERR_INVALID, "capacity %lld is below the %lld pairs one owner may receive", (long long)capacity, (long long)pairs);
    const int64_t rows = ranks * capacity;
    if (rows == 0) return KOEMI_OK;
    const size_t es = dtype_size(dtype);
    const bool vector = (width * es) % 16 == 0 && aligned(sorted_rows, 16) && aligned(slab, 16);
    const unsigned blocks = static_cast<unsigned>(ceil_div(rows, 8));
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: ep_pack_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float *>(sorted_rows), sorted_experts, segment_offsets, static_cast<float *>(slab), slab_experts, ranks, local_experts, capacity, width, vector); break;
        case KOEMI_F16: ep_pack_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(sorted_rows), sorted_experts, segment_offsets, static_cast<__half *>(slab), slab_experts, ranks, local_experts, capacity, width, vector); break;
        case KOEMI_BF16: ep_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(sorted_rows), sorted_experts, segment_offsets, static_cast<__nv_bfloat16 *>(slab), slab_experts, ranks, local_experts, capacity, width, vector); break;
        default: return fail(KOEMI_ERR_INVALID, "rows must be f32, f16 or bf16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

extern "C" int koemi_moe_ep_unpack(const void *slab, const int64_t *sorted_experts, const int64_t *segment_offsets,
                                   void *sorted_out, int64_t pairs, int64_t width, int64_t ranks,
                                   int64_t local_experts, int64_t capacity, int dtype, void *stream) {
    clear_error();
    if (pairs < 0 || width < 1 || ranks < 1 || local_experts < 1) return fail(KOEMI_ERR_INVALID, "bad expert-parallel sizes");
    if (capacity < pairs) return fail(KOEMI_ERR_INVALID, "capacity %lld is below the %lld pairs one owner may receive", (long long)capacity, (long long)pairs);
    if (pairs == 0) return KOEMI_OK;
    const size_t es = dtype_size(dtype);
    const bool vector = (width * es) % 16 == 0 && aligned(slab, 16) && aligned(sorted_out, 16);
    const unsigned blocks = static_cast<unsigned>(ceil_div(pairs, 8));
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case KOEMI_F32: ep_unpack_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float *>(slab), sorted_experts, segment_offsets, static_cast<float *>(sorted_out), pairs, ranks, local_experts, capacity, width, vector); break;
        case KOEMI_F16: ep_unpack_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half *>(slab), sorted_experts, segment_offsets, static_cast<__half *>(sorted_out), pairs, ranks, local_experts, capacity, width, vector); break;
        case KOEMI_BF16: ep_unpack_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(slab), sorted_experts, segment_offsets, static_cast<__nv_bfloat16 *>(sorted_out), pairs, ranks, local_experts, capacity, width, vector); break;
        default: return fail(KOEMI_ERR_INVALID, "rows must be f32, f16 or bf16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

// ---------------------------------------------------------------------------
// Combine fused with the next block's input norm (decode chains of blocks).

namespace {
int combine_next(const ReturnedRows &returned, const float *context, const void *expert_out,
                 const int64_t *pair_positions, const int64_t *segment_offsets, const float *weights,
                 const uint8_t *valid, const float *norm_weight, const float *next_norm_weight, void *out,
                 int out_dtype, int64_t tokens, int64_t width, int64_t top_k, int64_t expert_count, float eps,
                 int dtype, void *stream) {
    if (tokens < 0 || width < 0 || top_k < 1) return fail(KOEMI_ERR_INVALID, "bad combine sizes");
    if (tokens == 0 || width == 0) return KOEMI_OK;
    const int64_t quads_per_lane = ceil_div(width / 4, 32);
    if (width % 4 != 0 || quads_per_lane > 16 || top_k > 8 || !aligned(context, 16) || !aligned(norm_weight, 16) ||
        !aligned(expert_out, 8) || !aligned(out, 16) || (next_norm_weight != nullptr && !aligned(next_norm_weight, 16))) {
        return fail(KOEMI_ERR_UNSUPPORTED, "fused combine needs width %% 4 == 0, width <= 2048, top_k <= 8 and aligned rows");
    }
    const int rows_per_block = tokens >= static_cast<int64_t>(sm_count()) * 32 ? 8 : 2;
    const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, rows_per_block));
    const int threads = rows_per_block * 32;
    cudaStream_t s = as_stream(stream);
    auto run = [&](auto *typed, auto *out_typed) -> int {
        using T = std::remove_cv_t<std::remove_pointer_t<decltype(typed)>>;
        using TO = std::remove_pointer_t<decltype(out_typed)>;
        auto launch = [&](auto kernel) -> int {
            KOEMI_CUDA_TRY(launch_pdl(kernel, dim3(blocks), dim3(threads), 0, s, dim3(1, 1, 1), returned, context, typed, pair_positions, segment_offsets, weights, valid,
                                              norm_weight, next_norm_weight, out_typed, tokens, width, top_k,
                                              expert_count, eps));
            KOEMI_LAUNCH_CHECK();
            return KOEMI_OK;
        };
        if (quads_per_lane <= 4) return launch(combine_residual_rmsnorm_cached_kernel<T, 4, TO>);
        if (quads_per_lane <= 8) return launch(combine_residual_rmsnorm_cached_kernel<T, 8, TO>);
        return launch(combine_residual_rmsnorm_cached_kernel<T, 16, TO>);
    };
    auto by_out = [&](auto *typed) -> int {
        switch (out_dtype) {
            case KOEMI_F32: return run(typed, static_cast<float *>(out));
            case KOEMI_BF16: return run(typed, static_cast<__nv_bfloat16 *>(out));
            case KOEMI_F16: return run(typed, static_cast<__half *>(out));
            default: return fail(KOEMI_ERR_INVALID, "output must be f32, f16 or bf16");
        }
    };
    switch (dtype) {
        case KOEMI_F32: return by_out(static_cast<const float *>(expert_out));
        case KOEMI_F16: return by_out(static_cast<const __half *>(expert_out));
        case KOEMI_BF16: return by_out(static_cast<const __nv_bfloat16 *>(expert_out));
        default: return fail(KOEMI_ERR_INVALID, "expert outputs must be f32, f16 or bf16");
    }
}
}  // namespace

extern "C" int koemi_moe_combine_residual_rmsnorm_next(const float *context, const void *expert_out,
                                                       const int64_t *pair_positions,
                                                       const int64_t *segment_offsets, const float *weights,
                                                       const uint8_t *valid, const float *norm_weight,
                                                       const float *next_norm_weight, void *out, int out_dtype,
                                                       int64_t tokens, int64_t width, int64_t top_k,
                                                       int64_t expert_count, float eps, int dtype, void *stream) {
    clear_error();
    return combine_next(ReturnedRows{}, context, expert_out, pair_positions, segment_offsets, weights, valid,
                        norm_weight, next_norm_weight, out, out_dtype, tokens, width, top_k, expert_count, eps, dtype,
                        stream);
}

extern "C" int koemi_ep_combine_residual_rmsnorm_next(const float *context, const int64_t *pair_positions,
                                                      const int64_t *segment_offsets, const float *weights,
                                                      const uint8_t *valid, const float *norm_weight,
                                                      const float *next_norm_weight, void *out, int out_dtype,
                                                      int64_t tokens, int64_t width, int64_t top_k,
                                                      int64_t expert_count, float eps, int dtype, const void *own,
                                                      int64_t ranks, int64_t local_experts, int64_t capacity,
                                                      void *stream) {
    clear_error();
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16 && dtype != KOEMI_F32) {
        return fail(KOEMI_ERR_INVALID, "returned rows must be f32, f16 or bf16");
    }
    if (own == nullptr || !aligned(own, 256) || ranks < 1 || ranks > peer::kMaxRanks || local_experts < 1 ||
        capacity < 1 || expert_count != ranks * local_experts) {
        return fail(KOEMI_ERR_INVALID, "bad exchange arguments for the returned-row combine");
    }
    const peer::Layout l = peer::layout(ranks, capacity, width, dtype_size(dtype));
    const ReturnedRows returned{static_cast<const uint8_t *>(own), l.ret, capacity, local_experts, ranks,
                                device_status_word()};
    // the returned rows are the exchange buffer's: expert_out only fixes the
    // row type and its alignment check
    return combine_next(returned, context, static_cast<const uint8_t *>(own) + l.ret, pair_positions,
                        segment_offsets, weights, valid, norm_weight, next_norm_weight, out, out_dtype, tokens, width,
                        top_k, expert_count, eps, dtype, stream);
}

// ---------------------------------------------------------------------------
// Gather of sorted pair rows with a type conversion, for callers that reuse
// one permutation for several row sets (the hash route of a decode step is
// the same for every block; only the rows differ).

template <typename TI, typename TO>
__global__ void gather_convert_kernel(const TI *__restrict__ rows, const int64_t *__restrict__ sorted_rows,
                                      const int64_t *__restrict__ valid_count, TO *__restrict__ out, int64_t pairs,
                                      int64_t width) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (i >= pairs) return;
    const bool live = i < *valid_count;
    const TI *src = rows + (live ? sorted_rows[i] : 0) * width;
    TO *dst = out + i * width;
    for (int64_t c = lane * 4; c < width; c += 128) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live) {
            if constexpr (std::is_same<TI, float>::value) {
                v = __ldg(reinterpret_cast<const float4 *>(src + c));
            } else {
                v = load_quad(src + c);
            }
        }
        store_quad(dst + c, v);
    }
}

extern "C" int koemi_moe_gather_rows(const void *rows, int rows_dtype, const int64_t *sorted_rows,
                                     const int64_t *segment_offsets, int64_t expert_count, void *out, int out_dtype,
                                     int64_t pairs, int64_t width, void *stream) {
    clear_error();
    if (pairs < 0 || width < 1 || expert_count < 0) return fail(KOEMI_ERR_INVALID, "bad gather sizes");
    if (pairs == 0) return KOEMI_OK;
    if (width % 4 != 0 || !aligned(rows, 16) || !aligned(out, 16)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "row gather needs width %% 4 == 0 and 16-byte aligned rows");
    }
    const unsigned blocks = static_cast<unsigned>(ceil_div(pairs, 8));
    const int64_t *valid_count = segment_offsets + expert_count;
    cudaStream_t s = as_stream(stream);
    auto run = [&](const auto *in, auto *typed_out) -> int {
        using TI = std::remove_cv_t<std::remove_pointer_t<decltype(in)>>;
        using TO = std::remove_pointer_t<decltype(typed_out)>;
        KOEMI_CUDA_TRY(launch_pdl(gather_convert_kernel<TI, TO>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), in, sorted_rows, valid_count, typed_out, pairs, width));
        KOEMI_LAUNCH_CHECK();
        return KOEMI_OK;
    };
    auto by_out = [&](const auto *in) -> int {
        switch (out_dtype) {
            case KOEMI_F32: return run(in, static_cast<float *>(out));
            case KOEMI_BF16: return run(in, static_cast<__nv_bfloat16 *>(out));
            case KOEMI_F16: return run(in, static_cast<__half *>(out));
            default: return fail(KOEMI_ERR_INVALID, "output must be f32, f16 or bf16");
        }
    };
    switch (rows_dtype) {
        case KOEMI_F32: return by_out(static_cast<const float *>(rows));
        case KOEMI_BF16: return by_out(static_cast<const __nv_bfloat16 *>(rows));
        case KOEMI_F16: return by_out(static_cast<const __half *>(rows));
        default: return fail(KOEMI_ERR_INVALID, "rows must be f32, f16 or bf16");
    }
}

// ---------------------------------------------------------------------------
// The decode block's fusion RMSNorm fused with the row gather of its expert
// pairs: token row t of `fused` (fp32) is normalised with exactly the
// arithmetic of the cached RMSNorm row kernel (the same loads and sum order)
// into `context` (fp32, the combine's residual), and the normalised row is
// also stored, in the rows' dtype, at the sorted position of each of its
// top_k pairs below the valid count. Rows of `rows_out` past the valid pairs
// are left as they were (the expert GEMMs never store their results).

namespace koemi {
namespace {

template <typename T>
__global__ void norm_gather_kernel(const float *__restrict__ fused, const float *__restrict__ norm_weight,
                                   float eps, float *__restrict__ context, const int64_t *__restrict__ positions,
                                   const int64_t *__restrict__ offsets, int64_t experts, T *__restrict__ rows_out,
                                   int64_t tokens, int64_t width, int64_t top_k) {
    pdl_trigger();
    pdl_wait();
    constexpr int NV = 16;  // 16-byte fp32 packets per lane: width <= 2048
    const int lane = threadIdx.x & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    const int64_t packets = width / 4;
    const float *xr = fused + t * width;
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
    const float inv = rsqrtf(sum / static_cast<float>(width) + eps);
    float *cr = context + t * width;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t p = lane + 32 * i;
        if (p < packets) {
            v[i] = make_float4(v[i].x * inv * w[i].x, v[i].y * inv * w[i].y, v[i].z * inv * w[i].z,
                               v[i].w * inv * w[i].w);
            *reinterpret_cast<float4 *>(cr + p * 4) = v[i];
        }
    }
    const int64_t valid_pairs = offsets[experts];
    for (int64_t s = 0; s < top_k; ++s) {
        const int64_t pos = positions[t * top_k + s];
        if (pos < 0 || pos >= valid_pairs) continue;
        T *dst = rows_out + pos * width;
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

}  // namespace
}  // namespace koemi

extern "C" int koemi_moe_norm_gather(const float *fused, const float *norm_weight, float eps, float *context,
                                     const int64_t *pair_positions, const int64_t *segment_offsets,
                                     int64_t expert_count, void *rows_out, int rows_dtype, int64_t tokens,
                                     int64_t width, int64_t top_k, void *stream) {
    clear_error();
    if (tokens < 0 || width < 1 || top_k < 1 || expert_count < 1) return fail(KOEMI_ERR_INVALID, "bad norm-gather sizes");
    if (tokens == 0) return KOEMI_OK;
    if (width % 4 != 0 || width > 2048 || !aligned(fused, 16) || !aligned(norm_weight, 16) || !aligned(context, 16) ||
        !aligned(rows_out, 8) || pair_positions == nullptr || segment_offsets == nullptr) {
        return fail(KOEMI_ERR_UNSUPPORTED, "norm-gather needs width a multiple of 4 up to 2048 and aligned rows");
    }
    const unsigned blocks = static_cast<unsigned>(ceil_div(tokens, 8));
    cudaStream_t s = as_stream(stream);
    switch (rows_dtype) {
        case KOEMI_BF16:
            KOEMI_CUDA_TRY(launch_pdl(norm_gather_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1),
                                      fused, norm_weight, eps, context, pair_positions, segment_offsets, expert_count,
                                      static_cast<__nv_bfloat16 *>(rows_out), tokens, width, top_k));
            break;
        case KOEMI_F16:
            KOEMI_CUDA_TRY(launch_pdl(norm_gather_kernel<__half>, dim3(blocks), dim3(256), 0, s, dim3(1, 1, 1), fused,
                                      norm_weight, eps, context, pair_positions, segment_offsets, expert_count,
                                      static_cast<__half *>(rows_out), tokens, width, top_k));
            break;
        default: return fail(KOEMI_ERR_INVALID, "gathered rows must be bf16 or f16");
    }
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}
