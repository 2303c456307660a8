// Flag protocol and buffer layout of the expert-parallel peer exchange,
// shared by the exchange kernels (peer.cu), the expert output GEMM that
// stores its rows straight into the senders' buffers (umma.cu) and the
// combine that reads the returned rows in place (moe.cu).
//
// Buffer layout (every rank the same):
//   [0, 256)                     header: flags[2][ranks] (uint64, written by peers),
//                                epoch (uint64), ticket (uint32) at the end
//   recv_ids   [ranks][capacity] int32    rows' owner-local expert ids (-1 padding)
//   recv_rows  [ranks][capacity][width]   rows dispatched to this rank, block = sender
//   ret_rows   [ranks][capacity][width]   outputs returned to this rank, block = owner
// flags[0][s] = epoch once sender s's rows of exchange `epoch` have landed
// here; flags[1][g] = epoch once owner g's outputs have landed here.
#pragma once

#include "common.cuh"

namespace koemi {
namespace peer {

constexpr int64_t kMaxRanks = 8;
constexpr size_t kHeaderBytes = 256;
constexpr int64_t kEpochSlot = 2 * kMaxRanks;      // uint64 index of the local epoch
constexpr int64_t kTicketSlot = 2 * kMaxRanks + 1;  // uint64 index of the CTA ticket
constexpr uint64_t kSpinLimit = uint64_t(1) << 22;  // about a second of polling

struct Layout {
    size_t ids, rows, ret, total;
};

inline Layout layout(int64_t ranks, int64_t capacity, int64_t width, size_t es) {
    auto align = [](size_t v) { return (v + 255) & ~size_t(255); };
    Layout l{};
    l.ids = kHeaderBytes;
    l.rows = align(l.ids + static_cast<size_t>(ranks * capacity) * 4);
    l.ret = align(l.rows + static_cast<size_t>(ranks * capacity * width) * es);
    l.total = align(l.ret + static_cast<size_t>(ranks * capacity * width) * es);
    return l;
}

__device__ __forceinline__ void store_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t load_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t current_epoch(const uint8_t *own) {
    return reinterpret_cast<const volatile uint64_t *>(own)[kEpochSlot];
}

// Thread 0 of every CTA waits until flags[which][r] >= the local epoch for
// every rank r (bounded); the CTA then proceeds. Every thread of the CTA must
// call it. Returns false after a timeout (KOEMI_ERR_TIMEOUT in *status).
__device__ __forceinline__ bool wait_flags(const uint8_t *own, int which, int64_t ranks, int *status) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        const uint64_t *flags = reinterpret_cast<const uint64_t *>(own);
        const uint64_t epoch = current_epoch(own);
        ok = 1;
        for (int64_t r = 0; r < ranks && ok; ++r) {
            uint64_t spin = 0;
            while (load_acquire_sys(flags + which * kMaxRanks + r) < epoch) {
                if (++spin == kSpinLimit) {
                    ok = 0;
                    if (status != nullptr) atomicExch(status, KOEMI_ERR_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

// After every CTA's stores: the last CTA to arrive publishes `epoch` in
// flags[which][rank] of every peer (release, system scope). Every thread of
// every CTA must call it once, after its last store to peer memory.
__device__ __forceinline__ void signal_peers(uint8_t *own, const uint64_t *peers, int which, int64_t rank,
                                             int64_t ranks, uint64_t epoch, bool advance_epoch) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x != 0) return;
    unsigned int *ticket = reinterpret_cast<unsigned int *>(reinterpret_cast<uint64_t *>(own) + kTicketSlot);
    if (atomicAdd(ticket, 1u) != gridDim.x - 1) return;
    __threadfence_system();
    *ticket = 0;
    if (advance_epoch) reinterpret_cast<volatile uint64_t *>(own)[kEpochSlot] = epoch;
    for (int64_t g = 0; g < ranks; ++g) {
        uint64_t *flags = reinterpret_cast<uint64_t *>(peers[g]);
        store_release_sys(flags + which * kMaxRanks + rank, epoch);
    }
}

}  // namespace peer
}  // namespace koemi
