// tcgen05 tensor-core GEMMs with fused epilogues, for sm_100a.
//
// One persistent kernel per problem, one CTA per SM (192 KB of shared memory,
// all 512 TMEM columns). Warp roles:
//   warp 0      TMA producer: per K block of 64, loads the A tile [128 x 64]
//               and the B tile [256 x 64] (bf16/f16, 128B-swizzled K-major)
//               into a 4-stage shared-memory ring;
//   warp 1      allocates TMEM; one thread issues tcgen05.mma
//               (M=128, N=256, K=16, fp32 accumulate) into one of two
//               256-column accumulators and commits stage/accumulator
//               completion to mbarriers;
//   warps 2..   epilogue: tcgen05.ld each accumulator row (one TMEM lane per
//               thread), apply the fused epilogue, store to global memory,
//               release the accumulator (four warps; eight for the gated
//               problem, two per lane quarter splitting the columns).
// The epilogue of tile i overlaps the MMAs of tile i+1.
//
// Problems:
//   kGated   expert GEMM 1: B = [gate rows n*128.. ; value rows n*128..] of
//            the tile's expert; hidden = silu(g + bg) * (v + bv) (dtype).
//   kOutput  expert GEMM 2: y = hidden W_o^T + b_o (dtype).
//   kSurprise head contraction: logits = prior W^T + b folded into per-row
//            (max, sum exp, target logit) partials per 256-wide vocab tile.
//   kDense / kDenseCluster  fp32 projection out = A W^T + b, optionally split
//            along K, the splits reduced inside a thread-block cluster.
// Grouped problems map tiles to (expert, row tile) on the device from
// segment_offsets; rows past a segment's end are computed but never stored.
//
// Every mbarrier wait is bounded; a wait that runs out raises a CTA abort
// flag, records KOEMI_ERR_TIMEOUT in the device status word and every role
// leaves its loop, so the CTA frees its TMEM and exits. No multicast loads.
#include <algorithm>
#include <mutex>

#include "peer.cuh"
#include "vec.cuh"

namespace koemi {

__global__ void tile_prefix_kernel(const int64_t *offsets, int64_t experts, int64_t tile_rows, int32_t *prefix);

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;  // problems with four epilogue warps

// The gated problem's SwiGLU epilogue (two TMEM reads, bias adds and a SiLU
// per output) takes longer than the MMAs of a tile with four warps, so it
// runs eight: two per TMEM lane quarter, each on half of the columns. The
// direct dense problem runs eight as well: its paired tiles use both TMEM
// accumulators, so its epilogue (256 rows x 256 fp32 columns) does not
// overlap the next tile's MMAs and its length is lost time.
template <int kProblem>
constexpr int epilogue_warps() {
    return kProblem == 0 || kProblem == 3 ? 8 : 4;
}
template <int kProblem>
constexpr int threads_for() {
    return (2 + epilogue_warps<kProblem>()) * 32;
}
constexpr uint32_t kABytes = kBM * kBK * 2;
constexpr uint32_t kBBytes = kBN * kBK * 2;
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemColumns = 512;
constexpr int kMaxPipe = 8;  // barrier slots: the deepest ring (narrow tiles)
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
static_assert((2 * kMaxPipe + 4) * 8 + 8 <= 256, "barrier area");

enum Problem : int { kGated = 0, kOutput = 1, kSurprise = 2, kDense = 3, kDenseCluster = 4 };

// kDenseCluster: the K splits of one output tile run as one thread-block
// cluster (one CTA per split); each CTA parks its fp32 accumulator in its own
// shared memory, and after a cluster barrier CTA r sums column slice r over
// all splits in split order through distributed shared memory (deterministic),
// adds the bias and stores. Row stride of the parked accumulator, in floats
// (padded so the per-row float4 stores of a warp hit distinct banks):
constexpr int kAccStride = kBN + 4;
static_assert(kBM * kAccStride * 4 <= kStages * kStageBytes, "parked accumulator must fit in the stage ring");

struct UmmaArgs {
    CUtensorMap map_a;
    CUtensorMap map_b0;
    CUtensorMap map_b1;
    int64_t k;
    int64_t rows;             // rows of A (pairs or prior rows)
    int64_t n_tiles;          // tiles along N
    int64_t b_rows_per_group; // rows of B per expert (0 for surprise)
    int64_t n_out;            // valid output columns (H, D or C)
    int64_t out_stride;       // elements per output row
    int64_t experts;
    int64_t band;             // surprise: row tiles per band (tile order swizzle)
    int64_t splits;           // dense: K splits (partials reduced by a second kernel when > 1)
    int64_t k_per_split;      // dense: K blocks per split (every split non-empty)
    const int64_t *offsets;
    const int32_t *tile_prefix;
    const void *bias0;
    const void *bias1;
    void *out;
    float *partials;
    const int64_t *targets;   // surprise: target column per row, or NULL (no target logit)
    int64_t lse_rows;         // surprise: rows below fold into partials; rows at or above write logits to out
    int64_t pad_column;       // surprise: column left out of the log-sum-exp (-1: none)
    int64_t group_rows;       // dense, uniform groups: A rows per group (0: one ungrouped problem)
    const float *row_lse;     // surprise gradient: per-row log-sum-exp (NULL: forward modes)
    const float *row_scale;   // surprise gradient: per-row dL/dNLL (0 on invalid rows)
    float *grad_out;          // surprise gradient: fp32 dlogits [rows, n_out]
    int64_t weights_ready;    // dense: no earlier kernel of the stream writes B (its first stages load before pdl_wait)
    // expert-parallel return (output problem): row r's output goes to slot
    // ret_slots[r] = sender * ret_capacity + j of this owner's block in the
    // sender's exchange buffer, then the senders' return flags are raised
    const uint64_t *ret_peers;  // [ret_ranks] exchange buffer of every rank (NULL: store to out)
    uint8_t *ret_own;
    const int64_t *ret_slots;
    int64_t ret_offset, ret_capacity, ret_rank, ret_ranks;
    int *status;
    uint32_t idesc;
};

// ------------------------------------------------------------------ PTX

__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_address) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((smem_address & 0x3FFFF) >> 4);  // start address
    desc |= static_cast<uint64_t>(1) << 16;                          // LBO (unused for swizzled K-major)
    desc |= static_cast<uint64_t>(1024 >> 4) << 32;                  // SBO: 8 rows x 128 B
    desc |= static_cast<uint64_t>(1) << 46;                          // descriptor version (sm100)
    desc |= static_cast<uint64_t>(2) << 61;                          // 128-byte swizzle
    return desc;
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define KOEMI_TMEM_LD32(taddr, v)                                                                              \
    asm volatile(                                                                                              \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, " \
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"    \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),     \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),             \
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),           \
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),           \
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                                                                \
        : "r"(taddr))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait that also watches the CTA abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    for (uint32_t spin = 0; spin < kWaitSpinLimit; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 255) == 255 && *abort) return false;
    }
    *abort = 1;
    if (status != nullptr) atomicExch(status, KOEMI_ERR_TIMEOUT);
    return false;
}

__device__ __forceinline__ bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
__device__ __forceinline__ bool aligned8(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

// Cluster barrier over every thread of every CTA of the cluster, with
// release/acquire ordering of shared-memory writes at cluster scope.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// float4 from the shared memory of CTA `rank` of this cluster, at the offset
// that `local_addr` has in this CTA's shared memory.
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

// ------------------------------------------------------------- scheduling

struct Tile {
    int64_t row0;      // first A row of the tile
    int64_t row_end;   // rows >= row_end are not stored
    int64_t n;         // tile index along N
    int64_t group;     // expert (grouped) or 0
    int64_t m_tile;    // row tile index (surprise: partial slot)
    int64_t k_begin;   // K blocks [k_begin, k_end) of this tile
    int64_t k_end;
    int64_t split;     // dense: K split index
};

// kTileRows: A rows per tile, kBM, or 2 * kBM for the paired tiles of the
// dense and surprise problems (two M=128 MMAs share every B stage).
template <int kProblem, int kTileRows>
__device__ __forceinline__ int64_t total_tiles(const UmmaArgs &a) {
    if (kProblem == kSurprise) return ((a.rows + kTileRows - 1) / kTileRows) * a.n_tiles;
    if (kProblem == kDense && a.group_rows > 0) {
        return (a.rows / a.group_rows) * ((a.group_rows + kTileRows - 1) / kTileRows) * a.n_tiles;
    }
    if (kProblem == kDense || kProblem == kDenseCluster) {
        return ((a.rows + kTileRows - 1) / kTileRows) * a.n_tiles * a.splits;
    }
    return static_cast<int64_t>(a.tile_prefix[a.experts]) * a.n_tiles;
}

template <int kProblem, int kTileRows>
__device__ __forceinline__ Tile tile_at(const UmmaArgs &a, int64_t t) {
    Tile tile{};
    const int64_t k_blocks = (a.k + kBK - 1) / kBK;
    tile.k_begin = 0;
    tile.k_end = k_blocks;
    if (kProblem == kDenseCluster) {
        // split fastest: the CTAs of one cluster are the splits of one tile
        const int64_t m_tiles = (a.rows + kTileRows - 1) / kTileRows;
        tile.split = t % a.splits;
        const int64_t rest = t / a.splits;
        tile.m_tile = rest % m_tiles;
        tile.n = rest / m_tiles;
        tile.k_begin = tile.split * a.k_per_split;
        tile.k_end = min(k_blocks, tile.k_begin + a.k_per_split);
        tile.row0 = tile.m_tile * kTileRows;
        tile.row_end = a.rows;
        return tile;
    }
    if (kProblem == kDense && a.group_rows > 0) {
        // uniform groups (a batch of small products): group g's A rows are
        // [g * group_rows, (g + 1) * group_rows) and its B rows start at
        // g * b_rows_per_group; N fastest, so a group's A tile is reused from L2
        const int64_t per_group = (a.group_rows + kTileRows - 1) / kTileRows;
        tile.n = t % a.n_tiles;
        const int64_t rest = t / a.n_tiles;
        tile.group = rest / per_group;
        tile.m_tile = rest;
        tile.row0 = tile.group * a.group_rows + (rest - tile.group * per_group) * kTileRows;
        tile.row_end = (tile.group + 1) * a.group_rows;
        tile.split = 0;
        return tile;
    }
    if (kProblem == kDense && a.band > 0 && a.splits == 1) {
        // many row tiles (prefill): bands of `band` row tiles, N walked inside
        // a band, so the CTAs running together reuse the band's activation
        // tiles and each weight tile from L2 (row-tile-fastest order streams
        // the activations from HBM once per wave of weight tiles)
        const int64_t m_tiles = (a.rows + kTileRows - 1) / kTileRows;
        const int64_t per_band = a.band * a.n_tiles;
        const int64_t band = t / per_band;
        const int64_t in_band = t - band * per_band;
        const int64_t band_rows = min(a.band, m_tiles - band * a.band);
        tile.n = in_band / band_rows;
        tile.m_tile = band * a.band + (in_band - tile.n * band_rows);
        tile.split = 0;
        tile.row0 = tile.m_tile * kTileRows;
        tile.row_end = a.rows;
        return tile;
    }
    if (kProblem == kDense) {
        // m fastest, so CTAs running together share one weight tile from L2
        const int64_t m_tiles = (a.rows + kTileRows - 1) / kTileRows;
        tile.m_tile = t % m_tiles;
        const int64_t rest = t / m_tiles;
        tile.n = rest % a.n_tiles;
        tile.split = rest / a.n_tiles;
        tile.k_begin = tile.split * a.k_per_split;
        tile.k_end = min(k_blocks, tile.k_begin + a.k_per_split);
        tile.row0 = tile.m_tile * kTileRows;
        tile.row_end = a.rows;
        return tile;
    }
    if (kProblem == kSurprise) {
        // bands of `band` row tiles; inside a band walk N first so each vocab
        // tile is reused from L2 by every row tile of the band
        const int64_t m_tiles = (a.rows + kTileRows - 1) / kTileRows;
        const int64_t per_band = a.band * a.n_tiles;
        const int64_t band = t / per_band;
        const int64_t in_band = t - band * per_band;
        const int64_t band_rows = min(a.band, m_tiles - band * a.band);
        tile.n = in_band / band_rows;
        tile.m_tile = band * a.band + (in_band - tile.n * band_rows);
        tile.row0 = tile.m_tile * kTileRows;
        tile.row_end = a.rows;
        return tile;
    }
    const int64_t mt = t / a.n_tiles;
    tile.n = t - mt * a.n_tiles;
    int64_t lo = 0, hi = a.experts;
    while (lo + 1 < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (a.tile_prefix[mid] <= mt) lo = mid; else hi = mid;
    }
    tile.group = lo;
    tile.row0 = a.offsets[lo] + (mt - a.tile_prefix[lo]) * kBM;
    tile.row_end = a.offsets[lo + 1];
    tile.m_tile = mt;
    return tile;
}

// ---------------------------------------------------------------- kernel

// 32 bias values starting at column col0 as fp32 (zero past n_out): four
// 16-byte loads when the run is whole and aligned (every lane of a warp reads
// the same addresses), else element by element.
template <typename T>
__device__ __forceinline__ void load_bias32(const T *bias, int64_t col0, int64_t n_out, float (&out)[32]) {
    const T *src = bias + col0;
    if (col0 + 32 <= n_out && aligned16(src)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float part[8];
            unpack(load_cached(src + q * 8), part, T());
#pragma unroll
            for (int e = 0; e < 8; ++e) out[q * 8 + e] = part[e];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) out[j] = col0 + j < n_out ? to_acc(src[j]) : 0.0f;
    }
}

// Rows of one column quad summed over the S parked split accumulators of a
// cluster (distributed shared memory) in split order, plus the bias, stored
// as fp32. The loads of 32 / S rows (32 float4 per thread) are all requested
// before the first sum, so the remote latency is paid once per batch of rows.
// `dst` is the quad's column in row 0; `n_left` the valid columns from there.
template <int S>
__device__ __forceinline__ void reduce_parked_rows(uint32_t parked_base, int my_row, int row_step, int valid_rows,
                                                   int q, const float (&bias4)[4], float *dst, int64_t out_stride,
                                                   int64_t n_left) {
    constexpr int R = 32 / S;
    for (int r0 = my_row; r0 < valid_rows; r0 += R * row_step) {
        float4 v[R][S];
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int r = r0 + u * row_step;
            if (r < valid_rows) {
                const uint32_t offset = parked_base + static_cast<uint32_t>((r * kAccStride + q * 4) * 4);
#pragma unroll
                for (int sp = 0; sp < S; ++sp) v[u][sp] = ld_dsmem_f4(offset, static_cast<uint32_t>(sp));
            }
        }
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int r = r0 + u * row_step;
            if (r >= valid_rows) continue;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int sp = 0; sp < S; ++sp) {
                acc.x += v[u][sp].x;
                acc.y += v[u][sp].y;
                acc.z += v[u][sp].z;
                acc.w += v[u][sp].w;
            }
            const float o[4] = {acc.x + bias4[0], acc.y + bias4[1], acc.z + bias4[2], acc.w + bias4[3]};
            float *p = dst + static_cast<int64_t>(r) * out_stride;
            if (n_left >= 4 && aligned16(p)) {
                *reinterpret_cast<float4 *>(p) = make_float4(o[0], o[1], o[2], o[3]);
            } else if (n_left >= 4 && aligned8(p)) {
                reinterpret_cast<float2 *>(p)[0] = make_float2(o[0], o[1]);
                reinterpret_cast<float2 *>(p)[1] = make_float2(o[2], o[3]);
            } else {
                for (int e = 0; e < 4 && e < n_left; ++e) p[e] = o[e];
            }
        }
    }
}

// kTileN < 256 (output and direct dense problems): N = 128 or 64 tiles, for
// decode-sized problems whose 256-wide tiles would leave SMs idle or need a
// split-K reduction; the smaller stages run a deeper ring.
template <int kProblem, typename T, bool kPair, int kTileN = kBN>
__global__ __launch_bounds__(threads_for<kProblem>(), 1) void umma_gemm_kernel(const __grid_constant__ UmmaArgs args) {
    // paired tiles: 256 A rows (two 128-row halves) per tile, stages of
    // A0 | A1 | B (64 KB, 3 of them), both 256-column accumulators in use
    constexpr uint32_t kAStage = kPair ? 2 * kABytes : kABytes;
    constexpr uint32_t kBStage = static_cast<uint32_t>(kTileN) * kBK * 2;
    constexpr uint32_t kStage = kAStage + kBStage;
    constexpr int kDeepPipe = static_cast<int>((kStages * kStageBytes) / kStage);
    constexpr int kPipe = kPair ? 3 : (kTileN < kBN ? (kDeepPipe < kMaxPipe ? kDeepPipe : kMaxPipe) : kStages);
    static_assert(kTileN == kBN || kProblem == kOutput || kProblem == kDense,
                  "narrow tiles are for the expert output and direct dense problems");
    static_assert(kTileN == kBN || kTileN == kBN / 2 || kTileN == kBN / 4, "tile width 256, 128 or 64");
    constexpr int kTileRows = kPair ? 2 * kBM : kBM;
    constexpr int kHalves = kPair ? 2 : 1;
    constexpr int kAccBufs = kPair ? 1 : 2;
    static_assert(kPipe * kStage <= kStages * kStageBytes, "stage ring exceeds the shared-memory budget");
    static_assert(!kPair || kProblem == kSurprise || kProblem == kDense || kProblem == kDenseCluster,
                  "paired tiles are for the dense and surprise problems");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t *smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *empty = full + kMaxPipe;
    uint64_t *acc_full = empty + kMaxPipe;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t k_blocks = (args.k + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPipe; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kAccBufs; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], epilogue_warps<kProblem>());
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Dense problems whose weights no earlier kernel writes (launched with the
    // programmatic attribute): the weight tiles of this CTA's first stages are
    // requested before waiting for the previous kernel of the stream, so
    // their DRAM latency overlaps its tail. Everything else below pdl_wait may
    // read what the previous kernel wrote.
    int64_t early = 0;
    if constexpr (kProblem == kDense || kProblem == kDenseCluster) {
        if (args.weights_ready && warp == 0 && lane == 0 &&
            static_cast<int64_t>(blockIdx.x) < total_tiles<kProblem, kTileRows>(args)) {
            prefetch_tensor_map(&args.map_b0);
            const Tile tile = tile_at<kProblem, kTileRows>(args, blockIdx.x);
            early = min(static_cast<int64_t>(kPipe), tile.k_end - tile.k_begin);
            for (int s = 0; s < early; ++s) {
                mbar_arrive_expect_tx(&full[s], kStage);
                tma_load_2d(stages + s * kStage + kAStage, &args.map_b0, &full[s],
                            static_cast<int32_t>((tile.k_begin + s) * kBK),
                            static_cast<int32_t>(tile.group * args.b_rows_per_group + tile.n * kTileN));
            }
        }
    }
    pdl_wait();
    const int64_t tiles = total_tiles<kProblem, kTileRows>(args);

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tensor_map(&args.map_a);
            prefetch_tensor_map(&args.map_b0);
            if (kProblem == kGated) prefetch_tensor_map(&args.map_b1);
            int stage = 0;
            uint32_t phase = 0;
            for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                const Tile tile = tile_at<kProblem, kTileRows>(args, t);
                for (int64_t kb = tile.k_begin; kb < tile.k_end; ++kb) {
                    if (!wait_or_abort(&empty[stage], phase ^ 1, abort, args.status)) break;
                    uint8_t *a_dst = stages + stage * kStage;
                    uint8_t *b_dst = a_dst + kAStage;
                    // a stage whose weight tile went out before pdl_wait
                    // already expects the whole stage's bytes
                    const bool b_issued = t == static_cast<int64_t>(blockIdx.x) && kb - tile.k_begin < early;
                    if (!b_issued) mbar_arrive_expect_tx(&full[stage], kStage);
                    const int32_t kc = static_cast<int32_t>(kb * kBK);
                    tma_load_2d(a_dst, &args.map_a, &full[stage], kc, static_cast<int32_t>(tile.row0));
                    if (kPair) {  // rows past the end read as zeros (full box bytes still arrive)
                        tma_load_2d(a_dst + kABytes, &args.map_a, &full[stage], kc,
                                    static_cast<int32_t>(tile.row0 + kBM));
                    }
                    if (kProblem == kGated) {
                        const int32_t r = static_cast<int32_t>(tile.group * args.b_rows_per_group + tile.n * 128);
                        tma_load_2d(b_dst, &args.map_b0, &full[stage], kc, r);
                        tma_load_2d(b_dst + kBBytes / 2, &args.map_b1, &full[stage], kc, r);
                    } else if (!b_issued) {
                        const int32_t r = static_cast<int32_t>(tile.group * args.b_rows_per_group + tile.n * kTileN);
                        tma_load_2d(b_dst, &args.map_b0, &full[stage], kc, r);
                    }
                    if (++stage == kPipe) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                if (!wait_or_abort(&acc_empty[acc], acc_phase ^ 1, abort, args.status)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + static_cast<uint32_t>(acc * kBN);
                const Tile tile = tile_at<kProblem, kTileRows>(args, t);
                bool ok = true;
                for (int64_t kb = tile.k_begin; kb < tile.k_end; ++kb) {
                    if (!wait_or_abort(&full[stage], phase, abort, args.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(stages + stage * kStage);
                    const uint32_t b_addr = a_addr + kAStage;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        const uint32_t accumulate = (kb > tile.k_begin || k > 0) ? 1u : 0u;
                        umma_f16(tmem_d, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32),
                                 args.idesc, accumulate);
                        if (kPair) {
                            umma_f16(tmem_d + kBN, sw128_kmajor_desc(a_addr + kABytes + k * 32),
                                     sw128_kmajor_desc(b_addr + k * 32), args.idesc, accumulate);
                        }
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == kPipe) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(&acc_full[acc]);
                if (++acc == kAccBufs) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
        __syncwarp();
    } else {
        // epilogue warps: warp w reads TMEM lanes 32*(w%4) .. +31; with eight
        // warps, warps 2..5 take the first half of the columns, 6..9 the second
        const int quarter = warp & 3;
        constexpr int kParts = epilogue_warps<kProblem>() / 4;
        const int part = (warp - 2) / 4;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
            const Tile tile = tile_at<kProblem, kTileRows>(args, t);
            if (!wait_or_abort(&acc_full[acc], acc_phase, abort, args.status)) break;
            tc_fence_after();
#pragma unroll 1
            for (int h = 0; h < kHalves; ++h) {
            const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>((acc + h) * kBN);
            const int64_t row = tile.row0 + h * kBM + quarter * 32 + lane;
            const bool row_ok = row < tile.row_end && row < args.rows;
            if (kProblem == kGated) {
                const T *bg = static_cast<const T *>(args.bias0) + tile.group * args.b_rows_per_group;
                const T *bv = static_cast<const T *>(args.bias1) + tile.group * args.b_rows_per_group;
                T *out = static_cast<T *>(args.out);
                constexpr int kChunks = 4 / kParts;
#pragma unroll 1
                for (int cc = 0; cc < kChunks; ++cc) {
                    const int c = part * kChunks + cc;
                    uint32_t g[32], v[32];
                    KOEMI_TMEM_LD32(taddr + c * 32, g);
                    KOEMI_TMEM_LD32(taddr + 128 + c * 32, v);
                    tmem_wait_ld();
                    const int64_t col0 = tile.n * 128 + c * 32;
                    if (row_ok && col0 < args.n_out) {
                        float gb[32], vb[32];
                        load_bias32(bg, col0, args.n_out, gb);
                        load_bias32(bv, col0, args.n_out, vb);
                        float h[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            h[j] = silu_fast(__uint_as_float(g[j]) + gb[j]) * (__uint_as_float(v[j]) + vb[j]);
                        }
                        T *dst = out + row * args.out_stride + col0;
                        if (col0 + 32 <= args.n_out) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                float part8[8];
#pragma unroll
                                for (int e = 0; e < 8; ++e) part8[e] = h[q * 8 + e];
                                *reinterpret_cast<uint4 *>(dst + q * 8) = pack(part8, T());
                            }
                        } else {
                            for (int j = 0; j < 32 && col0 + j < args.n_out; ++j) dst[j] = from_acc<T>(h[j]);
                        }
                    }
                }
            } else if (kProblem == kOutput) {
                const T *bo = static_cast<const T *>(args.bias0) + tile.group * args.b_rows_per_group;
                T *out_row = static_cast<T *>(args.out) + row * args.out_stride;
                if (args.ret_peers != nullptr && row_ok) {
                    // the received slot of this row: straight back to its sender
                    const int64_t slot = args.ret_slots[row];
                    const int64_t sender = slot / args.ret_capacity;
                    const int64_t j = slot - sender * args.ret_capacity;
                    out_row = reinterpret_cast<T *>(reinterpret_cast<uint8_t *>(args.ret_peers[sender]) + args.ret_offset) +
                              (args.ret_rank * args.ret_capacity + j) * args.out_stride;
                }
#pragma unroll 1
                for (int c = 0; c < kTileN / 32; ++c) {
                    uint32_t y[32];
                    KOEMI_TMEM_LD32(taddr + c * 32, y);
                    tmem_wait_ld();
                    const int64_t col0 = tile.n * kTileN + c * 32;
                    if (row_ok && col0 < args.n_out) {
                        float o[32];
                        load_bias32(bo, col0, args.n_out, o);
#pragma unroll
                        for (int j = 0; j < 32; ++j) o[j] += __uint_as_float(y[j]);
                        T *dst = out_row + col0;
                        if (col0 + 32 <= args.n_out) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                float part8[8];
#pragma unroll
                                for (int e = 0; e < 8; ++e) part8[e] = o[q * 8 + e];
                                *reinterpret_cast<uint4 *>(dst + q * 8) = pack(part8, T());
                            }
                        } else {
                            for (int j = 0; j < 32 && col0 + j < args.n_out; ++j) dst[j] = from_acc<T>(o[j]);
                        }
                    }
                }
            } else if (kProblem == kDenseCluster) {
                // parked and reduced after the role loops, one half at a time
            } else if (kProblem == kDense) {
                // splits == 1: out = acc + bias (fp32, row stride out_stride);
                // splits  > 1: partials[split][row][col] = acc, reduced later
                const T *bias = static_cast<const T *>(args.bias0);
                const bool direct = args.splits == 1;
                float *dst_row = direct ? static_cast<float *>(args.out) + row * args.out_stride
                                        : args.partials + (tile.split * args.rows + row) * args.n_out;
                constexpr int kChunks = kTileN / 32 / kParts;
#pragma unroll 1
                for (int cc = 0; cc < kChunks; ++cc) {
                    const int c = part * kChunks + cc;
                    uint32_t y[32];
                    KOEMI_TMEM_LD32(taddr + c * 32, y);
                    tmem_wait_ld();
                    const int64_t col0 = tile.n * kTileN + c * 32;
                    if (row_ok && col0 < args.n_out) {
                        float o[32];
                        if (direct && bias != nullptr) {
                            load_bias32(bias, col0, args.n_out, o);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) o[j] = 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 32; ++j) o[j] += __uint_as_float(y[j]);
                        float *dst = dst_row + col0;
                        if (col0 + 32 <= args.n_out && aligned16(dst)) {
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                reinterpret_cast<float4 *>(dst)[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                            }
                        } else if (col0 + 32 <= args.n_out && aligned8(dst)) {
                            // rows of an even but not 4-aligned stride (the
                            // associative projection's 3 d + 2 columns)
#pragma unroll
                            for (int q = 0; q < 16; ++q) reinterpret_cast<float2 *>(dst)[q] = make_float2(o[2 * q], o[2 * q + 1]);
                        } else {
                            for (int j = 0; j < 32 && col0 + j < args.n_out; ++j) dst[j] = o[j];
                        }
                    }
                }
            } else {
                // rows below lse_rows fold into per-slice log-sum-exp
                // partials; rows at or above (the head pass's logits rows)
                // store acc + bias for every column (PAD included). The TMEM
                // loads stay outside the row-dependent branches: tcgen05.ld
                // is warp-aligned and a warp may hold both kinds of row.
                const T *bias = static_cast<const T *>(args.bias0);
                const bool logit_row = row >= args.lse_rows;
                const int64_t target = row_ok && !logit_row && args.targets != nullptr ? args.targets[row] : -1;
                float run_max = -INFINITY, run_sum = 0.0f, target_logit = -INFINITY;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t y[32];
                    KOEMI_TMEM_LD32(taddr + c * 32, y);
                    tmem_wait_ld();
                    const int64_t col0 = tile.n * kBN + c * 32;
                    if (args.grad_out != nullptr) {
                        // gradient mode: dlogits = scale * (softmax - onehot(target))
                        if (row_ok && col0 < args.n_out) {
                            const float lse = args.row_lse[row];
                            const float scale = args.row_scale[row];
                            float g[32];
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const int64_t col = col0 + j;
                                const float l = __uint_as_float(y[j]) + (col < args.n_out ? to_acc(bias[col]) : 0.0f);
                                g[j] = scale * (expf(l - lse) - (col == target ? 1.0f : 0.0f));
                            }
                            float *dst = args.grad_out + row * args.n_out + col0;
                            if (col0 + 32 <= args.n_out && aligned16(dst)) {
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    reinterpret_cast<float4 *>(dst)[q] = make_float4(g[4 * q], g[4 * q + 1], g[4 * q + 2], g[4 * q + 3]);
                                }
                            } else {
                                for (int j = 0; j < 32 && col0 + j < args.n_out; ++j) dst[j] = g[j];
                            }
                        }
                        continue;
                    }
                    if (logit_row) {
                        if (row_ok && col0 < args.n_out) {
                            float o[32];
                            load_bias32(bias, col0, args.n_out, o);
#pragma unroll
                            for (int j = 0; j < 32; ++j) o[j] += __uint_as_float(y[j]);
                            float *dst = static_cast<float *>(args.out) + (row - args.lse_rows) * args.out_stride + col0;
                            if (col0 + 32 <= args.n_out && aligned16(dst)) {
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    reinterpret_cast<float4 *>(dst)[q] =
                                        make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                                }
                            } else {
                                for (int j = 0; j < 32 && col0 + j < args.n_out; ++j) dst[j] = o[j];
                            }
                        }
                        continue;
                    }
                    float l[32];
                    float chunk_max = -INFINITY;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int64_t col = col0 + j;
                        l[j] = col < args.n_out && col != args.pad_column ? __uint_as_float(y[j]) + to_acc(bias[col])
                                                                          : -INFINITY;
                        chunk_max = fmaxf(chunk_max, l[j]);
                    }
                    if (target >= col0 && target < col0 + 32) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j == target) target_logit = l[j];
                        }
                    }
                    if (chunk_max != -INFINITY) {
                        const float m = fmaxf(run_max, chunk_max);
                        float s = run_sum * expf(run_max - m);
#pragma unroll
                        for (int j = 0; j < 32; ++j) s += expf(l[j] - m);
                        run_max = m;
                        run_sum = s;
                    }
                }
                if (row_ok && !logit_row && args.grad_out == nullptr) {
                    float *p = args.partials + (tile.n * args.lse_rows + row) * 3;
                    p[0] = run_max;
                    p[1] = run_sum;
                    p[2] = target_logit;
                }
            }
            }  // halves
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
            if (++acc == kAccBufs) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (kProblem == kOutput) {
        // every CTA's returned rows are stored: the last CTA raises this
        // owner's return flag in every sender's buffer
        if (args.ret_peers != nullptr) {
            peer::signal_peers(args.ret_own, args.ret_peers, 1, args.ret_rank, args.ret_ranks,
                               peer::current_epoch(args.ret_own), false);
        }
    }
    if constexpr (kProblem == kDenseCluster) {
        // Per 128-row half: the epilogue warps park the accumulator rows in
        // this CTA's shared memory (the stage ring is idle: every load was
        // consumed by the MMAs that acc_full covered), a cluster barrier, CTA r
        // sums column slice r over the splits through distributed shared
        // memory, a second barrier. Every thread of every CTA reaches every
        // cluster barrier, aborted or not.
        const bool have_tile = !*abort && blockIdx.x < tiles;
        const Tile tile = tile_at<kProblem, kTileRows>(args, blockIdx.x < tiles ? blockIdx.x : 0);
        const uint32_t rank = cluster_ctarank();
        const int64_t splits = args.splits;
        constexpr int kQuads = kBN / 4;
        const int q_begin = static_cast<int>(rank * kQuads / splits);
        const int q_count = static_cast<int>((rank + 1) * kQuads / splits) - q_begin;
        const T *bias = static_cast<const T *>(args.bias0);
        float *out = static_cast<float *>(args.out);
        const uint32_t parked_base = smem_addr(stages);
        for (int h = 0; h < kHalves; ++h) {
            const int64_t half_row0 = tile.row0 + h * kBM;
            // only the warps holding valid rows park them (a 32-row decode
            // batch fills one of the four lane quarters)
            if (have_tile && warp >= 2 && half_row0 + (warp & 3) * 32 < args.rows) {
                tc_fence_after();
                const int quarter = warp & 3;
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(h * kBN);
                float *parked = reinterpret_cast<float *>(stages) + (quarter * 32 + lane) * kAccStride;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t y[32];
                    KOEMI_TMEM_LD32(taddr + c * 32, y);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        reinterpret_cast<float4 *>(parked + c * 32)[q] =
                            make_float4(__uint_as_float(y[4 * q]), __uint_as_float(y[4 * q + 1]),
                                        __uint_as_float(y[4 * q + 2]), __uint_as_float(y[4 * q + 3]));
                    }
                }
            }
            cluster_sync_all();
            const int valid_rows = have_tile ? static_cast<int>(max(static_cast<int64_t>(0),
                                                                    min(static_cast<int64_t>(kBM), args.rows - half_row0)))
                                             : 0;
            // Thread t owns column quad q_begin + t % q_count (its bias read
            // once) and rows t / q_count + j * row_step; the loads of 32 / S
            // rows from every split are requested before any is summed.
            const int row_step = kThreads / q_count;
            const int my_row = threadIdx.x / q_count;
            const int q = q_begin + threadIdx.x % q_count;
            const int64_t col = tile.n * kBN + q * 4;
            if (my_row < row_step && col < args.n_out) {
                float bias4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (bias != nullptr) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) bias4[e] = col + e < args.n_out ? to_acc(bias[col + e]) : 0.0f;
                }
                float *dst_col = out + half_row0 * args.out_stride + col;
                switch (splits) {
                    case 2: reduce_parked_rows<2>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    case 3: reduce_parked_rows<3>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    case 4: reduce_parked_rows<4>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    case 5: reduce_parked_rows<5>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    case 6: reduce_parked_rows<6>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    case 7: reduce_parked_rows<7>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                    default: reduce_parked_rows<8>(parked_base, my_row, row_step, valid_rows, q, bias4, dst_col, args.out_stride, args.n_out - col); break;
                }
            }
            cluster_sync_all();
        }
        tc_fence_before();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemColumns));
    }
}

// ------------------------------------------------------------------- host

uint32_t make_idesc(int dtype, int n = kBN) {
    const uint32_t ab = dtype == KOEMI_BF16 ? 1u : 0u;  // 0 = f16, 1 = bf16
    uint32_t idesc = 0;
    idesc |= 1u << 4;                       // D format: f32
    idesc |= ab << 7;                       // A format
    idesc |= ab << 10;                      // B format
    idesc |= static_cast<uint32_t>(n >> 3) << 17;
    idesc |= static_cast<uint32_t>(kBM >> 4) << 24;
    return idesc;
}

int encode_kmajor(CUtensorMap *map, int dtype, const void *base, int64_t rows, int64_t k, uint32_t box_rows) {
    const CUtensorMapDataType type = dtype == KOEMI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k) * 2};
    const uint32_t box[2] = {kBK, box_rows};
    return encode_tensor_map(map, type, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int kProblem, bool kPair = false, int kTileN = kBN>
int launch(const UmmaArgs &args, int dtype, int64_t max_tiles, cudaStream_t stream) {
    auto kernel = dtype == KOEMI_BF16 ? umma_gemm_kernel<kProblem, __nv_bfloat16, kPair, kTileN>
                                      : umma_gemm_kernel<kProblem, __half, kPair, kTileN>;
    KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)));
    int64_t grid = sm_count();
    if (max_tiles < grid) grid = max_tiles > 0 ? max_tiles : 1;
    KOEMI_CUDA_TRY(launch_programmatic(args.weights_ready != 0, kernel, dim3(static_cast<unsigned>(grid)),
                                       dim3(threads_for<kProblem>()), kSmemBytes, stream, dim3(1, 1, 1), args));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

// Exactly `ctas` CTAs in clusters of `cluster` (one tile per CTA).
template <int kProblem, bool kPair = false>
int launch_clustered(const UmmaArgs &args, int dtype, int64_t ctas, int cluster, cudaStream_t stream) {
    auto kernel = dtype == KOEMI_BF16 ? umma_gemm_kernel<kProblem, __nv_bfloat16, kPair>
                                      : umma_gemm_kernel<kProblem, __half, kPair>;
    KOEMI_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)));
    KOEMI_CUDA_TRY(launch_programmatic(args.weights_ready != 0, kernel, dim3(static_cast<unsigned>(ctas)),
                                       dim3(threads_for<kProblem>()), kSmemBytes, stream,
                                       dim3(static_cast<unsigned>(cluster), 1, 1), args));
    KOEMI_LAUNCH_CHECK();
    return KOEMI_OK;
}

// CTAs of the dense cluster kernel that can be resident at once in clusters
// of `cluster` (GPC boundaries leave some SMs out), cached per device.
int64_t resident_cluster_ctas(int cluster) {
    static std::mutex mutex;
    static int64_t cache[64][9] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64 || cluster < 1 || cluster > 8) return 0;
    std::lock_guard<std::mutex> lock(mutex);
    if (cache[device][cluster] != 0) return cache[device][cluster];
    auto kernel = umma_gemm_kernel<kDenseCluster, __nv_bfloat16, false>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(cluster), 1, 1);
    config.blockDim = dim3(kThreads, 1, 1);
    config.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = static_cast<unsigned>(cluster);
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &config) != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
    }
    cache[device][cluster] = static_cast<int64_t>(clusters) * cluster;
    return cache[device][cluster];
}

bool umma_shape_ok(const void *p, int64_t k) { return k % 8 == 0 && aligned(p, 16) && k > 0; }

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

extern __global__ void zero_tail_rows_kernel(void *out, const int64_t *offsets, int64_t experts, int64_t pairs,
                                             int64_t row_bytes);

size_t grouped_mlp_umma_workspace(int64_t pairs, int64_t input_width, int64_t hidden_width, int64_t expert_count,
                                  int dtype) {
    (void)input_width;
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return 0;
    return align256((expert_count + 1) * sizeof(int32_t)) + align256(static_cast<size_t>(pairs) * hidden_width * 2);
}

int grouped_mlp_umma(const void *sorted_context, const int64_t *segment_offsets, const void *gate_w, const void *gate_b,
                     const void *value_w, const void *value_b, const void *out_w, const void *out_b, void *output,
                     int64_t pairs, int64_t input_width, int64_t hidden_width, int64_t expert_count, int dtype,
                     void *workspace, size_t workspace_bytes, cudaStream_t stream, bool *handled,
                     const int32_t *tile_prefix_in, bool zero_tail) {
    *handled = false;
    const int64_t d = input_width, h = hidden_width;
    if (!umma_shape_ok(sorted_context, d) || !umma_shape_ok(gate_w, d) || !umma_shape_ok(value_w, d) ||
        !umma_shape_ok(out_w, h) || pairs >= (int64_t(1) << 31) || expert_count * h >= (int64_t(1) << 31) ||
        expert_count * d >= (int64_t(1) << 31)) {
        return KOEMI_OK;  // the fp32 FMA path takes shapes TMA cannot describe
    }
    if (workspace_bytes < grouped_mlp_umma_workspace(pairs, d, h, expert_count, dtype)) {
        return fail(KOEMI_ERR_WORKSPACE, "grouped MLP tensor-core path needs more workspace");
    }
    char *ws = static_cast<char *>(workspace);
    const int32_t *prefix = tile_prefix_in;
    void *hidden = ws + align256((expert_count + 1) * sizeof(int32_t));
    if (prefix == nullptr) {  // the tile map of these segments (a caller may pass one it already has)
        int32_t *own_prefix = reinterpret_cast<int32_t *>(ws);
        KOEMI_CUDA_TRY(launch_pdl(tile_prefix_kernel, dim3(1), dim3(32), 0, stream, dim3(1, 1, 1), segment_offsets, expert_count, kBM, own_prefix));
        KOEMI_LAUNCH_CHECK();
        prefix = own_prefix;
    }
    const int64_t max_m_tiles = (pairs + kBM - 1) / kBM + expert_count;

    UmmaArgs g1{};
    int rc = encode_kmajor(&g1.map_a, dtype, sorted_context, pairs, d, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g1.map_b0, dtype, gate_w, expert_count * h, d, 128);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g1.map_b1, dtype, value_w, expert_count * h, d, 128);
    if (rc != KOEMI_OK) return rc;
    g1.k = d;
    g1.rows = pairs;
    g1.n_tiles = (h + 127) / 128;
    g1.b_rows_per_group = h;
    g1.n_out = h;
    g1.out_stride = h;
    g1.experts = expert_count;
    g1.offsets = segment_offsets;
    g1.tile_prefix = prefix;
    g1.bias0 = gate_b;
    g1.bias1 = value_b;
    g1.out = hidden;
    g1.status = device_status_word();
    g1.idesc = make_idesc(dtype);
    rc = launch<kGated>(g1, dtype, max_m_tiles * g1.n_tiles, stream);
    if (rc != KOEMI_OK) return rc;

    // Narrow (N = 128) output tiles when the 256-wide ones cannot fill the
    // SMs: with few pairs every touched expert has about one row tile, so the
    // row tiles are estimated by the number of experts the pairs can touch.
    const int64_t est_m_tiles = std::min(max_m_tiles, std::max((pairs + kBM - 1) / kBM, std::min(pairs, expert_count)));
    const bool narrow = est_m_tiles * ((d + kBN - 1) / kBN) < sm_count();
    const int64_t tile_n = narrow ? kBN / 2 : kBN;
    UmmaArgs g2{};
    rc = encode_kmajor(&g2.map_a, dtype, hidden, pairs, h, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g2.map_b0, dtype, out_w, expert_count * d, h, static_cast<uint32_t>(tile_n));
    if (rc != KOEMI_OK) return rc;
    g2.k = h;
    g2.rows = pairs;
    g2.n_tiles = (d + tile_n - 1) / tile_n;
    g2.b_rows_per_group = d;
    g2.n_out = d;
    g2.out_stride = d;
    g2.experts = expert_count;
    g2.offsets = segment_offsets;
    g2.tile_prefix = prefix;
    g2.bias0 = out_b;
    g2.out = output;
    g2.status = g1.status;
    g2.idesc = make_idesc(dtype, static_cast<int>(tile_n));
    rc = narrow ? launch<kOutput, false, kBN / 2>(g2, dtype, max_m_tiles * g2.n_tiles, stream)
                : launch<kOutput>(g2, dtype, max_m_tiles * g2.n_tiles, stream);
    if (rc != KOEMI_OK) return rc;
    if (zero_tail) {
        KOEMI_CUDA_TRY(launch_pdl(zero_tail_rows_kernel, dim3(256), dim3(256), 0, stream, dim3(1, 1, 1), output, segment_offsets, expert_count, pairs, d * 2));
        KOEMI_LAUNCH_CHECK();
    }
    *handled = true;
    return KOEMI_OK;
}

// The owner's grouped expert MLP of an expert-parallel exchange: the same two
// GEMMs as grouped_mlp_umma over the received rows in local expert order
// (tile map from the owner sort), with the output GEMM storing each row's
// result straight into its sender's exchange buffer and raising the return
// flags; no output tensor, no pad-row zeroing.
int expert_mlp_return_umma(const void *sorted_rows, const int64_t *segment_offsets, const int32_t *tile_prefix,
                           const int64_t *slots, const void *gate_w, const void *gate_b, const void *value_w,
                           const void *value_b, const void *out_w, const void *out_b, int64_t rows, int64_t d,
                           int64_t h, int64_t local_experts, int dtype, void *hidden, const uint64_t *peers,
                           uint8_t *own, size_t ret_offset, int64_t rank, int64_t ranks, int64_t capacity,
                           cudaStream_t stream) {
    const int64_t max_m_tiles = (rows + kBM - 1) / kBM + local_experts;
    UmmaArgs g1{};
    int rc = encode_kmajor(&g1.map_a, dtype, sorted_rows, rows, d, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g1.map_b0, dtype, gate_w, local_experts * h, d, 128);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g1.map_b1, dtype, value_w, local_experts * h, d, 128);
    if (rc != KOEMI_OK) return rc;
    g1.k = d;
    g1.rows = rows;
    g1.n_tiles = (h + 127) / 128;
    g1.b_rows_per_group = h;
    g1.n_out = h;
    g1.out_stride = h;
    g1.experts = local_experts;
    g1.offsets = segment_offsets;
    g1.tile_prefix = tile_prefix;
    g1.bias0 = gate_b;
    g1.bias1 = value_b;
    g1.out = hidden;
    g1.status = device_status_word();
    g1.idesc = make_idesc(dtype);
    rc = launch<kGated>(g1, dtype, max_m_tiles * g1.n_tiles, stream);
    if (rc != KOEMI_OK) return rc;
    // narrow output tiles when the 256-wide ones cannot fill the SMs (as in
    // grouped_mlp_umma, with the received slots as the pair count)
    const int64_t est_m_tiles = std::min(max_m_tiles, std::max((rows + kBM - 1) / kBM, std::min(rows, local_experts)));
    const bool narrow = est_m_tiles * ((d + kBN - 1) / kBN) < sm_count();
    const int64_t tile_n = narrow ? kBN / 2 : kBN;
    UmmaArgs g2{};
    rc = encode_kmajor(&g2.map_a, dtype, hidden, rows, h, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&g2.map_b0, dtype, out_w, local_experts * d, h, static_cast<uint32_t>(tile_n));
    if (rc != KOEMI_OK) return rc;
    g2.k = h;
    g2.rows = rows;
    g2.n_tiles = (d + tile_n - 1) / tile_n;
    g2.b_rows_per_group = d;
    g2.n_out = d;
    g2.out_stride = d;
    g2.experts = local_experts;
    g2.offsets = segment_offsets;
    g2.tile_prefix = tile_prefix;
    g2.bias0 = out_b;
    g2.out = nullptr;
    g2.ret_peers = peers;
    g2.ret_own = own;
    g2.ret_slots = slots;
    g2.ret_offset = static_cast<int64_t>(ret_offset);
    g2.ret_capacity = capacity;
    g2.ret_rank = rank;
    g2.ret_ranks = ranks;
    g2.status = g1.status;
    g2.idesc = make_idesc(dtype, static_cast<int>(tile_n));
    // the return flags need every CTA of the launch to reach the end, so the
    // grid is at least one CTA even when no tile exists
    return narrow ? launch<kOutput, false, kBN / 2>(g2, dtype, max_m_tiles * g2.n_tiles, stream)
                  : launch<kOutput>(g2, dtype, max_m_tiles * g2.n_tiles, stream);
}

// K splits of a dense projection: the largest S <= 8 whose tiles x S CTAs
// are resident at once in clusters of S, with at least 4 K blocks per split.
// A rows per surprise tile: 129..256 rows (a decode batch) run as one paired
// tile per vocabulary slice, so every head byte crosses L2 -> SM once instead
// of once per 128-row tile, in one wave. Longer inputs keep 128-row tiles
// and the double-buffered accumulators (an epilogue overlaps the next tile's
// MMAs), which measured faster there, as did 128-row tiles for the K-split
// dense projections (their shorter main loops gain less than the paired
// epilogue costs).
int64_t surprise_tile_rows(int64_t rows) { return rows > kBM && rows <= 2 * kBM ? 2 * kBM : kBM; }

int64_t dense_splits(int64_t rows, int64_t n, int64_t k) {
    const int64_t tiles = ((rows + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
    const int64_t k_blocks = (k + kBK - 1) / kBK;
    for (int64_t splits = 8; splits > 1; --splits) {
        if (k_blocks < 4 * splits) continue;
        if (tiles * splits <= resident_cluster_ctas(static_cast<int>(splits))) return splits;
    }
    return 1;
}

int64_t surprise_umma_slices(int64_t rows, int64_t width, int64_t content_vocab, int dtype) {
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return 0;
    if (width % 8 != 0 || rows <= 0 || content_vocab >= (int64_t(1) << 31)) return 0;
    return (content_vocab + kBN - 1) / kBN;
}

int surprise_umma_forward(const void *prior, const void *weight, const void *bias, const int64_t *targets,
                          int64_t rows, int64_t width, int64_t content_vocab, int dtype, float *partials,
                          int64_t slices, cudaStream_t stream, bool *handled) {
    *handled = false;
    if (!umma_shape_ok(prior, width) || !umma_shape_ok(weight, width) || rows >= (int64_t(1) << 31) ||
        slices != surprise_umma_slices(rows, width, content_vocab, dtype)) {
        return KOEMI_OK;
    }
    UmmaArgs a{};
    int rc = encode_kmajor(&a.map_a, dtype, prior, rows, width, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&a.map_b0, dtype, weight, content_vocab, width, kBN);
    if (rc != KOEMI_OK) return rc;
    a.k = width;
    a.rows = rows;
    a.n_tiles = slices;
    a.b_rows_per_group = 0;
    a.n_out = content_vocab;
    a.out_stride = 0;
    a.experts = 1;
    a.bias0 = bias;
    a.partials = partials;
    a.targets = targets;
    a.lse_rows = rows;
    a.pad_column = -1;
    a.status = device_status_word();
    a.idesc = make_idesc(dtype);
    const bool pair = surprise_tile_rows(rows) > kBM;
    a.band = 16;
    const int64_t tiles = ((rows + surprise_tile_rows(rows) - 1) / surprise_tile_rows(rows)) * slices;
    rc = pair ? launch<kSurprise, true>(a, dtype, tiles, stream) : launch<kSurprise, false>(a, dtype, tiles, stream);
    if (rc != KOEMI_OK) return rc;
    *handled = true;
    return KOEMI_OK;
}

// dlogits of the causal surprise on tensor cores: the logits tile recomputed
// by the MMAs, then scale_r * (exp(l - lse_r) - onehot(target_r)) stored as
// fp32 [rows, content_vocab]. False in *handled when TMA cannot describe the
// operands (the FMA kernel takes those).
int surprise_grad_umma(const void *prior, const void *weight, const void *bias, const int64_t *targets,
                       const float *row_lse, const float *row_scale, float *dlogits, int64_t rows, int64_t width,
                       int64_t content_vocab, int dtype, cudaStream_t stream, bool *handled) {
    *handled = false;
    if ((dtype != KOEMI_BF16 && dtype != KOEMI_F16) || !umma_shape_ok(prior, width) || !umma_shape_ok(weight, width) ||
        rows >= (int64_t(1) << 31) || content_vocab >= (int64_t(1) << 31)) {
        return KOEMI_OK;
    }
    UmmaArgs a{};
    int rc = encode_kmajor(&a.map_a, dtype, prior, rows, width, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&a.map_b0, dtype, weight, content_vocab, width, kBN);
    if (rc != KOEMI_OK) return rc;
    const int64_t slices = (content_vocab + kBN - 1) / kBN;
    a.k = width;
    a.rows = rows;
    a.n_tiles = slices;
    a.n_out = content_vocab;
    a.experts = 1;
    a.bias0 = bias;
    a.targets = targets;
    a.lse_rows = rows;
    a.pad_column = -1;
    a.row_lse = row_lse;
    a.row_scale = row_scale;
    a.grad_out = dlogits;
    a.status = device_status_word();
    a.idesc = make_idesc(dtype);
    a.band = 16;
    const bool pair = surprise_tile_rows(rows) > kBM;
    const int64_t tiles = ((rows + surprise_tile_rows(rows) - 1) / surprise_tile_rows(rows)) * slices;
    rc = pair ? launch<kSurprise, true>(a, dtype, tiles, stream) : launch<kSurprise, false>(a, dtype, tiles, stream);
    if (rc == KOEMI_OK) *handled = true;
    return rc;
}

int head_pass_umma(const void *rows_in, int64_t lse_rows, int64_t logit_rows, int64_t width, const void *weight,
                   const void *bias, int64_t vocab, int64_t pad_id, float *partials, float *logits, int dtype,
                   cudaStream_t stream) {
    const int64_t rows = lse_rows + logit_rows;
    UmmaArgs a{};
    int rc = encode_kmajor(&a.map_a, dtype, rows_in, rows, width, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&a.map_b0, dtype, weight, vocab, width, kBN);
    if (rc != KOEMI_OK) return rc;
    const int64_t slices = (vocab + kBN - 1) / kBN;
    a.k = width;
    a.rows = rows;
    a.n_tiles = slices;
    a.n_out = vocab;
    a.out_stride = vocab;
    a.experts = 1;
    a.bias0 = bias;
    a.out = logits;
    a.partials = partials;
    a.targets = nullptr;
    a.lse_rows = lse_rows;
    a.pad_column = pad_id;
    a.status = device_status_word();
    a.idesc = make_idesc(dtype);
    a.band = 16;
    const bool pair = surprise_tile_rows(rows) > kBM;
    const int64_t tiles = ((rows + surprise_tile_rows(rows) - 1) / surprise_tile_rows(rows)) * slices;
    return pair ? launch<kSurprise, true>(a, dtype, tiles, stream) : launch<kSurprise, false>(a, dtype, tiles, stream);
}

}  // namespace koemi

using namespace koemi;

extern "C" int64_t koemi_think_head_pass_slices(int64_t vocab) { return vocab < 1 ? 0 : (vocab + kBN - 1) / kBN; }

extern "C" int koemi_think_head_pass(const void *rows, int64_t lse_rows, int64_t logit_rows, int64_t width,
                                     const void *head_weight, const void *head_bias, int64_t vocab, int64_t pad_id,
                                     float *partials, float *logits, int dtype, void *stream) {
    clear_error();
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return fail(KOEMI_ERR_INVALID, "the head pass takes bf16 or f16 operands");
    if (lse_rows < 0 || logit_rows < 0 || width < 1 || vocab < 2) return fail(KOEMI_ERR_INVALID, "bad head pass sizes");
    if (lse_rows + logit_rows == 0) return KOEMI_OK;
    if (width % 8 != 0 || !aligned(rows, 16) || !aligned(head_weight, 16) || head_bias == nullptr ||
        lse_rows + logit_rows >= (int64_t(1) << 31) || vocab >= (int64_t(1) << 31)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the head pass needs width a multiple of 8, 16-byte aligned rows and head, and a bias");
    }
    if ((lse_rows > 0 && partials == nullptr) || (logit_rows > 0 && logits == nullptr)) {
        return fail(KOEMI_ERR_INVALID, "partials (surprise rows) and logits (logit rows) must be non-NULL");
    }
    return head_pass_umma(rows, lse_rows, logit_rows, width, head_weight, head_bias, vocab, pad_id, partials, logits,
                          dtype, as_stream(stream));
}

namespace {
struct DensePlan {
    int64_t splits;
    int64_t k_per_split;
};
// Measured alternatives that lost at decode sizes: full-K N = 64 / 128 tiles
// without a reduction (every narrow tile re-reads all activation rows from L2:
// gates 13.8 -> 17.0 us at 256 rows), a push-style reduction through
// distributed shared memory (13.8 -> 24.7 us), and swapped operands (weight
// rows as M = 128, activation rows as N): without K splits only n / 128 SMs
// run the MMAs (gates 22.2 us at 256 rows), with splits the parked
// accumulator is as large as here (gates 19.6 us at 256 rows, 9.0 us vs
// 8.8 us at 32 rows).
DensePlan dense_plan(int64_t rows, int64_t n, int64_t k) {
    const int64_t k_blocks = (k + kBK - 1) / kBK;
    const int64_t wanted = dense_splits(rows, n, k);
    const int64_t per = (k_blocks + wanted - 1) / wanted;
    return DensePlan{(k_blocks + per - 1) / per, per};
}
}  // namespace

extern "C" int koemi_grouped_projection(const void *a, const void *b, float *out, int64_t groups,
                                        int64_t rows_per_group, int64_t n, int64_t k, int dtype, void *stream) {
    clear_error();
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return fail(KOEMI_ERR_INVALID, "grouped projection takes bf16 or f16 operands");
    if (groups < 0 || rows_per_group < 1 || n < 1 || k < 1) return fail(KOEMI_ERR_INVALID, "bad grouped projection sizes");
    if (groups == 0) return KOEMI_OK;
    if (k % 8 != 0 || !aligned(a, 16) || !aligned(b, 16) || groups * rows_per_group >= (int64_t(1) << 31) ||
        groups * n >= (int64_t(1) << 31)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "grouped projection needs K a multiple of 8 and 16-byte aligned operands");
    }
    UmmaArgs args{};
    int rc = encode_kmajor(&args.map_a, dtype, a, groups * rows_per_group, k, kBM);
    if (rc == KOEMI_OK) rc = encode_kmajor(&args.map_b0, dtype, b, groups * n, k, kBN);
    if (rc != KOEMI_OK) return rc;
    const int64_t k_blocks = (k + kBK - 1) / kBK;
    args.k = k;
    args.rows = groups * rows_per_group;
    args.group_rows = rows_per_group;
    args.n_tiles = (n + kBN - 1) / kBN;
    args.b_rows_per_group = n;
    args.n_out = n;
    args.out_stride = n;
    args.experts = groups;
    args.splits = 1;
    args.k_per_split = k_blocks;
    args.bias0 = nullptr;
    args.out = out;
    args.status = device_status_word();
    args.idesc = make_idesc(dtype);
    const int64_t tiles = groups * ((rows_per_group + kBM - 1) / kBM) * args.n_tiles;
    return launch<kDense>(args, dtype, tiles, as_stream(stream));
}

extern "C" size_t koemi_dense_projection_workspace(int64_t rows, int64_t n, int64_t k, int dtype) {
    // the K splits are reduced in distributed shared memory: no scratch
    (void)rows;
    (void)n;
    (void)k;
    (void)dtype;
    return 256;
}

namespace {
int dense_projection(const void *a, int64_t a_stride, const void *weight, const void *bias, float *out,
                     int64_t out_stride, int64_t rows, int64_t n, int64_t k, int dtype, void *stream,
                     bool weights_ready) {
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return fail(KOEMI_ERR_INVALID, "dense projection takes bf16 or f16 operands");
    if (rows < 0 || n < 1 || k < 1) return fail(KOEMI_ERR_INVALID, "need rows >= 0 and positive n, k");
    if (rows == 0) return KOEMI_OK;
    if (k % 8 != 0 || a_stride < k || a_stride % 8 != 0 || !aligned(a, 16) || !aligned(weight, 16) ||
        rows >= (int64_t(1) << 31) || n >= (int64_t(1) << 31)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "dense projection needs K and the A row stride to be multiples of 8 and 16-byte aligned operands");
    }
    const DensePlan plan = dense_plan(rows, n, k);
    cudaStream_t s = as_stream(stream);
    UmmaArgs args{};
    const CUtensorMapDataType type = dtype == KOEMI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rows)};
        const uint64_t strides[1] = {static_cast<uint64_t>(a_stride) * 2};
        const uint32_t box[2] = {kBK, kBM};
        int rc = encode_tensor_map(&args.map_a, type, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != KOEMI_OK) return rc;
    }
    int rc = encode_kmajor(&args.map_b0, dtype, weight, n, k, kBN);
    if (rc != KOEMI_OK) return rc;
    args.k = k;
    args.rows = rows;
    args.n_tiles = (n + kBN - 1) / kBN;
    args.n_out = n;
    args.out_stride = out_stride;
    args.experts = 1;
    args.splits = plan.splits;
    args.k_per_split = plan.k_per_split;
    args.bias0 = bias;
    args.out = out;
    args.partials = nullptr;
    args.status = device_status_word();
    args.idesc = make_idesc(dtype);
    args.weights_ready = weights_ready ? 1 : 0;
    const int64_t m_tiles = (rows + kBM - 1) / kBM;
    const int64_t tiles = m_tiles * args.n_tiles * plan.splits;
    if (plan.splits > 1) return launch_clustered<kDenseCluster>(args, dtype, tiles, static_cast<int>(plan.splits), s);
    if (m_tiles >= 32) {
        // prefill-sized row counts: paired 256-row tiles (two M = 128 MMAs
        // share every weight stage, halving the weight bytes each MMA needs
        // from L2) in bands of 8 paired row tiles, N walked inside a band so
        // the CTAs running together reuse the band's activations from L2
        args.band = 8;
        return launch<kDense, true>(args, dtype, ((rows + 2 * kBM - 1) / (2 * kBM)) * args.n_tiles, s);
    }
    return launch<kDense>(args, dtype, tiles, s);
}
}  // namespace

extern "C" int koemi_dense_projection(const void *a, int64_t a_stride, const void *weight, const void *bias,
                                      float *out, int64_t out_stride, int64_t rows, int64_t n, int64_t k, int dtype,
                                      void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    (void)workspace;
    (void)workspace_bytes;
    return dense_projection(a, a_stride, weight, bias, out, out_stride, rows, n, k, dtype, stream, false);
}

extern "C" int koemi_dense_projection_resident(const void *a, int64_t a_stride, const void *weight, const void *bias,
                                               float *out, int64_t out_stride, int64_t rows, int64_t n, int64_t k,
                                               int dtype, void *workspace, size_t workspace_bytes, void *stream) {
    clear_error();
    (void)workspace;
    (void)workspace_bytes;
    return dense_projection(a, a_stride, weight, bias, out, out_stride, rows, n, k, dtype, stream, true);
}

extern "C" int koemi_ep_expert_mlp_return(const void *sorted_rows, const int64_t *segment_offsets,
                                          const int32_t *tile_prefix, const int64_t *slots, const void *gate_weights,
                                          const void *gate_biases, const void *value_weights,
                                          const void *value_biases, const void *output_weights,
                                          const void *output_biases, int64_t rows, int64_t input_width,
                                          int64_t hidden_width, int64_t local_experts, int dtype, void *workspace,
                                          size_t workspace_bytes, const uint64_t *peers, void *own, int64_t rank,
                                          int64_t ranks, int64_t capacity, void *stream) {
    clear_error();
    if (dtype != KOEMI_BF16 && dtype != KOEMI_F16) return fail(KOEMI_ERR_INVALID, "the returning expert MLP takes bf16 or f16 rows");
    if (rows < 1 || input_width < 1 || hidden_width < 1 || local_experts < 1 || capacity < 1 || ranks < 1 ||
        ranks > peer::kMaxRanks || rank < 0 || rank >= ranks || rows > ranks * capacity) {
        return fail(KOEMI_ERR_INVALID, "bad returning expert MLP sizes");
    }
    if (sorted_rows == nullptr || segment_offsets == nullptr || tile_prefix == nullptr || slots == nullptr ||
        peers == nullptr || own == nullptr || !aligned(own, 256)) {
        return fail(KOEMI_ERR_INVALID, "returning expert MLP pointers must be non-NULL (own 256-byte aligned)");
    }
    if (!umma_shape_ok(sorted_rows, input_width) || !umma_shape_ok(gate_weights, input_width) ||
        !umma_shape_ok(value_weights, input_width) || !umma_shape_ok(output_weights, hidden_width) ||
        rows >= (int64_t(1) << 31) || local_experts * hidden_width >= (int64_t(1) << 31) ||
        local_experts * input_width >= (int64_t(1) << 31)) {
        return fail(KOEMI_ERR_UNSUPPORTED, "the returning expert MLP needs widths that are multiples of 8 and 16-byte aligned operands");
    }
    const size_t hidden_bytes = static_cast<size_t>(rows) * static_cast<size_t>(hidden_width) * 2;
    if (workspace == nullptr || workspace_bytes < hidden_bytes || !aligned(workspace, 16)) {
        return fail(KOEMI_ERR_WORKSPACE, "the returning expert MLP needs %zu workspace bytes (16-byte aligned)", hidden_bytes);
    }
    const peer::Layout l = peer::layout(ranks, capacity, input_width, 2);
    return expert_mlp_return_umma(sorted_rows, segment_offsets, tile_prefix, slots, gate_weights, gate_biases,
                                  value_weights, value_biases, output_weights, output_biases, rows, input_width,
                                  hidden_width, local_experts, dtype, workspace, peers, static_cast<uint8_t *>(own),
                                  l.ret, rank, ranks, capacity, as_stream(stream));
}
