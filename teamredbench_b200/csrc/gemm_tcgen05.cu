// gemm_tcgen05.cu -- dense GEMM C = A * B on B200 5th-gen tensor cores.
//
// Replaces the reference's mfma_gemm_lowp_kernel / mfma_gemm_highp_kernel
// (src/teamredbench/native/kernels/mfu_gemm_lowp.hip.hpp:134-334,
// mfu_gemm_highp.hip.hpp:39-218) and, for result semantics, the torch path's
// torch.mm(a, b, out=out) (src/teamredbench/benchmarks/mfu.py:229-234).
//
// Design (kernel templates shared by all five input types):
//  * persistent grid, one 192-thread CTA per SM (or CTA pair), static tile
//    schedule with grouped rasterisation (group m-blocks share each B column
//    panel in L2);
//  * single-CTA tiles 128 x BN (BN = 256, 128, 64) and 256 x 256 CTA-pair
//    tiles (cta_group::2); K moves in k-blocks of 128 bytes (64 bf16/f16, 32
//    tf32, 128 e4m3/int8) through a ~192 KiB shared-memory ring fed by TMA (no
//    multicast), several k-blocks per stage for the narrow tiles;
//  * warp 0: TMA producer; warp 1: a single thread issues tcgen05.mma (32 K
//    bytes per instruction) into a TMEM accumulator; warps 2-5: epilogue
//    (tcgen05.ld -> convert -> shared staging -> TMA store for whole tiles);
//  * two TMEM accumulators so the epilogue of tile i overlaps the main loop
//    of tile i+1;
//  * skinny problems (one row of tiles) use cluster split-K over distributed
//    shared memory, or the swapped-operand kernel for M <= 64;
//  * A is row-major (K-major operand, 128B swizzle); B is row-major K x N,
//    i.e. an MN-major operand, consumed directly through the MN-major 128B
//    swizzle layout (no re-layout pass: the reference needed an untimed
//    pack_b_tiles_kernel, mfu_gemm_lowp.hip.hpp:82-132, this kernel does not);
//  * every mbarrier wait is bounded (trb::kWaitTimeoutNs); a wait that gives
//    up records a code in g_gemm_error, raises a CTA-wide abort flag, drains
//    its own in-flight TMA / MMA work and frees TMEM before returning.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "trb_common.cuh"

namespace trb {
namespace gemm {

__device__ int g_gemm_error;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBKBytes = 128;       // K bytes per stage: one 128-byte swizzle row
constexpr int kInstrKBytes = 32;    // K bytes consumed by one tcgen05.mma
constexpr int kKSteps = kBKBytes / kInstrKBytes;
constexpr int kStages = 4;
constexpr int kAStage = kBM * kBKBytes;  // 16 KiB
constexpr int kBStage = kBN * kBKBytes;  // 32 KiB
constexpr int kNumAcc = 2;
constexpr int kTmemCols = kNumAcc * kBN;  // 512
constexpr int kThreads = 192;

// Single-CTA tile-width variants: BN = 256 (default), 128 and 64 (skinny
// problems: M <= 128 gives one row of tiles, so a narrow N tile is what puts
// every SM to work).  The ring is as deep as the 227 KiB of shared memory
// allows; TMEM holds two BN-column accumulators.
// KD k-blocks share one ring stage (one full/empty barrier round trip).  A
// one-k-block stage of a 64- or 128-wide tile holds only 4 MMAs' worth of
// work (~140 ns), less than the MMA thread's per-stage cost on B200 (~260 ns
// measured with a 4-MMA stage), so the 128-wide ring takes 2 k-blocks per
// stage (3 stages) and the 64-wide ring 4 (2 stages): 1024^3 bf16 went from
// 6.9 to 6.0 (2 per stage) and 5.8 us (4 per stage).  Cluster split-K runs
// (one row of tiles, an HBM stream of B) keep the deeper one-k-block ring
// for 16- and 32-bit types, where the MMAs keep up with HBM anyway (M = 128,
// N = K = 8192: 28.1 us against 28.7 with 2 per stage); 8-bit types, whose
// k-blocks carry twice the K, take 2 per stage there (13.7 against 14.4 us).
__host__ __device__ constexpr int tile_kd(int bn, int cl, int es) {
    return bn == 256 ? 1 : cl > 1 ? (es == 1 ? 2 : 1) : (bn == 64 ? 4 : 2);
}

template <int BN, int KD, int EPI>
struct TileCfg {
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
    static_assert(KD == 1 || KD == 2 || KD == 4, "k-blocks per stage");
    static constexpr int kKD = KD;
    static constexpr int kEpiBytes = EPI;  // TMA-store staging after the ring
    static constexpr int kBStage = BN * kBKBytes;  // one k-block of B
    static constexpr int kStageBytes = kKD * (kAStage + kBStage);
    static constexpr int kStages = (210 * 1024) / kStageBytes > 8 ? 8 : (210 * 1024) / kStageBytes;
    static constexpr int kTmemCols = kNumAcc * BN;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + EPI;
};

// Instruction descriptor (kind::f16 / tf32 / f8f6f4 / i8): D format, A/B formats,
// A K-major (bit 15 = 0), B MN-major (bit 16 = 1), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt) {
    return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (0u << 15) | (1u << 16) |
           ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}
// Same descriptor with B switched to K-major (bit 16 cleared).
__host__ __device__ constexpr uint32_t idesc_b_kmajor(uint32_t idesc) { return idesc & ~(1u << 16); }
// Same descriptor with instruction N = n (bits [17,23) hold N >> 3).
__host__ __device__ constexpr uint32_t idesc_with_n(uint32_t idesc, int n) {
    return (idesc & ~(0x3Fu << 17)) | ((uint32_t)(n >> 3) << 17);
}

// Per-input-type traits.  kind: 0 f16, 1 tf32, 2 f8f6f4, 3 i8.
// B (MN-major) smem layout: 128-byte swizzle with 16-byte atoms (descriptor
// layout type 2, 8-row period, SBO = 1024) for 8/16-bit types; tf32 MN-major
// operands only exist in the 128-byte swizzle with 32-byte atoms (layout type
// 1, 4-row period, SBO = 512), loaded with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
struct BLayout16 {
    static constexpr uint32_t kLayoutType = 2, kSbo = 1024;
    static constexpr CUtensorMapSwizzle kTmaSwizzle = CU_TENSOR_MAP_SWIZZLE_128B;
};
struct BLayout32 {
    static constexpr uint32_t kLayoutType = 1, kSbo = 512;
    static constexpr CUtensorMapSwizzle kTmaSwizzle = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
};

template <int DT>
struct Traits;
template <>
struct Traits<TRB_BFLOAT16> {
    using BLayout = BLayout16;
    static constexpr int kEsize = 2, kKind = 0;
    static constexpr uint32_t kIdesc = make_idesc(1, 1, 1);  // F32 <- BF16 x BF16
};
template <>
struct Traits<TRB_FLOAT16> {
    using BLayout = BLayout16;
    static constexpr int kEsize = 2, kKind = 0;
    static constexpr uint32_t kIdesc = make_idesc(1, 0, 0);  // F32 <- F16 x F16
};
template <>
struct Traits<TRB_TFLOAT32> {
    using BLayout = BLayout32;
    static constexpr int kEsize = 4, kKind = 1;
    static constexpr uint32_t kIdesc = make_idesc(1, 2, 2);  // F32 <- TF32 x TF32
};
template <>
struct Traits<TRB_FLOAT8_E4M3FN> {
    using BLayout = BLayout16;
    static constexpr int kEsize = 1, kKind = 2;
    static constexpr uint32_t kIdesc = make_idesc(1, 0, 0);  // F32 <- E4M3 x E4M3
};
template <>
struct Traits<TRB_INT8> {
    using BLayout = BLayout16;
    static constexpr int kEsize = 1, kKind = 3;
    static constexpr uint32_t kIdesc = make_idesc(2, 1, 1);  // S32 <- S8 x S8
};

// Shared-memory matrix descriptor, sm100 version (bit 46), swizzled layout
// type at [61,64) (2 = 128B swizzle, 1 = 128B swizzle with 32B atoms).
// Addresses and offsets are in 16-byte units.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint32_t layout_type = 2) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout_type << 61;
    return d;
}

template <int KIND>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if constexpr (KIND == 0) mma_f16(d, a, b, idesc, acc);
    else if constexpr (KIND == 1) mma_tf32(d, a, b, idesc, acc);
    else if constexpr (KIND == 2) mma_f8f6f4(d, a, b, idesc, acc);
    else mma_i8(d, a, b, idesc, acc);
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb, int& nb) {
    const int kGroupM = group_m > 0 ? group_m : 16;
    const int group = kGroupM * num_n;
    const int g = tile / group;
    const int first_m = g * kGroupM;
    const int gm = min(num_m - first_m, kGroupM);
    const int local = tile - g * group;
    mb = first_m + local % gm;
    nb = local / gm;
    // Serpentine: odd groups walk the columns backwards, so the first tiles of a
    // group reuse the B panels the previous group's last tiles left in L2.
    if (g & 1) nb = num_n - 1 - nb;
}

// Output element bytes: bf16 for bf16 / e4m3 inputs, f16 for f16, f32 for
// tf32, s32 for int8.
template <int DT>
__host__ __device__ constexpr int out_esize() {
    return (DT == TRB_TFLOAT32 || DT == TRB_INT8) ? 4 : 2;
}

// 32 fp32 accumulator words of one row -> 16 words of packed bf16 / f16 pairs
// (e4m3 results scaled by out_scale first).
template <int DT>
__device__ __forceinline__ void convert16(const uint32_t (&r)[32], float out_scale, uint32_t (&w)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float lo = __uint_as_float(r[2 * i]), hi = __uint_as_float(r[2 * i + 1]);
        if constexpr (DT == TRB_FLOAT8_E4M3FN) {
            lo *= out_scale;
            hi *= out_scale;
        }
        if constexpr (DT == TRB_FLOAT16) {
            __half2 h = __floats2half2_rn(lo, hi);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
            __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
    }
}

// Convert 32 accumulator words of one row and store them at C[row, col .. col+31].
template <int DT>
__device__ __forceinline__ void store_chunk(void* C, int row, int col, int N, const uint32_t (&r)[32],
                                            float out_scale) {
    const bool full = col + 32 <= N;
    if constexpr (out_esize<DT>() == 2) {
        uint16_t* out = static_cast<uint16_t*>(C) + (size_t)row * N + col;
        uint32_t w[16];
        convert16<DT>(r, out_scale, w);
        if (full) {
            uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
            for (int i = 0; i < 4; ++i) o4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col + i < N) out[i] = (uint16_t)(w[i >> 1] >> ((i & 1) * 16));
        }
    } else {  // tf32 -> f32, int8 -> s32: raw 32-bit words
        uint32_t* out = static_cast<uint32_t*>(C) + (size_t)row * N + col;
        if (full) {
            uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
            for (int i = 0; i < 8; ++i) o4[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col + i < N) out[i] = r[i];
        }
    }
}

// TMA-store epilogue of whole (unsplit) tiles.  Each epilogue warp owns 32
// TMEM lanes (rows) and writes its rows 32 columns at a time: convert, place
// the 32 x 32 box in shared memory in the C tensor map's swizzle, and one lane
// stores it with cp.async.bulk.tensor, which writes whole sectors and lets the
// warp go on to the next box (two staging buffers per warp).  Rows or columns
// past M / N are clipped by the store.  Stores of 16 bytes per row per lane
// straight from registers cost 11-13% of a 128 x 256 tile's time at 2048^3 and
// 4096^3 bf16 (measured by dropping them).
template <int DT>
__host__ __device__ constexpr int epi_box_bytes() {
    return 32 * 32 * out_esize<DT>();
}
template <int DT>
__host__ __device__ constexpr int epi_bytes() {
    return 4 * 2 * epi_box_bytes<DT>();  // 4 epilogue warps x 2 buffers
}

// Shared-memory plan of gemm_tcgen05_kernel<DT, *, BN, CL>.  Cluster split-K
// runs store through the exchange path and need no staging; 64-wide tiles
// keep direct stores (two boxes per warp per tile, where waiting for the
// last store before exit outweighs the gain: 1024^3 bf16 5.78 against 5.69 us).
template <int DT, int BN, int CL>
using TileCfgFor = TileCfg<BN, tile_kd(BN, CL, Traits<DT>::kEsize), (CL == 1 && BN >= 128) ? epi_bytes<DT>() : 0>;

// Row `row` (0..31) of a staging box at `buf` (1 KiB aligned): 16-bit outputs
// are 64-byte rows in the 64-byte swizzle (16-byte chunk j at j ^ ((row >> 1) & 3)),
// 32-bit outputs 128-byte rows in the 128-byte swizzle (chunk j at j ^ (row & 7)),
// the layouts CU_TENSOR_MAP_SWIZZLE_64B / _128B read.  A warp's stores of one
// chunk index then fill whole shared-memory wavefronts.
template <int DT>
__device__ __forceinline__ void stage_row(uint32_t buf, int row, const uint32_t (&r)[32], float out_scale) {
    if constexpr (out_esize<DT>() == 2) {
        uint32_t w[16];
        convert16<DT>(r, out_scale, w);
        const uint32_t base = buf + (uint32_t)(row * 64);
        const int sw = (row >> 1) & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            st_shared_v4(base + (uint32_t)((j ^ sw) * 16), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    } else {  // tf32 -> f32, int8 -> s32: raw 32-bit words
        const uint32_t base = buf + (uint32_t)(row * 128);
        const int sw = row & 7;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            st_shared_v4(base + (uint32_t)((j ^ sw) * 16), r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    }
}

// Split-K parameters.  With splits == 1 each work unit is one output tile and
// the epilogue stores C directly.  With splits > 1 a unit is (tile, split):
// its k-block range is [split * kb_per_split, min(.. + kb_per_split, num_kb)),
// the epilogue writes an fp32 partial to ws[unit] (kBM x kBN floats), and the
// last unit of a tile to finish (per-tile arrival counter) sums the partials
// of splits 0..S-1 in that fixed order -- deterministic -- then writes C and
// resets the counter to 0 for the next launch.
struct SplitK {
    int splits;
    int kb_per_split;
    float* ws;
    unsigned int* counters;
    int rotate_k;  // 1: start each tile's K loop at k-block (tile % nk) and wrap
    int group_m;   // m-blocks per raster group (consecutive tiles walk down a group's column)
    int chunk_kb;  // > 0: K-chunked accumulation, chunk_kb k-blocks per chain (below); 0: one chain per unit
};

// ---- K-chunked accumulation (tf32 inputs: tf32 and the float32 path) ----
// The tensor core's fp32 accumulation error grows with the length of one
// accumulation chain.  Measured on B200 with tf32-exact N(0,1)/sqrt(K) inputs
// (max |C - C_fp64| / max |C_fp64|, K-chunks of one chain): 5.2e-6 for 2048 K
// elements, 8.0e-6 for ~2730, 1.1e-5 for 4096, 2.2e-5 for 8192 -- and cuBLAS's
// tf32 GEMM gives the same 2.2e-5 at K = 8192.  With chunk_kb > 0 a unit's K
// range runs as chunks of chunk_kb k-blocks: the MMA thread accumulates each
// chunk from zero into the TMEM accumulator the previous chunk did not use,
// and the epilogue folds every completed chunk into the running sum held in
// the other accumulator, cur += prev in fp32 on the CUDA cores (round to
// nearest), then frees prev for the chunk after next.  The last chunk's
// accumulator then holds the unit's sum and takes the usual epilogue path.
// Chunks count k-block positions from the unit's start, so the chains -- and
// the bits of the result -- do not depend on the launch shape.
__host__ __device__ __forceinline__ int unit_chunks(int nk, int chunk_kb) {
    return chunk_kb > 0 && nk > chunk_kb ? (nk + chunk_kb - 1) / chunk_kb : 1;
}
// k-blocks per accumulation chain: 64 k-blocks = 2048 tf32 elements for tf32
// inputs (a multiple of every ring's k-blocks per stage); one chain per unit
// for the other kinds (fp32 accumulation of 16/8-bit inputs is far inside
// their 1e-2 bound; int8 accumulates exactly in s32).
template <int DT>
constexpr int chain_kb() {
    return DT == TRB_TFLOAT32 ? 64 : 0;
}

// cur += prev over COLS accumulator columns of this warp's 32 TMEM lanes
// (t_prev / t_cur: lane-quarter base addresses of the two accumulators), 64
// columns per TMEM round trip.  `release` runs as soon as the last columns of
// prev are in registers -- before the last sums are stored -- so the MMA
// thread, which waits for prev to start the chunk after next, restarts early.
template <int COLS, typename Release>
__device__ __forceinline__ void fold_chunk(uint32_t t_prev, uint32_t t_cur, Release release) {
    if constexpr (COLS == 16 || COLS == 32) {
        uint32_t p[COLS], r[COLS];
        if constexpr (COLS == 16) {
            tmem_ld_32x32b_x16(t_prev, p);
            tmem_ld_32x32b_x16(t_cur, r);
        } else {
            tmem_ld_32x32b_x32(t_prev, p);
            tmem_ld_32x32b_x32(t_cur, r);
        }
        tmem_wait_ld();
        release();
#pragma unroll
        for (int i = 0; i < COLS; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(p[i]));
        if constexpr (COLS == 16) tmem_st_32x32b_x16(t_cur, r);
        else tmem_st_32x32b_x32(t_cur, r);
    } else {
        static_assert(COLS % 64 == 0, "fold width");
#pragma unroll 1
        for (int c = 0; c < COLS / 64; ++c) {
            uint32_t p[64], r[64];
            tmem_ld_32x32b_x64(t_prev + (uint32_t)(c * 64), p);
            tmem_ld_32x32b_x64(t_cur + (uint32_t)(c * 64), r);
            tmem_wait_ld();
            if (c == COLS / 64 - 1) release();
#pragma unroll
            for (int i = 0; i < 64; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(p[i]));
            tmem_st_32x32b_x64(t_cur + (uint32_t)(c * 64), r);
        }
    }
    tmem_wait_st();
}

// One unit of a worker's schedule: a k-block range of a tile.  slot >= 0: the
// tile is split and this range's fp32 partial goes to workspace slot `slot`
// (x 2 CTAs of a pair); `contributors` ranges make up the tile.
struct WorkItem {
    int tile, kb0, kb1, slot, contributors;
};

// The idx-th (tile, split) unit of worker `w` out of `P`; false past the last.
__device__ __forceinline__ bool work_item(int idx, int w, int P, int num_tiles, int num_kb, const SplitK& sk,
                                          WorkItem& it) {
    const int unit = w + idx * P;
    if (unit >= num_tiles * sk.splits) return false;
    it.tile = unit / sk.splits;
    it.kb0 = (unit % sk.splits) * sk.kb_per_split;
    it.kb1 = min(it.kb0 + sk.kb_per_split, num_kb);
    it.slot = sk.splits > 1 ? unit : -1;
    it.contributors = sk.splits;
    return true;
}

// Workspace slot of the i-th contributor (in K order) of a split tile.
__device__ __forceinline__ int contributor_slot(int tile, int i, const SplitK& sk) { return tile * sk.splits + i; }

// K order of a unit: with rotate_k, tiles that run at the same time start at
// different k-blocks, so CTAs sharing one A panel (a single row of tiles,
// M <= 128) do not all request the same A tile from the same L2 slices at
// once.  Each tile always uses the same order, so results stay deterministic.
__device__ __forceinline__ int k_rotation(const SplitK& sk, int tile, int nk) {
    return sk.rotate_k && nk > 0 ? tile % nk : 0;
}


// KB: B is stored K-major (N x K row-major, "B transposed"); otherwise B is
// the row-major K x N matrix, an MN-major operand.
// CL > 1: cluster split-K for skinny problems.  The grid is tiles x CL, one
// unit per CTA, the CL CTAs of a cluster are the K splits of one tile (rank =
// split).  After every CTA's main loop has drained, the shared-memory rings
// are free: rank r owns columns [r * BN / CL, (r + 1) * BN / CL) of the tile,
// every CTA writes its fp32 partials of each column block into the owner's
// ring (distributed shared memory), and the owner sums the CL partials in
// split order -- the order, hence the bits, of the workspace fix-up -- and
// stores C.  No workspace and no L2 round trips after the main loop.
template <int DT, bool KB, int BN, int CL = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, void* __restrict__ C, int M, int N, int K,
                        float out_scale, SplitK sk) {
    using Tr = Traits<DT>;
    constexpr int kBKElems = kBKBytes / Tr::kEsize;         // K elements per stage
    constexpr int kBoxN = 128 / Tr::kEsize;                 // N elements per B box (one swizzle row)
    constexpr int kBBoxes = BN / kBoxN;                    // B boxes per stage
    constexpr int kBBoxBytes = kBKElems * 128;              // bytes of one B box == MN-atom stride (LBO)
    constexpr int kInstrKRows = kInstrKBytes / Tr::kEsize;  // K rows of B per instruction
    using Cfg = TileCfgFor<DT, BN, CL>;
    constexpr int kStagesT = Cfg::kStages;
    constexpr int kKD = Cfg::kKD;                   // k-blocks per stage
    constexpr int kBStageT = Cfg::kBStage;          // B bytes of one k-block
    constexpr int kAStageKD = kKD * kAStage;        // A bytes of one stage
    constexpr int kBStageKD = kKD * kBStageT;       // B bytes of one stage
    constexpr uint32_t kIdesc1 = idesc_with_n(KB ? idesc_b_kmajor(Tr::kIdesc) : Tr::kIdesc, BN);
    static_assert(KB || BN >= kBoxN, "MN-major B needs at least one 128-byte swizzle row per tile");
    static_assert(CL == 1 || ((CL == 2 || CL == 4 || CL == 8) && (BN / CL) % 32 == 0), "cluster split");
    static_assert(CL == 1 || (size_t)kBM * BN * 4 <= (size_t)kStagesT * (kAStageKD + kBStageKD), "receive buffer");
    static_assert((size_t)kStagesT * (kAStageKD + kBStageKD) + 1024 + Cfg::kEpiBytes == Cfg::kSmem, "footprint");

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kStagesT];
    __shared__ __align__(8) uint64_t empty_bar[kStagesT];
    __shared__ __align__(8) uint64_t accf_bar[kNumAcc];
    __shared__ __align__(8) uint64_t acce_bar[kNumAcc];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ int last_split_flag;
    __shared__ __align__(8) uint64_t recv_bar;  // cluster split-K: the peers' partials have landed

    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t sA = smem_base;
    const uint32_t sB = smem_base + kStagesT * kAStageKD;
    const uint32_t sEpi = sB + kStagesT * kBStageKD;  // TMA-store staging (CL == 1), 1 KiB aligned

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + kBM - 1) / kBM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + kBKElems - 1) / kBKElems;
    const int num_units = num_tiles * sk.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesT; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int a = 0; a < kNumAcc; ++a) {
            mbar_init(smem_u32(&accf_bar[a]), 1);
            mbar_init(smem_u32(&acce_bar[a]), 4);  // one arrival per epilogue warp
        }
        mbar_init(smem_u32(&drain_bar), 1);
        if constexpr (CL > 1) mbar_init(smem_u32(&recv_bar), 1);
        abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if constexpr (CL == 1) tma_prefetch_desc(&tmC);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    // The next grid may set up (barriers, TMEM, descriptors) while this one
    // runs; it reads and writes global memory only after its own wait.
    grid_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            grid_dependency_wait();  // A and B may be outputs of the previous grid
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;  // per stage: a load is outstanding / its parity
            bool ok = true;
            for (int unit = blockIdx.x; ok && unit < num_units; unit += gridDim.x) {
                int mb, nb;
                tile_coords(unit / sk.splits, num_m, num_n, sk.group_m, mb, nb);
                const int kb0 = (unit % sk.splits) * sk.kb_per_split;
                const int nk = min(kb0 + sk.kb_per_split, num_kb) - kb0;
                const int rot = k_rotation(sk, unit / sk.splits, nk);
                for (int i0 = 0; i0 < nk; i0 += kKD) {  // one stage: k-blocks i0 .. i0 + cnt - 1
                    const int cnt = min(kKD, nk - i0);
                    if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrProducerWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(&full_bar[stage]);
                    mbar_arrive_expect_tx(fb, (uint32_t)cnt * (kAStage + kBStageT));
#pragma unroll
                    for (int d = 0; d < kKD; ++d) {
                        if (d >= cnt) break;
                        const int i = i0 + d;
                        const int kb = kb0 + (i + rot < nk ? i + rot : i + rot - nk);
                        const uint32_t a_dst = sA + stage * kAStageKD + d * kAStage;
                        const uint32_t b_dst = sB + stage * kBStageKD + d * kBStageT;
                        tma_load_2d(a_dst, &tmA, fb, kb * kBKElems, mb * kBM);
                        if constexpr (KB) {
                            tma_load_2d(b_dst, &tmB, fb, kb * kBKElems, nb * BN);
                        } else {
#pragma unroll
                            for (int j = 0; j < kBBoxes; ++j)
                                tma_load_2d(b_dst + j * kBBoxBytes, &tmB, fb, nb * BN + j * kBoxN, kb * kBKElems);
                        }
                    }
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStagesT) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: the CTA must not exit while a TMA write into its smem is pending.
            for (int s = 0; s < kStagesT; ++s)
                if (issued_mask & (1u << s))
                    if (!mbar_wait(smem_u32(&full_bar[s]), (issued_phase >> s) & 1u, nullptr))
                        atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer (single thread)
            // Stage-0 descriptors; a stage / K-step moves only the start address.
            const uint64_t a_desc0 = make_sdesc(sA, 16, 1024);
            const uint64_t b_desc0 = KB ? make_sdesc(sB, 16, 1024)
                                        : make_sdesc(sB, kBBoxBytes, Tr::BLayout::kSbo, Tr::BLayout::kLayoutType);
            constexpr int kBKStep = KB ? kInstrKBytes : kInstrKRows * 128;  // B bytes per instruction K step
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            int t_local = 0;
            for (int unit = blockIdx.x; ok && unit < num_units; unit += gridDim.x, ++t_local) {
                const int kb0 = (unit % sk.splits) * sk.kb_per_split;
                const int nk = min(kb0 + sk.kb_per_split, num_kb) - kb0;
                const int chunk = unit_chunks(nk, sk.chunk_kb) > 1 ? sk.chunk_kb : nk;  // a multiple of kKD
                int acc = 0, chunk_left = 0;
                uint32_t d_tmem = tmem_base;
                for (int i0 = 0; i0 < nk; i0 += kKD) {  // same stages as the producer; only the counts matter here
                    const int cnt = min(kKD, nk - i0);
                    if (chunk_left == 0) {  // a chunk starts: take the next accumulator, zero it by its first MMA
                        if (i0 != 0) {
                            tc_commit(smem_u32(&accf_bar[acc]));  // chunk complete -> epilogue folds it
                            ++t_local;
                        }
                        acc = t_local & 1;
                        if (!mbar_wait(smem_u32(&acce_bar[acc]), ((uint32_t)(t_local >> 1) & 1u) ^ 1u, &abort_flag)) {
                            atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                            abort_flag = 1;
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        d_tmem = tmem_base + (uint32_t)(acc * BN);
                        chunk_left = chunk;
                    }
                    const bool fresh = chunk_left == chunk;
                    chunk_left -= cnt;
                    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    // TMA completion is ordered before the MMA by the barrier's
                    // transaction count: no tcgen05 fence is needed per stage.
                    const uint64_t a_stage = a_desc0 + (uint64_t)((stage * kAStageKD) >> 4);
                    const uint64_t b_stage = b_desc0 + (uint64_t)((stage * kBStageKD) >> 4);
#pragma unroll
                    for (int d = 0; d < kKD; ++d) {
                        if (d >= cnt) break;
#pragma unroll
                        for (int ks = 0; ks < kKSteps; ++ks)
                            mma<Tr::kKind>(d_tmem, a_stage + (uint64_t)((d * kAStage + ks * kInstrKBytes) >> 4),
                                           b_stage + (uint64_t)((d * kBStageT + ks * kBKStep) >> 4), kIdesc1,
                                           (!fresh || d != 0 || ks != 0) ? 1u : 0u);
                    }
                    tc_commit(smem_u32(&empty_bar[stage]));  // frees the smem stage when these MMAs finish
                    if (++stage == kStagesT) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) tc_commit(smem_u32(&accf_bar[acc]));  // accumulator complete -> epilogue
            }
            // Drain: all MMAs of this thread complete before TMEM is released.
            tc_commit(smem_u32(&drain_bar));
            if (!mbar_wait(smem_u32(&drain_bar), 0, nullptr)) atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else if constexpr (CL == 1) {
        // ---------------- epilogue: warps 2..5 own TMEM lane quarters (warp % 4)
        grid_dependency_wait();  // C and the split-K workspace may be in use by the previous grid
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        const bool first_epi_thread = threadIdx.x == 64;
        int t_local = 0;
        uint32_t boxes = 0;  // TMA-store boxes this warp has issued (selects its staging buffer)
        const uint32_t t_quarter = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++t_local) {
            const int tile = unit / sk.splits;
            int mb, nb;
            tile_coords(tile, num_m, num_n, sk.group_m, mb, nb);
            const int kb0 = (unit % sk.splits) * sk.kb_per_split;
            const int nch = unit_chunks(min(kb0 + sk.kb_per_split, num_kb) - kb0, sk.chunk_kb);
            bool ok = true;
            for (int ch = 0; ch < nch; ++ch) {  // K chunks: fold each into the running sum
                if (ch > 0) ++t_local;
                const int a = t_local & 1;
                ok = mbar_wait(smem_u32(&accf_bar[a]), (uint32_t)(t_local >> 1) & 1u, &abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (sk.splits > 1) ok = named_barrier_and(1, 128, ok);  // the fix-up below is CTA-wide
                if (!ok) break;
                tc_fence_after();
                if (ch > 0) {
                    fold_chunk<BN>(t_quarter + (uint32_t)((a ^ 1) * BN), t_quarter + (uint32_t)(a * BN), [&] {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&acce_bar[a ^ 1]));  // running sum read: free it
                    });
                }
            }
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                    abort_flag = 1;
                }
                break;
            }
            const int acc = t_local & 1;
            const int grow = mb * kBM + row_in_tile;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            if (sk.splits == 1 && Cfg::kEpiBytes == 0) {
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                    tmem_wait_ld();
                    const int gcol = nb * BN + c * 32;
                    if (grow < M && gcol < N) store_chunk<DT>(C, grow, gcol, N, r, out_scale);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&acce_bar[acc]));
                continue;
            }
            if (sk.splits == 1) {
                const int row0 = mb * kBM + q * 32;  // first row of this warp's boxes
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                    tmem_wait_ld();
                    const int gcol = nb * BN + c * 32;
                    if (row0 >= M || gcol >= N) continue;  // warp-uniform: the box lies outside C
                    const uint32_t buf = sEpi + (uint32_t)((q * 2 + (int)(boxes & 1u)) * epi_box_bytes<DT>());
                    if (lane == 0) bulk_wait_read<1>();  // the store issued two boxes ago has read `buf`
                    __syncwarp();
                    stage_row<DT>(buf, lane, r, out_scale);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, buf, gcol, row0);
                        bulk_commit();
                    }
                    ++boxes;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&acce_bar[acc]));
                continue;
            }
            // ---- split-K: publish this unit's fp32 partial.  Workspace blocks are
            // [16-byte column group][row], row-minor, so a warp's 16-byte stores
            // (and the fix-up's loads) cover 512 contiguous bytes.
            uint4* wblk = reinterpret_cast<uint4*>(sk.ws) + (size_t)unit * (BN / 4) * kBM + row_in_tile;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                tmem_wait_ld();
                if (grow < M && nb * BN + c * 32 < N) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        wblk[(size_t)(c * 8 + i) * kBM] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acce_bar[acc]));  // TMEM free for the next unit
            __threadfence();
            named_barrier(1, 128);
            if (first_epi_thread)
                last_split_flag = atomicAdd(&sk.counters[tile], 1u) == (unsigned)(sk.splits - 1);
            named_barrier(1, 128);
            if (!last_split_flag) continue;
            // ---- last arrival: deterministic sum over splits 0..S-1, convert, store C
            __threadfence();
            if (grow < M) {
                const float4* base =
                    reinterpret_cast<const float4*>(sk.ws) + (size_t)tile * sk.splits * (BN / 4) * kBM + row_in_tile;
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    const int gcol = nb * BN + c * 32;
                    if (gcol >= N) break;
                    float acc_f[32];
                    const float4* p0 = base + (size_t)c * 8 * kBM;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 v = __ldcg(p0 + (size_t)i * kBM);
                        acc_f[4 * i] = v.x; acc_f[4 * i + 1] = v.y; acc_f[4 * i + 2] = v.z; acc_f[4 * i + 3] = v.w;
                    }
                    for (int sp = 1; sp < sk.splits; ++sp) {
                        const float4* ps = base + ((size_t)sp * (BN / 4) + c * 8) * kBM;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 v = __ldcg(ps + (size_t)i * kBM);
                            if constexpr (DT == TRB_INT8) {  // exact integer partial sums
                                acc_f[4 * i] = __int_as_float(__float_as_int(acc_f[4 * i]) + __float_as_int(v.x));
                                acc_f[4 * i + 1] = __int_as_float(__float_as_int(acc_f[4 * i + 1]) + __float_as_int(v.y));
                                acc_f[4 * i + 2] = __int_as_float(__float_as_int(acc_f[4 * i + 2]) + __float_as_int(v.z));
                                acc_f[4 * i + 3] = __int_as_float(__float_as_int(acc_f[4 * i + 3]) + __float_as_int(v.w));
                            } else {
                                acc_f[4 * i] += v.x; acc_f[4 * i + 1] += v.y; acc_f[4 * i + 2] += v.z; acc_f[4 * i + 3] += v.w;
                            }
                        }
                    }
                    uint32_t r[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(acc_f[i]);
                    store_chunk<DT>(C, grow, gcol, N, r, out_scale);
                }
            }
            if (first_epi_thread) sk.counters[tile] = 0u;  // ready for the next launch
        }
        if (lane == 0) bulk_wait_all();  // this warp's TMA stores are complete before the CTA exits
        __syncwarp();
    }

    if constexpr (CL > 1) {
        // ---------------- cluster split-K epilogue (one unit per CTA)
        const bool epi = warp >= 2;
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        bool ok = true;
        int acc = 0;  // accumulator holding this CTA's partial after the chunk folds
        if (epi) {
            grid_dependency_wait();
            const int kb0 = (int)(blockIdx.x % CL) * sk.kb_per_split;
            const int nch = unit_chunks(min(kb0 + sk.kb_per_split, num_kb) - kb0, sk.chunk_kb);
            const uint32_t t_quarter = tmem_base + ((uint32_t)(q * 32) << 16);
            for (int ch = 0; ch < nch; ++ch) {  // one unit per CTA: chunk ch uses accumulator ch & 1
                acc = ch & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&accf_bar[acc]), (uint32_t)(ch >> 1) & 1u, &abort_flag));
                if (!ok) break;
                tc_fence_after();
                if (ch > 0) {
                    fold_chunk<BN>(t_quarter + (uint32_t)((acc ^ 1) * BN), t_quarter + (uint32_t)(acc * BN), [&] {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&acce_bar[acc ^ 1]));
                    });
                }
            }
            if (!ok && lane == 0) {
                atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                abort_flag = 1;
            }
        }
        __syncwarp();
        cluster_sync_all();  // every CTA's MMAs and TMA writes are done: the rings can receive
        constexpr int kOwnCols = BN / CL;
        constexpr int kOwnChunks = kOwnCols / 32;
        const int rank = (int)cluster_ctarank();
        // Receive buffer in the ring: 16-byte slots [src rank][owned 32-column
        // chunk][float4 i][row], row-minor, so the 32 lanes of one store (or
        // load) cover 512 contiguous bytes.  Peers' slots arrive by st.async,
        // completing on recv_bar; this CTA's own slots are written and read
        // back by the same thread.
        const uint32_t sRecv = smem_base;
        const uint32_t recv_bar_addr = smem_u32(&recv_bar);
        if (epi && ok) {
            if (threadIdx.x == 64) mbar_arrive_expect_tx(recv_bar_addr, (uint32_t)((CL - 1) * kOwnCols * kBM * 4));
            uint4* recv4 = reinterpret_cast<uint4*>(smem_raw + (sRecv - smem_u32(smem_raw)));
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                tmem_wait_ld();
                const int owner = c / kOwnChunks;
                const int slot0 = ((rank * kOwnChunks + c % kOwnChunks) * 8) * kBM + row_in_tile;
                if (owner == rank) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        recv4[slot0 + i * kBM] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
                } else {
                    const uint32_t dst = mapa_shared(sRecv + (uint32_t)(slot0 * 16), (uint32_t)owner);
                    const uint32_t bar = mapa_shared(recv_bar_addr, (uint32_t)owner);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        st_async_v4(dst + (uint32_t)(i * kBM * 16),
                                    make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]), bar);
                }
            }
            if (!mbar_wait_cluster(recv_bar_addr, 0, &abort_flag)) {
                atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                abort_flag = 1;
                ok = false;
            }
        }
        // Every partial sent to this CTA has landed (recv_bar) and its own sends
        // are issued.  The exit barrier that keeps peers' shared memory alive
        // while sends may still target it is split around the sum and stores,
        // which hide its latency.
        __syncwarp();
        cluster_arrive();
        if (epi && ok) {
            int mb, nb;
            tile_coords((int)blockIdx.x / CL, num_m, num_n, sk.group_m, mb, nb);
            const int grow = mb * kBM + row_in_tile;
            const float4* recv = reinterpret_cast<const float4*>(smem_raw + (sRecv - smem_u32(smem_raw)));
            if (grow < M) {
#pragma unroll 1
                for (int cc = 0; cc < kOwnChunks; ++cc) {
                    const int gcol = nb * BN + rank * kOwnCols + cc * 32;
                    if (gcol >= N) break;
                    float acc_f[32];
#pragma unroll
                    for (int src = 0; src < CL; ++src) {  // split order
                        const float4* p4 = recv + (size_t)(src * kOwnChunks + cc) * 8 * kBM + row_in_tile;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 v = p4[i * kBM];
                            if (src == 0) {
                                acc_f[4 * i] = v.x; acc_f[4 * i + 1] = v.y; acc_f[4 * i + 2] = v.z; acc_f[4 * i + 3] = v.w;
                            } else if constexpr (DT == TRB_INT8) {
                                acc_f[4 * i] = __int_as_float(__float_as_int(acc_f[4 * i]) + __float_as_int(v.x));
                                acc_f[4 * i + 1] = __int_as_float(__float_as_int(acc_f[4 * i + 1]) + __float_as_int(v.y));
                                acc_f[4 * i + 2] = __int_as_float(__float_as_int(acc_f[4 * i + 2]) + __float_as_int(v.z));
                                acc_f[4 * i + 3] = __int_as_float(__float_as_int(acc_f[4 * i + 3]) + __float_as_int(v.w));
                            } else {
                                acc_f[4 * i] += v.x; acc_f[4 * i + 1] += v.y; acc_f[4 * i + 2] += v.z; acc_f[4 * i + 3] += v.w;
                            }
                        }
                    }
                    uint32_t r[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(acc_f[i]);
                    store_chunk<DT>(C, grow, gcol, N, r, out_scale);
                }
            }
        }
        __syncwarp();
        cluster_wait();  // no CTA leaves while a peer's stores may still target it
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ------------------------------------------------------------------ swapped-operand skinny kernel
// For M <= 64 a 128-row MMA tile is mostly padding, and its A boxes (128 rows
// x 128 bytes per stage) crowd B out of shared memory.  This kernel computes
// C^T = B^T * A^T instead: the MMA's M side (128 TMEM lanes) runs along N and
// its N side (BS = 16, 32 or 64 columns) along the few rows of A.
//  * wide operand W = B^T, 128 rows of N x one 128-byte K slice per stage:
//    K-major when B is stored N x K, otherwise row-major B read in place
//    through the MN-major swizzle (instruction-descriptor bit 15);
//  * small operand S = A, BS rows x one 128-byte K slice, K-major (rows past
//    M are zero-filled by TMA);
//  * the ring is as deep as shared memory allows (11 stages at BS = 16), so
//    each SM keeps ~176 KiB of B requests in flight, what streaming B at HBM
//    rate needs;
//  * work units are 128-column panels of C times K splits (the split count
//    balances units over the SMs), with the main kernel's deterministic
//    last-arrival split-K fix-up;
//  * the epilogue thread of TMEM lane l owns column n = panel * 128 + l and
//    writes its BS values down that column; for each row m the 32 lanes of a
//    warp store 32 consecutive elements.
template <int BS, int KD, int CL>
struct SwapCfg {
    static_assert(BS == 16 || BS == 32 || BS == 64, "swap tile width");
    static_assert(KD == 1 || KD == 2 || KD == 4, "k-blocks per stage");
    static_assert(CL == 1 || CL == 2 || CL == 4 || CL == 8, "cluster split count");
    static constexpr int kSBlock = BS * kBKBytes;          // one k-block of S
    static constexpr int kWStage = KD * kAStage;            // KD k-blocks of W (128 rows each)
    static constexpr int kSStage = KD * kSBlock;
    static constexpr int kStageBytes = kWStage + kSStage;
    // Cluster split-K: fp32 partials of the lanes this CTA owns, one slot per peer.
    static constexpr int kRecvBytes = CL > 1 ? kBM * BS * 4 : 0;
    static constexpr int kRingBudget = 210 * 1024 - kRecvBytes;
    static constexpr int kStages = kRingBudget / kStageBytes > 12 ? 12 : kRingBudget / kStageBytes;
    static_assert(kStages >= 2, "ring too shallow");
    static constexpr int kTmemCols = kNumAcc * BS < 32 ? 32 : kNumAcc * BS;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + kRecvBytes + 1024;
};

// One output element from a 32-bit accumulator word (same conversions as store_chunk).
template <int DT>
__device__ __forceinline__ void store_elem(void* C, size_t idx, uint32_t v, float out_scale) {
    if constexpr (DT == TRB_BFLOAT16 || DT == TRB_FLOAT8_E4M3FN) {
        float f = __uint_as_float(v);
        if constexpr (DT == TRB_FLOAT8_E4M3FN) f *= out_scale;
        static_cast<__nv_bfloat16*>(C)[idx] = __float2bfloat16_rn(f);
    } else if constexpr (DT == TRB_FLOAT16) {
        static_cast<__half*>(C)[idx] = __float2half_rn(__uint_as_float(v));
    } else {
        static_cast<uint32_t*>(C)[idx] = v;
    }
}

template <int BS>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, uint32_t (&r)[BS]) {
    if constexpr (BS == 16) {
        tmem_ld_32x32b_x16(taddr, r);
    } else {
#pragma unroll
        for (int c = 0; c < BS / 32; ++c)
            tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
    }
    tmem_wait_ld();
}

// CL > 1: cluster split-K.  The grid is tiles x CL, one unit per CTA, and the
// CL CTAs of a cluster are the K splits of one tile (cluster rank = split).
// Rank r owns TMEM lanes [r * 128 / CL, (r + 1) * 128 / CL): every CTA writes
// the partials of lanes it does not own into the owner's receive buffer
// (distributed shared memory), then arrives on the owner's receive barrier;
// the owner sums the CL partials in split order -- the same order, hence the
// same bits, as the global-workspace fix-up -- and stores C.  No workspace,
// no counters, and no round trips through L2 after the main loop.
template <int DT, bool KB, int BS, int KD, int CL>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_swap_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                     void* __restrict__ C, int M, int N, int K, float out_scale, SplitK sk) {
    using Tr = Traits<DT>;
    using Cfg = SwapCfg<BS, KD, CL>;
    constexpr int kBKElems = kBKBytes / Tr::kEsize;
    constexpr int kBoxN = 128 / Tr::kEsize;   // N elements per MN-major W box (one swizzle row)
    constexpr int kWBoxes = kBM / kBoxN;      // MN-major W boxes per stage
    constexpr int kWBoxBytes = KD * kBKElems * 128;  // one MN-major W box: KD k-blocks tall
    constexpr int kWKBlockBytes = kBKElems * 128;    // one k-block inside such a box
    constexpr int kInstrKRows = kInstrKBytes / Tr::kEsize;
    constexpr int kStagesT = Cfg::kStages;
    constexpr int kWStage = Cfg::kWStage;
    constexpr int kSStage = Cfg::kSStage;
    constexpr int kSBlock = Cfg::kSBlock;
    // A operand = W (MN-major unless B is stored K-major), B operand = S (K-major), N = BS.
    constexpr uint32_t kIdescS = idesc_with_n(idesc_b_kmajor(Tr::kIdesc) | (KB ? 0u : (1u << 15)), BS);
    static_assert(KB || KD * kBKElems <= 256, "TMA box height");

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kStagesT];
    __shared__ __align__(8) uint64_t empty_bar[kStagesT];
    __shared__ __align__(8) uint64_t accf_bar[kNumAcc];
    __shared__ __align__(8) uint64_t acce_bar[kNumAcc];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ int last_split_flag;
    __shared__ __align__(8) uint64_t recv_bar;  // cluster split-K: the peers' partials have landed

    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t sW = smem_base;
    const uint32_t sS = smem_base + kStagesT * kWStage;
    const uint32_t sRecv = sS + kStagesT * kSStage;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = (N + kBM - 1) / kBM;
    const int num_kb = (K + kBKElems - 1) / kBKElems;
    const int num_units = num_tiles * sk.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesT; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int a = 0; a < kNumAcc; ++a) {
            mbar_init(smem_u32(&accf_bar[a]), 1);
            mbar_init(smem_u32(&acce_bar[a]), 4);
        }
        mbar_init(smem_u32(&drain_bar), 1);
        if constexpr (CL > 1) mbar_init(smem_u32(&recv_bar), 1);
        abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmS);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    if constexpr (CL > 1) cluster_sync_all();  // peers' receive barriers initialised before any arrival
    // The next grid may set up (barriers, TMEM, descriptors) while this one
    // streams; it reads and writes global memory only after its own wait.
    grid_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            grid_dependency_wait();  // A and B may be outputs of the previous grid
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for (int unit = blockIdx.x; ok && unit < num_units; unit += gridDim.x) {
                const int tile = unit / sk.splits;
                const int kb0 = (unit % sk.splits) * sk.kb_per_split;
                const int nk = min(kb0 + sk.kb_per_split, num_kb) - kb0;
                for (int g = 0; g * KD < nk; ++g) {  // one stage = KD consecutive k-blocks
                    const int kbg = kb0 + g * KD;
                    const int valid = min(KD, nk - g * KD);
                    if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrProducerWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(&full_bar[stage]);
                    // MN-major W boxes always span KD k-blocks (rows past K are
                    // zero-filled, rows of the next split are loaded but unused).
                    mbar_arrive_expect_tx(fb, (uint32_t)((KB ? valid * kAStage : kWStage) + valid * kSBlock));
                    if constexpr (KB) {
                        for (int i = 0; i < valid; ++i)
                            tma_load_2d(sW + stage * kWStage + i * kAStage, &tmW, fb, (kbg + i) * kBKElems, tile * kBM);
                    } else {
#pragma unroll
                        for (int j = 0; j < kWBoxes; ++j)
                            tma_load_2d(sW + stage * kWStage + j * kWBoxBytes, &tmW, fb, tile * kBM + j * kBoxN,
                                        kbg * kBKElems);
                    }
                    for (int i = 0; i < valid; ++i)
                        tma_load_2d(sS + stage * kSStage + i * kSBlock, &tmS, fb, (kbg + i) * kBKElems, 0);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStagesT) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int s = 0; s < kStagesT; ++s)
                if (issued_mask & (1u << s))
                    if (!mbar_wait(smem_u32(&full_bar[s]), (issued_phase >> s) & 1u, nullptr))
                        atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            const uint64_t a_desc0 = KB ? make_sdesc(sW, 16, 1024)
                                        : make_sdesc(sW, kWBoxBytes, Tr::BLayout::kSbo, Tr::BLayout::kLayoutType);
            const uint64_t b_desc0 = make_sdesc(sS, 16, 1024);
            constexpr int kWStep = KB ? kInstrKBytes : kInstrKRows * 128;  // W bytes per instruction K step
            constexpr int kWBlock = KB ? kAStage : kWKBlockBytes;          // W bytes per k-block in a stage
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            int t_local = 0;
            for (int unit = blockIdx.x; ok && unit < num_units; unit += gridDim.x, ++t_local) {
                const int kb0 = (unit % sk.splits) * sk.kb_per_split;
                const int nk = min(kb0 + sk.kb_per_split, num_kb) - kb0;
                const int chunk = unit_chunks(nk, sk.chunk_kb) > 1 ? sk.chunk_kb : nk;  // a multiple of KD
                int acc = 0, chunk_left = 0;
                uint32_t d_tmem = tmem_base;
                for (int g = 0; g * KD < nk; ++g) {
                    const int valid = min(KD, nk - g * KD);
                    if (chunk_left == 0) {  // a chunk starts: take the next accumulator, zero it by its first MMA
                        if (g != 0) {
                            tc_commit(smem_u32(&accf_bar[acc]));
                            ++t_local;
                        }
                        acc = t_local & 1;
                        if (!mbar_wait(smem_u32(&acce_bar[acc]), ((uint32_t)(t_local >> 1) & 1u) ^ 1u, &abort_flag)) {
                            atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                            abort_flag = 1;
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        d_tmem = tmem_base + (uint32_t)(acc * BS);
                        chunk_left = chunk;
                    }
                    const bool fresh = chunk_left == chunk;
                    chunk_left -= valid;
                    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint64_t a_stage = a_desc0 + (uint64_t)((stage * kWStage) >> 4);
                    const uint64_t b_stage = b_desc0 + (uint64_t)((stage * kSStage) >> 4);
                    for (int i = 0; i < valid; ++i) {
#pragma unroll
                        for (int ks = 0; ks < kKSteps; ++ks)
                            mma<Tr::kKind>(d_tmem, a_stage + (uint64_t)((i * kWBlock + ks * kWStep) >> 4),
                                           b_stage + (uint64_t)((i * kSBlock + ks * kInstrKBytes) >> 4), kIdescS,
                                           (!fresh || i != 0 || ks != 0) ? 1u : 0u);
                    }
                    tc_commit(smem_u32(&empty_bar[stage]));
                    if (++stage == kStagesT) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) tc_commit(smem_u32(&accf_bar[acc]));
            }
            tc_commit(smem_u32(&drain_bar));
            if (!mbar_wait(smem_u32(&drain_bar), 0, nullptr)) atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else {
        // ---------------- epilogue: warps 2..5 own TMEM lane quarters (warp % 4)
        grid_dependency_wait();  // C and the split-K workspace may be in use by the previous grid
        const int q = warp & 3;
        const int n_in_tile = q * 32 + lane;
        const bool first_epi_thread = threadIdx.x == 64;
        const int rows = M < BS ? M : BS;
        int t_local = 0;
        const uint32_t t_quarter = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++t_local) {
            const int tile = unit / sk.splits;
            const int kb0 = (unit % sk.splits) * sk.kb_per_split;
            const int nch = unit_chunks(min(kb0 + sk.kb_per_split, num_kb) - kb0, sk.chunk_kb);
            bool ok = true;
            for (int ch = 0; ch < nch; ++ch) {  // K chunks: fold each into the running sum
                if (ch > 0) ++t_local;
                const int a = t_local & 1;
                ok = mbar_wait(smem_u32(&accf_bar[a]), (uint32_t)(t_local >> 1) & 1u, &abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (sk.splits > 1) ok = named_barrier_and(1, 128, ok);
                if (!ok) break;
                tc_fence_after();
                if (ch > 0) {
                    fold_chunk<BS>(t_quarter + (uint32_t)((a ^ 1) * BS), t_quarter + (uint32_t)(a * BS), [&] {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&acce_bar[a ^ 1]));  // running sum read: free it
                    });
                }
            }
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                    abort_flag = 1;
                }
                break;
            }
            const int acc = t_local & 1;
            const int gn = tile * kBM + n_in_tile;
            uint32_t r[BS];
            tmem_ld_row<BS>(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BS), r);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acce_bar[acc]));  // TMEM free for the next unit
            if (sk.splits == 1) {
                if (gn < N) {
#pragma unroll
                    for (int m = 0; m < BS; ++m)
                        if (m < rows) store_elem<DT>(C, (size_t)m * N + gn, r[m], out_scale);
                }
                continue;
            }
            if constexpr (CL > 1) {
                // ---- cluster split-K through distributed shared memory
                constexpr int kOwn = kBM / CL;
                const int rank = (int)cluster_ctarank();
                const int owner = n_in_tile / kOwn;
                const int slot = n_in_tile % kOwn;
                // Receive buffer: 16-byte slots [src rank][float4 i][owned lane], lane-minor
                // so one store (or load) of a warp covers 512 contiguous bytes.  Peers'
                // partials arrive by st.async and complete on the owner's recv_bar.
                if (owner != rank) {
                    const uint32_t dst =
                        mapa_shared(sRecv + (uint32_t)((rank * (BS / 4) * kOwn + slot) * 16), (uint32_t)owner);
                    const uint32_t bar = mapa_shared(smem_u32(&recv_bar), (uint32_t)owner);
#pragma unroll
                    for (int i = 0; i < BS / 4; ++i)
                        st_async_v4(dst + (uint32_t)(i * kOwn * 16),
                                    make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]), bar);
                }
                if (first_epi_thread) mbar_arrive_expect_tx(smem_u32(&recv_bar), (uint32_t)((CL - 1) * kOwn * BS * 4));
                if (owner == rank) {
                    if (!mbar_wait_cluster(smem_u32(&recv_bar), 0, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                        abort_flag = 1;
                    } else if (gn < N) {
                        const float* recv = reinterpret_cast<const float*>(smem_raw + (sRecv - smem_u32(smem_raw)));
                        float acc_f[BS];
#pragma unroll
                        for (int src = 0; src < CL; ++src) {  // split order: src 0 first, as in the workspace fix-up
#pragma unroll
                            for (int i = 0; i < BS / 4; ++i) {
                                float4 v;
                                if (src == rank) {
                                    v = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                    __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                                } else {
                                    v = reinterpret_cast<const float4*>(recv)[(size_t)(src * (BS / 4) + i) * kOwn + slot];
                                }
                                if (src == 0) {
                                    acc_f[4 * i] = v.x; acc_f[4 * i + 1] = v.y; acc_f[4 * i + 2] = v.z; acc_f[4 * i + 3] = v.w;
                                } else if constexpr (DT == TRB_INT8) {
                                    acc_f[4 * i] = __int_as_float(__float_as_int(acc_f[4 * i]) + __float_as_int(v.x));
                                    acc_f[4 * i + 1] = __int_as_float(__float_as_int(acc_f[4 * i + 1]) + __float_as_int(v.y));
                                    acc_f[4 * i + 2] = __int_as_float(__float_as_int(acc_f[4 * i + 2]) + __float_as_int(v.z));
                                    acc_f[4 * i + 3] = __int_as_float(__float_as_int(acc_f[4 * i + 3]) + __float_as_int(v.w));
                                } else {
                                    acc_f[4 * i] += v.x; acc_f[4 * i + 1] += v.y; acc_f[4 * i + 2] += v.z; acc_f[4 * i + 3] += v.w;
                                }
                            }
                        }
#pragma unroll
                        for (int m = 0; m < BS; ++m)
                            if (m < rows) store_elem<DT>(C, (size_t)m * N + gn, __float_as_uint(acc_f[m]), out_scale);
                    }
                }
                continue;
            }
            // ---- split-K: publish this unit's fp32 partial (one TMEM lane = BS words),
            // lane-minor [16-byte group][lane] so a warp's stores are contiguous
            {
                uint4* w4 = reinterpret_cast<uint4*>(sk.ws) + (size_t)unit * (BS / 4) * kBM + n_in_tile;
#pragma unroll
                for (int i = 0; i < BS / 4; ++i)
                    w4[(size_t)i * kBM] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
            }
            __threadfence();
            named_barrier(1, 128);
            if (first_epi_thread)
                last_split_flag = atomicAdd(&sk.counters[tile], 1u) == (unsigned)(sk.splits - 1);
            named_barrier(1, 128);
            if (!last_split_flag) continue;
            __threadfence();
            if (gn < N) {
                const float4* base =
                    reinterpret_cast<const float4*>(sk.ws) + (size_t)tile * sk.splits * (BS / 4) * kBM + n_in_tile;
                float acc_f[BS];
#pragma unroll
                for (int i = 0; i < BS / 4; ++i) {
                    const float4 v = __ldcg(base + (size_t)i * kBM);
                    acc_f[4 * i] = v.x; acc_f[4 * i + 1] = v.y; acc_f[4 * i + 2] = v.z; acc_f[4 * i + 3] = v.w;
                }
                for (int sp = 1; sp < sk.splits; ++sp) {
                    const float4* ps = base + (size_t)sp * (BS / 4) * kBM;
#pragma unroll
                    for (int i = 0; i < BS / 4; ++i) {
                        const float4 v = __ldcg(ps + (size_t)i * kBM);
                        if constexpr (DT == TRB_INT8) {
                            acc_f[4 * i] = __int_as_float(__float_as_int(acc_f[4 * i]) + __float_as_int(v.x));
                            acc_f[4 * i + 1] = __int_as_float(__float_as_int(acc_f[4 * i + 1]) + __float_as_int(v.y));
                            acc_f[4 * i + 2] = __int_as_float(__float_as_int(acc_f[4 * i + 2]) + __float_as_int(v.z));
                            acc_f[4 * i + 3] = __int_as_float(__float_as_int(acc_f[4 * i + 3]) + __float_as_int(v.w));
                        } else {
                            acc_f[4 * i] += v.x; acc_f[4 * i + 1] += v.y; acc_f[4 * i + 2] += v.z; acc_f[4 * i + 3] += v.w;
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < BS; ++m)
                    if (m < rows) store_elem<DT>(C, (size_t)m * N + gn, __float_as_uint(acc_f[m]), out_scale);
            }
            if (first_epi_thread) sk.counters[tile] = 0u;
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (CL > 1) cluster_sync_all();  // no CTA leaves while a peer may still write into it
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ------------------------------------------------------------------ CTA-pair kernel
// A cluster of 2 CTAs (one TPC) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256): CTA r loads rows
// [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128) of the B
// tile into its own shared memory (32 KiB per stage, 6 stages), the pair's
// even CTA (the leader) issues the MMAs, which read both CTAs' operands and
// write each CTA's 128 x 256 fp32 (s32) accumulator into that CTA's TMEM.
// Against the single-CTA 128 x 256 tile this halves the B bytes each SM pulls
// from L2 per FLOP (32 KiB instead of 48 KiB per 128 x 256 x 128-byte step)
// and gives the ring 50% more time in flight.  All loads are plain TMA
// (cta_group::2 completion on the leader's barrier, no multicast).
constexpr int kPairM = 256;                       // rows per pair tile
constexpr int kPairN = 256;                       // cols per pair tile
constexpr int kHalfN = kPairN / 2;                // B cols loaded per CTA
constexpr int kPairStages = 6;
constexpr int kPairAStage = kBM * kBKBytes;       // 16 KiB
constexpr int kPairBStage = kHalfN * kBKBytes;    // 16 KiB
constexpr size_t kPairRingBytes = (size_t)kPairStages * (kPairAStage + kPairBStage);
// Ring, alignment slack and the epilogue's TMA-store staging.
template <int DT>
constexpr size_t pair_smem_bytes() {
    return kPairRingBytes + 1024 + (size_t)epi_bytes<DT>();
}

__host__ __device__ constexpr uint32_t make_idesc_pair(uint32_t base_idesc) {
    // replace M (bits [24,29)) by 256
    return (base_idesc & ~(0x1Fu << 24)) | ((uint32_t)(kPairM >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if constexpr (KIND == 0) mma_pair_f16(d, a, b, idesc, acc);
    else if constexpr (KIND == 1) mma_pair_tf32(d, a, b, idesc, acc);
    else if constexpr (KIND == 2) mma_pair_f8f6f4(d, a, b, idesc, acc);
    else mma_pair_i8(d, a, b, idesc, acc);
}

template <int DT, bool KB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, void* __restrict__ C, int M, int N, int K,
                             float out_scale, SplitK sk) {
    using Tr = Traits<DT>;
    constexpr int kBKElems = kBKBytes / Tr::kEsize;
    constexpr int kBoxN = 128 / Tr::kEsize;
    constexpr int kBBoxes = kHalfN / kBoxN;                 // B boxes per CTA per stage
    constexpr int kBBoxBytes = kBKElems * 128;
    constexpr int kInstrKRows = kInstrKBytes / Tr::kEsize;
    constexpr uint32_t kIdesc = KB ? idesc_b_kmajor(make_idesc_pair(Tr::kIdesc)) : make_idesc_pair(Tr::kIdesc);

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kPairStages];   // leader: both CTAs' TMA bytes land here
    __shared__ __align__(8) uint64_t empty_bar[kPairStages];  // both: MMA finished reading the stage
    __shared__ __align__(8) uint64_t accf_bar[kNumAcc];       // both: accumulator ready for the epilogue
    __shared__ __align__(8) uint64_t acce_bar[kNumAcc];       // leader: both CTAs' epilogues drained it
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    __shared__ int last_split_flag;

    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t sA = smem_base;
    const uint32_t sB = smem_base + kPairStages * kPairAStage;
    const uint32_t sEpi = smem_base + (uint32_t)kPairRingBytes;  // TMA-store staging, 1 KiB aligned

    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;
    const int num_m = (M + kPairM - 1) / kPairM;
    const int num_n = (N + kPairN - 1) / kPairN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + kBKElems - 1) / kBKElems;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int a = 0; a < kNumAcc; ++a) {
            mbar_init(smem_u32(&accf_bar[a]), 1);
            mbar_init(smem_u32(&acce_bar[a]), 8);  // 4 epilogue warps x 2 CTAs
        }
        mbar_init(smem_u32(&drain_bar), 1);
        abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 0) {
        tmem_alloc_pair(smem_u32(&tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // barrier inits of both CTAs visible before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    grid_launch_dependents();  // the next grid may set up; its global accesses wait for this one

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs; completion on the leader's full barriers)
            grid_dependency_wait();  // A and B may be outputs of the previous grid
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            WorkItem it;
            for (int idx = 0; ok && work_item(idx, pair, num_pairs, num_tiles, num_kb, sk, it); ++idx) {
                int mb, nb;
                tile_coords(it.tile, num_m, num_n, sk.group_m, mb, nb);
                const int kb0 = it.kb0, kb1 = it.kb1;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_cluster(smem_u32(&empty_bar[stage]), phase ^ 1u, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrProducerWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t fb_local = smem_u32(&full_bar[stage]);
                    if (leader) mbar_arrive_expect_tx(fb_local, 2 * (kPairAStage + kPairBStage));
                    const uint32_t fb = fb_local & kPeerBitMask;
                    tma_load_2d_pair(sA + stage * kPairAStage, &tmA, fb, kb * kBKElems, mb * kPairM + rank * kBM);
                    if constexpr (KB) {
                        tma_load_2d_pair(sB + stage * kPairBStage, &tmB, fb, kb * kBKElems,
                                         nb * kPairN + rank * kHalfN);
                    } else {
#pragma unroll
                        for (int j = 0; j < kBBoxes; ++j)
                            tma_load_2d_pair(sB + stage * kPairBStage + j * kBBoxBytes, &tmB, fb,
                                             nb * kPairN + rank * kHalfN + j * kBoxN, kb * kBKElems);
                    }
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (leader)  // every armed phase completes only once both CTAs' bytes have landed
                for (int s = 0; s < kPairStages; ++s)
                    if (issued_mask & (1u << s))
                        if (!mbar_wait_cluster(smem_u32(&full_bar[s]), (issued_phase >> s) & 1u, nullptr))
                            atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer: the leader CTA only
            const uint64_t a_desc0 = make_sdesc(sA, 16, 1024);
            const uint64_t b_desc0 = KB ? make_sdesc(sB, 16, 1024)
                                        : make_sdesc(sB, kBBoxBytes, Tr::BLayout::kSbo, Tr::BLayout::kLayoutType);
            constexpr int kBKStep = KB ? kInstrKBytes : kInstrKRows * 128;
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            int t_local = 0;
            WorkItem it;
            for (int idx = 0; ok && work_item(idx, pair, num_pairs, num_tiles, num_kb, sk, it); ++idx, ++t_local) {
                const int kb0 = it.kb0, kb1 = it.kb1;
                const int chunk = unit_chunks(kb1 - kb0, sk.chunk_kb) > 1 ? sk.chunk_kb : kb1 - kb0;
                int acc = 0, chunk_left = 0;
                uint32_t d_tmem = tmem_base;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (chunk_left == 0) {  // a chunk starts: take the next accumulator, zero it by its first MMA
                        if (kb != kb0) {
                            tc_commit_pair_multicast(smem_u32(&accf_bar[acc]), 0x3);  // both CTAs fold it
                            ++t_local;
                        }
                        acc = t_local & 1;
                        if (!mbar_wait_cluster(smem_u32(&acce_bar[acc]), ((uint32_t)(t_local >> 1) & 1u) ^ 1u,
                                               &abort_flag)) {
                            atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                            abort_flag = 1;
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        d_tmem = tmem_base + (uint32_t)(acc * kPairN);
                        chunk_left = chunk;
                    }
                    const bool fresh = chunk_left == chunk;
                    --chunk_left;
                    if (!mbar_wait_cluster(smem_u32(&full_bar[stage]), phase, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint64_t a_stage = a_desc0 + (uint64_t)((stage * kPairAStage) >> 4);
                    const uint64_t b_stage = b_desc0 + (uint64_t)((stage * kPairBStage) >> 4);
#pragma unroll
                    for (int ks = 0; ks < kKSteps; ++ks)
                        mma_pair<Tr::kKind>(d_tmem, a_stage + (uint64_t)(ks * kInstrKBytes >> 4),
                                            b_stage + (uint64_t)(ks * kBKStep >> 4), kIdesc,
                                            (!fresh || ks != 0) ? 1u : 0u);
                    tc_commit_pair_multicast(smem_u32(&empty_bar[stage]), 0x3);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) tc_commit_pair_multicast(smem_u32(&accf_bar[acc]), 0x3);
            }
            tc_commit_pair_multicast(smem_u32(&drain_bar), 0x1);
            if (!mbar_wait_cluster(smem_u32(&drain_bar), 0, nullptr)) atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else {
        // ---------------- epilogue (both CTAs): warps 2..5 read this CTA's 128 accumulator rows
        grid_dependency_wait();  // C and the split-K workspace may be in use by the previous grid
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        const bool first_epi_thread = threadIdx.x == 64;
        const uint32_t acce_leader0 = mapa_shared(smem_u32(&acce_bar[0]), 0);
        const uint32_t acce_leader1 = mapa_shared(smem_u32(&acce_bar[1]), 0);
        int t_local = 0;
        uint32_t boxes = 0;  // TMA-store boxes this warp has issued (selects its staging buffer)
        WorkItem it;
        const uint32_t t_quarter = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int idx = 0; work_item(idx, pair, num_pairs, num_tiles, num_kb, sk, it); ++idx, ++t_local) {
            const int tile = it.tile;
            int mb, nb;
            tile_coords(tile, num_m, num_n, sk.group_m, mb, nb);
            const int nch = unit_chunks(it.kb1 - it.kb0, sk.chunk_kb);
            bool ok = true;
            for (int ch = 0; ch < nch; ++ch) {  // K chunks: fold each into the running sum (this CTA's half)
                if (ch > 0) ++t_local;
                const int a = t_local & 1;
                ok = mbar_wait_cluster(smem_u32(&accf_bar[a]), (uint32_t)(t_local >> 1) & 1u, &abort_flag);
                ok = __all_sync(0xffffffffu, ok);
                if (sk.splits > 1) ok = named_barrier_and(1, 128, ok);  // the fix-up below is CTA-wide
                if (!ok) break;
                tc_fence_after();
                if (ch > 0) {
                    fold_chunk<kPairN>(t_quarter + (uint32_t)((a ^ 1) * kPairN), t_quarter + (uint32_t)(a * kPairN),
                                       [&] {
                                           tc_fence_before();
                                           __syncwarp();
                                           if (lane == 0) mbar_arrive_cluster(a ? acce_leader0 : acce_leader1);
                                       });
                }
            }
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                    abort_flag = 1;
                }
                break;
            }
            const int acc = t_local & 1;
            const int grow = mb * kPairM + (int)rank * kBM + row_in_tile;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kPairN);
            const uint32_t acce_remote = acc ? acce_leader1 : acce_leader0;
            if (it.slot < 0) {
                const int row0 = mb * kPairM + (int)rank * kBM + q * 32;  // first row of this warp's boxes
#pragma unroll 1
                for (int c = 0; c < kPairN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                    tmem_wait_ld();
                    const int gcol = nb * kPairN + c * 32;
                    if (row0 >= M || gcol >= N) continue;  // warp-uniform: the box lies outside C
                    const uint32_t buf = sEpi + (uint32_t)((q * 2 + (int)(boxes & 1u)) * epi_box_bytes<DT>());
                    if (lane == 0) bulk_wait_read<1>();  // the store issued two boxes ago has read `buf`
                    __syncwarp();
                    stage_row<DT>(buf, lane, r, out_scale);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, buf, gcol, row0);
                        bulk_commit();
                    }
                    ++boxes;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acce_remote);
                continue;
            }
            // ---- split tile: slot (it.slot, rank) holds this CTA's 128-row partial
            // (blocks [16-byte column group][row], row-minor: a warp's stores are contiguous)
            const size_t slot = (size_t)it.slot * 2 + rank;
            uint4* wblk = reinterpret_cast<uint4*>(sk.ws) + slot * (kPairN / 4) * kBM + row_in_tile;
#pragma unroll 1
            for (int c = 0; c < kPairN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
                tmem_wait_ld();
                if (grow < M && nb * kPairN + c * 32 < N) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        wblk[(size_t)(c * 8 + i) * kBM] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acce_remote);
            __threadfence();
            named_barrier(1, 128);
            const size_t counter = (size_t)tile * 2 + rank;
            if (first_epi_thread)
                last_split_flag = atomicAdd(&sk.counters[counter], 1u) == (unsigned)(it.contributors - 1);
            named_barrier(1, 128);
            if (!last_split_flag) continue;
            __threadfence();
            if (grow < M) {
#pragma unroll 1
                for (int c = 0; c < kPairN / 32; ++c) {
                    const int gcol = nb * kPairN + c * 32;
                    if (gcol >= N) break;
                    float acc_f[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc_f[i] = 0.0f;
                    for (int sp = 0; sp < it.contributors; ++sp) {  // K order
                        const size_t sslot = (size_t)contributor_slot(tile, sp, sk) * 2 + rank;
                        const float4* ps = reinterpret_cast<const float4*>(sk.ws) +
                                           (sslot * (kPairN / 4) + (size_t)c * 8) * kBM + row_in_tile;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 v = __ldcg(ps + (size_t)i * kBM);
                            if constexpr (DT == TRB_INT8) {
                                acc_f[4 * i] = __int_as_float(__float_as_int(acc_f[4 * i]) + __float_as_int(v.x));
                                acc_f[4 * i + 1] = __int_as_float(__float_as_int(acc_f[4 * i + 1]) + __float_as_int(v.y));
                                acc_f[4 * i + 2] = __int_as_float(__float_as_int(acc_f[4 * i + 2]) + __float_as_int(v.z));
                                acc_f[4 * i + 3] = __int_as_float(__float_as_int(acc_f[4 * i + 3]) + __float_as_int(v.w));
                            } else if (sp == 0) {
                                acc_f[4 * i] = v.x; acc_f[4 * i + 1] = v.y; acc_f[4 * i + 2] = v.z; acc_f[4 * i + 3] = v.w;
                            } else {
                                acc_f[4 * i] += v.x; acc_f[4 * i + 1] += v.y; acc_f[4 * i + 2] += v.z; acc_f[4 * i + 3] += v.w;
                            }
                        }
                    }
                    uint32_t r[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(acc_f[i]);
                    store_chunk<DT>(C, grow, gcol, N, r, out_scale);
                }
            }
            if (first_epi_thread) sk.counters[counter] = 0u;
        }
        if (lane == 0) bulk_wait_all();  // this warp's TMA stores are complete before teardown
        __syncwarp();
    }

    // Teardown: the leader's MMAs read the peer's shared memory and write its
    // TMEM, so neither CTA releases TMEM or exits before both are done.
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------------ wide CTA-pair kernel
// The CTA pair with 256 x 512 tiles: each k-block's A rows feed two
// cta_group::2 MMAs (N = 256 each: tile columns [0, 256) and [256, 512)) into
// one 512-column accumulator per CTA, all of its TMEM.  Each SM then pulls
// 48 KiB from L2 per 128 x 512 x 128-byte step instead of 2 x 32 KiB: 25%
// fewer L2 -> SM bytes per FLOP, without multicast.  With no second
// accumulator the next tile waits until the epilogue has read this one out, so
// eight epilogue warps (two per TMEM lane quarter, 128 columns of each half
// apiece) copy it into registers as packed 16-bit results, release TMEM at
// once, and stage / store from registers while the next tile runs.  16-bit
// outputs only (bf16, f16, e4m3 -> bf16): 32-bit ones would not fit in
// registers.  Every accumulator sums its k-blocks in increasing order with the
// pair kernel's instructions, so the two agree bit for bit.  Whole tiles only.
constexpr int kWideN = 2 * kPairN;              // cols per wide tile
constexpr int kWideStages = 4;
constexpr int kWideBStage = 2 * kPairBStage;    // 32 KiB: this CTA's B columns of both halves
constexpr size_t kWideRingBytes = (size_t)kWideStages * (kPairAStage + kWideBStage);
constexpr int kWideEpiWarps = 8;
constexpr int kWideThreads = 64 + 32 * kWideEpiWarps;  // producer, MMA issuer, 8 epilogue warps
template <int DT>
__host__ __device__ constexpr size_t wide_smem_bytes() {
    return kWideRingBytes + 1024 + (size_t)kWideEpiWarps * 2 * epi_box_bytes<DT>();
}

// Two fp32 accumulator words -> one word of packed bf16 / f16 (convert16's rounding).
template <int DT>
__device__ __forceinline__ uint32_t pack2(uint32_t r0, uint32_t r1, float out_scale) {
    float lo = __uint_as_float(r0), hi = __uint_as_float(r1);
    if constexpr (DT == TRB_FLOAT8_E4M3FN) {
        lo *= out_scale;
        hi *= out_scale;
    }
    if constexpr (DT == TRB_FLOAT16) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

// Row `row` of a 16-bit staging box from 16 packed words (the layout of stage_row).
__device__ __forceinline__ void stage_row_packed(uint32_t buf, int row, const uint32_t (&w)[16]) {
    const uint32_t base = buf + (uint32_t)(row * 64);
    const int sw = (row >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        st_shared_v4(base + (uint32_t)((j ^ sw) * 16), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

template <int DT, bool KB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWideThreads, 1)
    gemm_tcgen05_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, int M, int N, int K, float out_scale,
                             int group_m) {
    using Tr = Traits<DT>;
    constexpr int kBKElems = kBKBytes / Tr::kEsize;
    constexpr int kBoxN = 128 / Tr::kEsize;
    constexpr int kBBoxes = kHalfN / kBoxN;                 // B boxes per CTA per half per stage
    constexpr int kBBoxBytes = kBKElems * 128;
    constexpr int kInstrKRows = kInstrKBytes / Tr::kEsize;
    constexpr uint32_t kIdesc = KB ? idesc_b_kmajor(make_idesc_pair(Tr::kIdesc)) : make_idesc_pair(Tr::kIdesc);
    static_assert(out_esize<DT>() == 2, "the wide pair holds 16-bit results in registers");
    static_assert(wide_smem_bytes<DT>() <= 227 * 1024, "wide pair shared memory");

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kWideStages];   // leader: both CTAs' TMA bytes land here
    __shared__ __align__(8) uint64_t empty_bar[kWideStages];  // both: MMA finished reading the stage
    __shared__ __align__(8) uint64_t accf_bar;                // both: the tile's accumulator is complete
    __shared__ __align__(8) uint64_t acce_bar;                // leader: both CTAs' epilogues read it out
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t sA = smem_base;
    const uint32_t sB = smem_base + kWideStages * kPairAStage;
    const uint32_t sEpi = smem_base + (uint32_t)kWideRingBytes;  // TMA-store staging, 1 KiB aligned

    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;
    const int num_m = (M + kPairM - 1) / kPairM;
    const int num_n = (N + kWideN - 1) / kWideN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + kBKElems - 1) / kBKElems;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWideStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(&accf_bar), 1);
        mbar_init(smem_u32(&acce_bar), 2 * kWideEpiWarps);  // 8 epilogue warps x 2 CTAs
        mbar_init(smem_u32(&drain_bar), 1);
        abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 0) {
        tmem_alloc_pair(smem_u32(&tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // barrier inits of both CTAs visible before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    grid_launch_dependents();  // the next grid may set up; its global accesses wait for this one

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs; completion on the leader's full barriers)
            grid_dependency_wait();  // A and B may be outputs of the previous grid
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += num_pairs) {
                int mb, nb;
                tile_coords(tile, num_m, num_n, group_m, mb, nb);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(smem_u32(&empty_bar[stage]), phase ^ 1u, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrProducerWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t fb_local = smem_u32(&full_bar[stage]);
                    if (leader) mbar_arrive_expect_tx(fb_local, 2 * (kPairAStage + kWideBStage));
                    const uint32_t fb = fb_local & kPeerBitMask;
                    tma_load_2d_pair(sA + stage * kPairAStage, &tmA, fb, kb * kBKElems, mb * kPairM + rank * kBM);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t dst = sB + stage * kWideBStage + h * kPairBStage;
                        const int col0 = nb * kWideN + h * kPairN + (int)rank * kHalfN;
                        if constexpr (KB) {
                            tma_load_2d_pair(dst, &tmB, fb, kb * kBKElems, col0);
                        } else {
#pragma unroll
                            for (int j = 0; j < kBBoxes; ++j)
                                tma_load_2d_pair(dst + j * kBBoxBytes, &tmB, fb, col0 + j * kBoxN, kb * kBKElems);
                        }
                    }
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kWideStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (leader)  // every armed phase completes only once both CTAs' bytes have landed
                for (int s = 0; s < kWideStages; ++s)
                    if (issued_mask & (1u << s))
                        if (!mbar_wait_cluster(smem_u32(&full_bar[s]), (issued_phase >> s) & 1u, nullptr))
                            atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer: the leader CTA only
            const uint64_t a_desc0 = make_sdesc(sA, 16, 1024);
            const uint64_t b_desc0 = KB ? make_sdesc(sB, 16, 1024)
                                        : make_sdesc(sB, kBBoxBytes, Tr::BLayout::kSbo, Tr::BLayout::kLayoutType);
            constexpr int kBKStep = KB ? kInstrKBytes : kInstrKRows * 128;
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            int t_local = 0;
            for (int tile = pair; ok && tile < num_tiles; tile += num_pairs, ++t_local) {
                // the epilogues have read the previous tile's accumulator out of TMEM
                if (!mbar_wait_cluster(smem_u32(&acce_bar), ((uint32_t)t_local & 1u) ^ 1u, &abort_flag)) {
                    atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(smem_u32(&full_bar[stage]), phase, &abort_flag)) {
                        atomicCAS(&g_gemm_error, 0, kErrMmaWait);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint64_t a_stage = a_desc0 + (uint64_t)((stage * kPairAStage) >> 4);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint64_t b_stage = b_desc0 + (uint64_t)((stage * kWideBStage + h * kPairBStage) >> 4);
                        const uint32_t d_tmem = tmem_base + (uint32_t)(h * kPairN);
#pragma unroll
                        for (int ks = 0; ks < kKSteps; ++ks)
                            mma_pair<Tr::kKind>(d_tmem, a_stage + (uint64_t)(ks * kInstrKBytes >> 4),
                                                b_stage + (uint64_t)(ks * kBKStep >> 4), kIdesc,
                                                (kb != 0 || ks != 0) ? 1u : 0u);
                    }
                    tc_commit_pair_multicast(smem_u32(&empty_bar[stage]), 0x3);
                    if (++stage == kWideStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) tc_commit_pair_multicast(smem_u32(&accf_bar), 0x3);
            }
            tc_commit_pair_multicast(smem_u32(&drain_bar), 0x1);
            if (!mbar_wait_cluster(smem_u32(&drain_bar), 0, nullptr)) atomicCAS(&g_gemm_error, 0, kErrDrainWait);
        }
    } else {
        // ---------------- epilogue (both CTAs): warps 2..9; warp w reads TMEM lanes
        // [32 (w % 4), +32) -- this CTA's accumulator rows -- in columns [128 cb, +128) of each
        // half, cb = (w - 2) / 4: 8 boxes of 32 x 32 results per tile
        grid_dependency_wait();  // C may be in use by the previous grid
        const int q = warp & 3;
        const int ew = warp - 2;
        const int cb = ew >> 2;
        const uint32_t acce_leader = mapa_shared(smem_u32(&acce_bar), 0);
        const uint32_t t_rows = tmem_base + ((uint32_t)(q * 32) << 16);
        uint32_t boxes = 0;  // TMA-store boxes this warp has issued (selects its staging buffer)
        int t_local = 0;
        for (int tile = pair; tile < num_tiles; tile += num_pairs, ++t_local) {
            int mb, nb;
            tile_coords(tile, num_m, num_n, group_m, mb, nb);
            bool ok = mbar_wait_cluster(smem_u32(&accf_bar), (uint32_t)t_local & 1u, &abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
                    abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            uint32_t w[8][16];  // box i: half i / 4, columns 128 cb + 32 (i % 4) of that half
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t r0[16], r1[16];  // two loads of 16 columns in flight per wait
                const uint32_t col = (uint32_t)((i >> 2) * kPairN + cb * 128 + (i & 3) * 32);
                tmem_ld_32x32b_x16(t_rows + col, r0);
                tmem_ld_32x32b_x16(t_rows + col + 16, r1);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    w[i][j] = pack2<DT>(r0[2 * j], r0[2 * j + 1], out_scale);
                    w[i][8 + j] = pack2<DT>(r1[2 * j], r1[2 * j + 1], out_scale);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acce_leader);  // TMEM free: the next tile may start
            const int row0 = mb * kPairM + (int)rank * kBM + q * 32;  // first row of this warp's boxes
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int gcol = nb * kWideN + (i >> 2) * kPairN + cb * 128 + (i & 3) * 32;
                if (row0 >= M || gcol >= N) continue;  // warp-uniform: the box lies outside C
                const uint32_t buf = sEpi + (uint32_t)((ew * 2 + (int)(boxes & 1u)) * epi_box_bytes<DT>());
                if (lane == 0) bulk_wait_read<1>();  // the store issued two boxes ago has read `buf`
                __syncwarp();
                stage_row_packed(buf, lane, w[i]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, buf, gcol, row0);
                    bulk_commit();
                }
                ++boxes;
            }
        }
        if (lane == 0) bulk_wait_all();  // this warp's TMA stores are complete before teardown
        __syncwarp();
    }

    // Teardown: the leader's MMAs read the peer's shared memory and write its
    // TMEM, so neither CTA releases TMEM or exits before both are done.
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

static int encode_2d(CUtensorMap* map, const void* base, int esize, uint64_t inner, uint64_t outer,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (fn == nullptr) {
        set_error("cuTensorMapEncodeTiled entry point unavailable");
        return TRB_ERR_CUDA;
    }
    const CUtensorMapDataType dt = esize == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * (uint64_t)esize};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u", (int)r, (unsigned long long)inner,
                  (unsigned long long)outer, box_inner, box_outer);
        return TRB_ERR_CUDA;
    }
    return TRB_OK;
}

// Split-K workspace of one device: fp32 partials + per-tile arrival counters.
// Grow-only, allocated on first use; counters are zeroed when allocated and
// every launch leaves them at zero.  Launches that overlap on one device
// would share it, hence the one-call-per-device rule of the C ABI.
struct Workspace {
    float* ws = nullptr;
    size_t ws_bytes = 0;
    unsigned int* counters = nullptr;
    size_t counter_count = 0;
    std::mutex mu;
};
static Workspace g_workspace[64];

static int ensure_workspace(int dev, size_t ws_bytes, size_t counters, SplitK* sk) {
    if (dev < 0 || dev >= 64) {
        set_error("device id %d out of range for the split-K workspace", dev);
        return TRB_ERR_ARGS;
    }
    Workspace& w = g_workspace[dev];
    std::lock_guard<std::mutex> lock(w.mu);
    if (w.ws_bytes < ws_bytes) {
        if (w.ws) cudaFree(w.ws);
        w.ws = nullptr;
        w.ws_bytes = 0;
        TRB_CUDA(cudaMalloc(&w.ws, ws_bytes));
        w.ws_bytes = ws_bytes;
    }
    if (w.counter_count < counters) {
        if (w.counters) cudaFree(w.counters);
        w.counters = nullptr;
        w.counter_count = 0;
        TRB_CUDA(cudaMalloc(&w.counters, counters * sizeof(unsigned int)));
        TRB_CUDA(cudaMemset(w.counters, 0, counters * sizeof(unsigned int)));
        w.counter_count = counters;
    }
    sk->ws = w.ws;
    sk->counters = w.counters;
    return TRB_OK;
}

// Splits for a problem: split K only when the output tiles leave more than
// half of the SMs idle (skinny M or small N), keeping >= 4 k-blocks per split.
static int choose_splits(long tiles, int num_kb, int sms) {
    if (tiles * 2 > sms) return 1;
    long s = std::min<long>(sms / std::max<long>(tiles, 1), num_kb / 4);
    return (int)std::max<long>(1, std::min<long>(s, 16));
}


// Automatic kernel choice for M > 64: the candidate with the highest
//   (work units / (waves x slots)) x per-tile efficiency,
// where slots are the SMs (single CTA) or SM pairs (CTA pair).  Per-tile
// factors, relative to the CTA pair, calibrated on B200 (bf16 and e4m3,
// 1024^3 ... 16384^3, CUDA-graph timing): 128 x 256 single-CTA tiles 0.89,
// 128 x 128 0.72, 128 x 64 0.50.  A CTA that owns one tile cannot hide its
// pipeline fill and epilogue behind a next tile, which costs the pair (heavier
// setup) its edge on a short K loop: the pair's factor is 0.85 when it runs a
// single wave with < 40 k-blocks (bf16 2048^3: 128 x 256 tiles 1099 TFLOP/s
// vs the pair 1031; e4m3 4096^3, four waves: the pair 2721 vs 2499).
// Cluster split-K (256-wide tiles, x 0.85 for its exchange) is a candidate
// only when every split keeps >= 16 k-blocks and all clusters are
// co-resident.  Workspace split-K lost in every measured case; it is used
// only when no candidate fills a quarter of the slots and K is long
// (>= 256 k-blocks, e.g. 256 x 256 x 65536), where its fix-up amortises.
// Picks: 1024^3 -> 128 x 64, 1536^3 -> 128 x 128, 2048^3 -> 128 x 256,
// >= 2560^3 -> pair, M = 128 x N = K = 8192 -> 128 x 256 with clusters of 4.
struct KernelChoice {
    bool pair;
    int tile_n;
    int cluster;
    double score;
};
template <typename Capacity>
static KernelChoice choose_kernel(int m, int n, int num_kb, bool allow_bn64, int sms, Capacity capacity) {
    auto wave_eff = [](long units, long slots) {
        if (units <= 0 || slots <= 0) return 0.0;
        const long waves = (units + slots - 1) / slots;
        return (double)units / (double)(waves * slots);
    };
    const long mb = (m + kBM - 1) / kBM;
    // One row of tiles (M <= 128) is an HBM stream: what counts is filling the
    // SMs and, for split-K, the fp32 partial each CTA exchanges.  Candidates in
    // order of preference at equal SM fill: 128-wide tiles in clusters of 2
    // (32 KB exchanged per CTA), 256-wide in clusters of 4 (96 KB), 128-wide
    // in 4, 256-wide in 2 and 8.  Measured at M = 128, N = K = 8192 (bf16 /
    // e4m3): 128 x 2: 29.0 / 15.0 us, 256 x 4: 31.0 / 16.7, 256 x 2: 35.3,
    // 128 x 4: 35.6, best no-split narrow tiles: 36.1 / 20.6.
    if (mb == 1) {
        struct Cand { int bn, cl; double pref; };
        const Cand cands[] = {{128, 2, 1.0}, {256, 4, 0.95}, {128, 4, 0.9}, {256, 2, 0.9}, {256, 8, 0.85}};
        KernelChoice pick{false, 256, 1, -1.0};
        for (const Cand& c : cands) {
            const long tiles = (n + c.bn - 1) / c.bn;
            const int kbps = (num_kb + c.cl - 1) / c.cl;
            if (kbps < 16 || (long)(c.cl - 1) * kbps >= num_kb || tiles > capacity(c.cl) || tiles * c.cl > sms)
                continue;
            const double score = wave_eff(tiles * c.cl, sms) * c.pref;
            if (score > pick.score + 1e-9) pick = {false, c.bn, c.cl, score};
        }
        if (pick.score >= 0.5) return pick;
    }
    KernelChoice best{sms >= 2, 256, 1, 0.0};
    double best_score = -1.0;
    if (sms >= 2) {
        const long tiles = (long)((m + kPairM - 1) / kPairM) * ((n + kPairN - 1) / kPairN);
        const bool one_wave = tiles <= sms / 2;
        best_score = wave_eff(tiles, sms / 2) * (one_wave && num_kb < 40 ? 0.85 : 1.0);
    }
    // Per-tile efficiency of the single-CTA widths relative to the CTA pair,
    // from full-wave runs at 4096^3 bf16 (105 / 120 / 177 us for 256 / 128 /
    // 64 wide; the 64- and 128-wide rings take 4 and 2 k-blocks per stage).
    for (int bn : {256, 128, 64}) {
        if (bn == 64 && !allow_bn64) continue;
        const double f = bn == 256 ? 0.89 : bn == 128 ? 0.78 : 0.53;
        const double score = wave_eff(mb * ((n + bn - 1) / bn), sms) * f;
        if (score > best_score + 1e-9) {
            best_score = score;
            best = {false, bn, 1, score};
        }
    }
    const long tiles256 = mb * ((n + 255) / 256);
    for (int cl : {2, 4, 8}) {  // general case: 256-wide tiles
        const int kbps = (num_kb + cl - 1) / cl;
        if (kbps < 16 || (long)(cl - 1) * kbps >= num_kb || tiles256 > capacity(cl)) continue;
        const double score = wave_eff(tiles256 * cl, sms) * 0.89 * 0.85;
        if (score > best_score + 1e-9) {
            best_score = score;
            best = {false, 256, cl, score};
        }
    }
    best.score = best_score;
    return best;
}

// Raster group: consecutive tiles walk down `group` m-blocks of one column
// of tiles, so the group's A rows and one B column panel are what the
// running tiles share in L2.  Measured on B200 for the CTA pair:
//  * A panels above 2 MB per m-block: 8 is best (bf16 8192^3 / 16384^3 1520 /
//    1514 TFLOP/s vs 1482 / 1465 with 16 and 1487 / 1419 with 4; e4m3 16384^3
//    3030 vs 2910 with 16);
//  * panels of 2 MB or less take 16 (e4m3 8192^3 3049 vs 2997, bf16 4096^3
//    1512 vs 1485, int8 8192^3 +1%);
// single-CTA tiles (not measured with 16) keep 8; and the group's A rows are
// kept under ~80 MB of the 126 MB L2 for very long K.
static int raster_group(int rows_per_block, int k, int es) {
    const double a_bytes = (double)rows_per_block * k * es;
    const int g = (int)(80.0e6 / a_bytes);
    const int cap = (rows_per_block == kPairM && a_bytes <= 2.1e6) ? 16 : 8;
    return std::max(2, std::min(cap, g));
}

// Launch with programmatic stream serialization (the kernels' griddepcontrol
// waits order their global accesses after the previous grid) and, for
// cluster split-K, the cluster shape.
template <typename Kernel, typename... Args>
static int launch_ex_threads(Kernel kernel, int grid, int threads, size_t smem, int cluster, cudaStream_t stream,
                             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    int nattr = 0;
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
    if (cluster > 1) {
        attr[nattr].id = cudaLaunchAttributeClusterDimension;
        attr[nattr].val.clusterDim.x = (unsigned)cluster;
        attr[nattr].val.clusterDim.y = 1;
        attr[nattr].val.clusterDim.z = 1;
        ++nattr;
    }
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    TRB_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...));
    return TRB_OK;
}

template <typename Kernel, typename... Args>
static int launch_ex(Kernel kernel, int grid, size_t smem, int cluster, cudaStream_t stream, Args... args) {
    return launch_ex_threads(kernel, grid, kThreads, smem, cluster, stream, args...);
}

template <int DT, bool KB, int BN, int CL = 1>
static int launch_single(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, int m, int n,
                         int k, void* c, float out_scale, int splits, int dev, int sms, cudaStream_t stream,
                         LaunchInfo* info) {
    using Tr = Traits<DT>;
    using Cfg = TileCfgFor<DT, BN, CL>;
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev]) {
        TRB_CUDA(cudaFuncSetAttribute(gemm_tcgen05_kernel<DT, KB, BN, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)Cfg::kSmem));
        attr_set[dev] = true;
    }
    const long tiles = (long)((m + kBM - 1) / kBM) * ((n + BN - 1) / BN);
    const int num_kb = (int)(((long)k * Tr::kEsize + kBKBytes - 1) / kBKBytes);
    SplitK sk{1, num_kb, nullptr, nullptr, m <= kBM ? 1 : 0, raster_group(kBM, k, Tr::kEsize), chain_kb<DT>()};
    int grid;
    if constexpr (CL > 1) {
        sk.splits = CL;
        sk.kb_per_split = (num_kb + CL - 1) / CL;  // the caller checked that every split owns >= 1 k-block
        grid = (int)(tiles * CL);
    } else {
        if (splits <= 0) splits = choose_splits(tiles, num_kb, sms);
        splits = std::max(1, std::min(splits, num_kb));
        const int kbps = (num_kb + splits - 1) / splits;
        splits = (num_kb + kbps - 1) / kbps;  // every split owns at least one k-block
        sk.splits = splits;
        sk.kb_per_split = kbps;
        if (splits > 1) {
            const int rc = ensure_workspace(dev, (size_t)tiles * splits * kBM * BN * sizeof(float), (size_t)tiles, &sk);
            if (rc != TRB_OK) return rc;
        }
        grid = (int)std::max<long>(1, std::min<long>(tiles * splits, sms));
    }
    const int rc = launch_ex(gemm_tcgen05_kernel<DT, KB, BN, CL>, grid, Cfg::kSmem, CL, stream, tmA, tmB, tmC, c, m, n, k,
                             out_scale, sk);
    if (rc != TRB_OK) return rc;
    TRB_CUDA(cudaGetLastError());
    if (info) {
        *info = LaunchInfo{};
        info->grid = grid;
        info->block = kThreads;
        info->splits = sk.splits;
        info->tile_n = BN;
        info->cluster = CL;
    }
    return TRB_OK;
}

// How many clusters of `cl` CTAs of one-CTA-per-SM kernels the device runs at
// once (GPC boundaries: 74 / 33 / 15 clusters of 2 / 4 / 8 on a 148-SM B200).
// Queried once per device and size with a representative cluster kernel.
template <typename Kernel>
static int cluster_capacity(Kernel kernel, size_t smem, int dev, int cl) {
    static int cache[64][9] = {};
    const int slot = cl == 2 ? 2 : cl == 4 ? 4 : 8;
    if (dev >= 0 && dev < 64 && cache[dev][slot] > 0) return cache[dev][slot];
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(cl * 32));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    if (dev >= 0 && dev < 64 && n > 0) cache[dev][slot] = n;
    return n;
}

// Split count for the swapped kernel: minimise waves x k-blocks per unit
// (+2 k-blocks of per-unit overhead: pipeline fill and epilogue), keeping
// >= 4 k-blocks per split.  Ties keep the smaller split count.
static int choose_swap_splits(long tiles, int num_kb, int sms) {
    int best = 1;
    long best_cost = -1;
    const int max_s = std::max(1, std::min(32, num_kb / 4));
    for (int s = 1; s <= max_s; ++s) {
        const int kbps = (num_kb + s - 1) / s;
        const int s_eff = (num_kb + kbps - 1) / kbps;
        const long waves = (tiles * s_eff + sms - 1) / sms;
        const long cost = waves * (kbps + 2);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s_eff;
        }
    }
    return best;
}

template <int DT, bool KB, int BS, int KD, int CL>
static int launch_swap(const void* a, const void* b, int m, int n, int k, void* c, float out_scale, int splits,
                       int dev, int sms, cudaStream_t stream, LaunchInfo* info) {
    using Tr = Traits<DT>;
    using Cfg = SwapCfg<BS, KD, CL>;
    constexpr int es = Tr::kEsize;
    CUtensorMap tmW, tmS;
    int rc = KB ? encode_2d(&tmW, b, es, (uint64_t)k, (uint64_t)n, kBKBytes / es, kBM, CU_TENSOR_MAP_SWIZZLE_128B)
                : encode_2d(&tmW, b, es, (uint64_t)n, (uint64_t)k, 128 / es, KD * kBKBytes / es,
                            Tr::BLayout::kTmaSwizzle);
    if (rc != TRB_OK) return rc;
    rc = encode_2d(&tmS, a, es, (uint64_t)k, (uint64_t)m, kBKBytes / es, BS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TRB_OK) return rc;
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev]) {
        TRB_CUDA(cudaFuncSetAttribute(gemm_swap_kernel<DT, KB, BS, KD, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)Cfg::kSmem));
        attr_set[dev] = true;
    }
    const long tiles = (n + kBM - 1) / kBM;
    const int num_kb = (int)(((long)k * es + kBKBytes - 1) / kBKBytes);
    // No K rotation: the S box is only BS x 128 bytes, and CTAs that walk K in
    // step read whole rows of B together (measured 29.1 vs 30.7 us at
    // M = 16, N = K = 8192 bf16 with per-tile rotation).
    SplitK sk{1, num_kb, nullptr, nullptr, 0, 0, chain_kb<DT>()};
    int grid;
    if constexpr (CL > 1) {
        sk.splits = CL;
        sk.kb_per_split = (num_kb + CL - 1) / CL;  // the caller checked that every split owns >= 1 k-block
        grid = (int)(tiles * CL);
    } else {
        if (splits <= 0) splits = choose_swap_splits(tiles, num_kb, sms);
        splits = std::max(1, std::min(splits, num_kb));
        const int kbps = (num_kb + splits - 1) / splits;
        splits = (num_kb + kbps - 1) / kbps;
        sk.splits = splits;
        sk.kb_per_split = kbps;
        if (splits > 1) {
            rc = ensure_workspace(dev, (size_t)tiles * splits * kBM * BS * sizeof(float), (size_t)tiles, &sk);
            if (rc != TRB_OK) return rc;
        }
        grid = (int)std::max<long>(1, std::min<long>(tiles * splits, sms));
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    int nattr = 0;
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
    if (CL > 1) {
        attr[nattr].id = cudaLaunchAttributeClusterDimension;
        attr[nattr].val.clusterDim.x = CL;
        attr[nattr].val.clusterDim.y = 1;
        attr[nattr].val.clusterDim.z = 1;
        ++nattr;
    }
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    TRB_CUDA(cudaLaunchKernelEx(&cfg, gemm_swap_kernel<DT, KB, BS, KD, CL>, tmW, tmS, c, m, n, k, out_scale, sk));
    TRB_CUDA(cudaGetLastError());
    if (info) {
        *info = LaunchInfo{};
        info->grid = grid;
        info->block = kThreads;
        info->splits = sk.splits;
        info->tile_n = BS;
        info->swap = 1;
        info->cluster = CL;
    }
    return TRB_OK;
}

// Cluster split count for the swapped kernel: the largest of 8, 4, 2 whose
// tiles x splits CTAs fit on the SMs at once with >= 4 k-blocks per split
// (every split non-empty); 1 when the panels alone fill most SMs or no count fits.
template <typename Capacity>
static int choose_swap_cluster(long tiles, int num_kb, int sms, Capacity capacity) {
    if (tiles * 2 > sms) return 1;
    for (int cl : {8, 4, 2}) {
        const int kbps = (num_kb + cl - 1) / cl;
        if (tiles * cl <= sms && num_kb >= 4 * cl && (long)(cl - 1) * kbps < num_kb && tiles <= capacity(cl)) return cl;
    }
    return 1;
}

// K-blocks per stage: 2 (MN-major W boxes 2 k-blocks tall measured 4-7% faster
// than 1; 4 gave no further gain).  cluster: < 0 automatic, 0 = global
// workspace split-K (`splits`), 2 / 4 / 8 = cluster split-K of that size.
template <int DT, bool KB, int BS>
static int launch_swap_kd(int cluster, const void* a, const void* b, int m, int n, int k, void* c, float out_scale,
                          int splits, int dev, int sms, cudaStream_t stream, LaunchInfo* info) {
    constexpr int kKD = 2;
    constexpr int es = Traits<DT>::kEsize;
    const long tiles = (n + kBM - 1) / kBM;
    const int num_kb = (int)(((long)k * es + kBKBytes - 1) / kBKBytes);
    int cl = cluster;
    if (cl < 0) {
        auto capacity = [dev](int c) {
            return c == 2   ? cluster_capacity(gemm_swap_kernel<DT, KB, BS, kKD, 2>, SwapCfg<BS, kKD, 2>::kSmem, dev, 2)
                   : c == 4 ? cluster_capacity(gemm_swap_kernel<DT, KB, BS, kKD, 4>, SwapCfg<BS, kKD, 4>::kSmem, dev, 4)
                            : cluster_capacity(gemm_swap_kernel<DT, KB, BS, kKD, 8>, SwapCfg<BS, kKD, 8>::kSmem, dev, 8);
        };
        cl = splits > 0 ? 1 : choose_swap_cluster(tiles, num_kb, sms, capacity);
    }
    if (cl > 1) {
        const int kbps = (num_kb + cl - 1) / cl;
        if ((cl != 2 && cl != 4 && cl != 8) || (long)(cl - 1) * kbps >= num_kb) {
            set_error("trb_gemm_launch: cluster split-K of %d needs every split to own a k-block (%d k-blocks)", cl,
                      num_kb);
            return TRB_ERR_ARGS;
        }
    }
    switch (cl) {
        case 2: return launch_swap<DT, KB, BS, kKD, 2>(a, b, m, n, k, c, out_scale, 0, dev, sms, stream, info);
        case 4: return launch_swap<DT, KB, BS, kKD, 4>(a, b, m, n, k, c, out_scale, 0, dev, sms, stream, info);
        case 8: return launch_swap<DT, KB, BS, kKD, 8>(a, b, m, n, k, c, out_scale, 0, dev, sms, stream, info);
        default: return launch_swap<DT, KB, BS, kKD, 1>(a, b, m, n, k, c, out_scale, splits, dev, sms, stream, info);
    }
}

// The 256 x 512 CTA pair: whole tiles, one persistent pair per SM pair.
template <int DT, bool KB>
static int launch_wide(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, int m, int n, int k,
                       float out_scale, int group_m, int dev, int sms, cudaStream_t stream, LaunchInfo* info) {
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev]) {
        TRB_CUDA(cudaFuncSetAttribute(gemm_tcgen05_wide_kernel<DT, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)wide_smem_bytes<DT>()));
        attr_set[dev] = true;
    }
    const long tiles = (long)((m + kPairM - 1) / kPairM) * ((n + kWideN - 1) / kWideN);
    const int grid_workers = (int)std::max<long>(1, std::min<long>(tiles, sms / 2));
    const int rc = launch_ex_threads(gemm_tcgen05_wide_kernel<DT, KB>, grid_workers * 2, kWideThreads,
                                     wide_smem_bytes<DT>(), 1, stream, tmA, tmB, tmC, m, n, k, out_scale, group_m);
    if (rc != TRB_OK) return rc;
    TRB_CUDA(cudaGetLastError());
    if (info) {
        *info = LaunchInfo{};
        info->grid = grid_workers * 2;
        info->block = kWideThreads;
        info->pair = 1;
        info->tile_n = kWideN;
    }
    return TRB_OK;
}

template <int DT, bool KB>
static int launch_typed(int m, int n, int k, const void* a, const void* b, void* c, float out_scale, int splits,
                        int cta_pair, int tile_n_opt, cudaStream_t stream, LaunchInfo* info) {
    using Tr = Traits<DT>;
    constexpr int es = Tr::kEsize;
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    // M <= 64: swapped operands (C^T = B^T A^T), unless a kernel is forced.
    if (tile_n_opt < 0 || (tile_n_opt == 0 && cta_pair < 0 && m <= 64)) {
        if (m > 64) {
            set_error("trb_gemm_launch: the swapped-operand kernel takes m <= 64 (got %d)", m);
            return TRB_ERR_ARGS;
        }
        // splits < 0: cluster split-K of -splits CTAs; > 0: workspace split-K; 0: automatic.
        const int cluster = splits < 0 ? -splits : (splits > 0 ? 0 : -1);
        if (m <= 16) return launch_swap_kd<DT, KB, 16>(cluster, a, b, m, n, k, c, out_scale, splits, dev, sms, stream, info);
        if (m <= 32) return launch_swap_kd<DT, KB, 32>(cluster, a, b, m, n, k, c, out_scale, splits, dev, sms, stream, info);
        return launch_swap_kd<DT, KB, 64>(cluster, a, b, m, n, k, c, out_scale, splits, dev, sms, stream, info);
    }
    // Forced choices first (tile_n, splits, cta_pair); the automatic choice is
    // choose_kernel's wave model below.
    int tile_n_single = 256;
    if (tile_n_opt > 0) {
        if (tile_n_opt != 64 && tile_n_opt != 128 && tile_n_opt != 256) {
            set_error("trb_gemm_launch: tile_n must be 64, 128 or 256 (got %d)", tile_n_opt);
            return TRB_ERR_ARGS;
        }
        if (tile_n_opt == 64 && es == 1 && !KB) {
            set_error("trb_gemm_launch: 8-bit row-major B needs tile_n >= 128");
            return TRB_ERR_ARGS;
        }
        tile_n_single = tile_n_opt;
    }
    const int num_kb = (int)(((long)k * es + kBKBytes - 1) / kBKBytes);
    int cluster = 1;
    bool pair_auto = false;
    if (splits < 0) {
        // Cluster split-K of the single-CTA kernel with 256-wide tiles.
        cluster = -splits;
        const int kbps = (num_kb + cluster - 1) / cluster;
        const int bn = tile_n_opt > 0 ? tile_n_opt : 256;
        if ((cluster != 2 && cluster != 4 && cluster != 8) || cta_pair > 0 || (bn != 256 && bn != 128) ||
            (bn / cluster) % 32 != 0 || (long)(cluster - 1) * kbps >= num_kb) {
            set_error("trb_gemm_launch: cluster split-K takes 2, 4 or 8 splits of 256-wide (or 2 / 4 of 128-wide) "
                      "single-CTA tiles, each split owning a k-block (splits %d, tile_n %d, %d k-blocks)", splits, bn,
                      num_kb);
            return TRB_ERR_ARGS;
        }
        tile_n_single = bn;
    } else if (splits == 0 && cta_pair < 0 && tile_n_opt == 0) {
        auto capacity = [dev](int c) {
            return c == 2   ? cluster_capacity(gemm_tcgen05_kernel<DT, KB, 256, 2>, TileCfgFor<DT, 256, 2>::kSmem, dev, 2)
                   : c == 4 ? cluster_capacity(gemm_tcgen05_kernel<DT, KB, 256, 4>, TileCfgFor<DT, 256, 4>::kSmem, dev, 4)
                            : cluster_capacity(gemm_tcgen05_kernel<DT, KB, 256, 8>, TileCfgFor<DT, 256, 8>::kSmem, dev, 8);
        };
        const KernelChoice kc = choose_kernel(m, n, num_kb, KB || es >= 2, sms, capacity);
        pair_auto = kc.pair;
        tile_n_single = kc.tile_n;
        cluster = kc.cluster;
        if (kc.score >= 0.25 || num_kb < 256) splits = 1;  // else: workspace split-K count chosen below
    } else if (cta_pair < 0 && tile_n_opt == 0) {
        pair_auto = true;  // explicit workspace split-K count: the pair, as before
    }
    const bool pair = cluster == 1 && (cta_pair > 0 || pair_auto) && sms >= 2;
    const int tile_n = pair ? kPairN : tile_n_single;
    if (cta_pair == 2 && (!pair || out_esize<DT>() != 2 || splits > 1 || tile_n_opt != 0)) {
        set_error("trb_gemm_launch: cta_pair = 2 (CTA pair, 256 x 512 tiles) takes whole tiles (splits 0 or 1, "
                  "tile_n 0) of bf16, f16 or e4m3 inputs");
        return TRB_ERR_ARGS;
    }
    // Automatic: the 256 x 512 pair replaces a whole-tile 256 x 256 pair for
    // bf16 / f16 inputs with >= 64 k-blocks when its tiles fill the SM pairs
    // as well (waves x useful columns).  Measured on B200 against the 256 x 256
    // pair, each burst after an idle gap: bf16 8192^3 +4.2% (1621 vs 1555
    // TFLOP/s; cuBLAS 1610), 16384^3 +6.6%, 6144^3 +1.6%, 4096^3 +0.4%; f16
    // 8192^3 +4.8%; ~2 s power-capped loops: bf16 8192^3 +4.1% (1411; cuBLAS
    // 1390).  Not taken for e4m3 (+0.4% / +0.5%: its tiles are half as long, so
    // the accumulator hand-off eats the gain) or short K (bf16 8192^2 x 2048: -0.8%).
    bool wide = cta_pair == 2;
    if (!wide && pair && pair_auto && splits == 1 && (DT == TRB_BFLOAT16 || DT == TRB_FLOAT16) && num_kb >= 64) {
        const int workers = sms / 2;
        auto fill = [workers](long units, long cols, long tile_cols) {  // wave fill x useful share of the columns
            const long waves = (units + workers - 1) / workers;
            const long padded = tile_cols * ((cols + tile_cols - 1) / tile_cols);
            return (double)units / (double)(waves * workers) * (double)cols / (double)padded;
        };
        const long mrows = (m + kPairM - 1) / kPairM;
        const double f_pair = fill(mrows * ((n + kPairN - 1) / kPairN), n, kPairN);
        const double f_wide = fill(mrows * ((n + kWideN - 1) / kWideN), n, kWideN);
        wide = f_wide >= f_pair - 0.01;
    }

    CUtensorMap tmA, tmB;
    int rc = encode_2d(&tmA, a, es, (uint64_t)k, (uint64_t)m, kBKBytes / es, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TRB_OK) return rc;
    if (KB)  // B^T: N rows of K elements, boxes of (128-byte K slice) x (tile N rows)
        rc = encode_2d(&tmB, b, es, (uint64_t)k, (uint64_t)n, kBKBytes / es, pair ? kHalfN : tile_n,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    else
        rc = encode_2d(&tmB, b, es, (uint64_t)n, (uint64_t)k, 128 / es, kBKBytes / es, Tr::BLayout::kTmaSwizzle);
    if (rc != TRB_OK) return rc;
    // C as TMA-store boxes of 32 rows x 32 columns (whole-tile epilogues).
    CUtensorMap tmC;
    rc = encode_2d(&tmC, c, out_esize<DT>(), (uint64_t)n, (uint64_t)m, 32, 32,
                   out_esize<DT>() == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TRB_OK) return rc;
    if (cluster > 1 && tile_n_single == 128) {
        if (cluster == 2) return launch_single<DT, KB, 128, 2>(tmA, tmB, tmC, m, n, k, c, out_scale, 0, dev, sms, stream, info);
        return launch_single<DT, KB, 128, 4>(tmA, tmB, tmC, m, n, k, c, out_scale, 0, dev, sms, stream, info);
    }
    if (cluster == 2) return launch_single<DT, KB, 256, 2>(tmA, tmB, tmC, m, n, k, c, out_scale, 0, dev, sms, stream, info);
    if (cluster == 4) return launch_single<DT, KB, 256, 4>(tmA, tmB, tmC, m, n, k, c, out_scale, 0, dev, sms, stream, info);
    if (cluster == 8) return launch_single<DT, KB, 256, 8>(tmA, tmB, tmC, m, n, k, c, out_scale, 0, dev, sms, stream, info);
    if (!pair) {
        if (tile_n == 64) {
            if constexpr (KB || es >= 2)
                return launch_single<DT, KB, 64>(tmA, tmB, tmC, m, n, k, c, out_scale, splits, dev, sms, stream, info);
        } else if (tile_n == 128) {
            return launch_single<DT, KB, 128>(tmA, tmB, tmC, m, n, k, c, out_scale, splits, dev, sms, stream, info);
        }
        return launch_single<DT, KB, 256>(tmA, tmB, tmC, m, n, k, c, out_scale, splits, dev, sms, stream, info);
    }
    if (wide) {
        if constexpr (out_esize<DT>() == 2)
            return launch_wide<DT, KB>(tmA, tmB, tmC, m, n, k, out_scale, raster_group(kPairM, k, es), dev, sms, stream,
                                       info);
    }
    static bool attr_set[64] = {};
    if (dev < 64 && !attr_set[dev]) {
        TRB_CUDA(cudaFuncSetAttribute(gemm_tcgen05_pair_kernel<DT, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pair_smem_bytes<DT>()));
        attr_set[dev] = true;
    }
    const int workers = sms / 2;
    const long tiles = (long)((m + kPairM - 1) / kPairM) * ((n + kPairN - 1) / kPairN);
    if (splits <= 0) splits = choose_splits(tiles, num_kb, workers);
    splits = std::max(1, std::min(splits, num_kb));
    const int kbps = (num_kb + splits - 1) / splits;
    splits = (num_kb + kbps - 1) / kbps;
    SplitK sk{splits, kbps, nullptr, nullptr, 0, raster_group(kPairM, k, es), chain_kb<DT>()};
    // (A stream-K tail -- the last partial wave's tiles spread over all pairs in
    // equal k-block ranges -- measured 15-45% slower than whole tiles at 4096^3
    // and 3072 x 4096 x 2048 on B200, and was dropped.)
    if (splits > 1) {
        rc = ensure_workspace(dev, (size_t)tiles * splits * 2 * kBM * kPairN * sizeof(float), (size_t)tiles * 2, &sk);
        if (rc != TRB_OK) return rc;
    }
    const long units = tiles * splits;
    const int grid_workers = (int)std::max<long>(1, std::min<long>(units, workers));
    // The pair kernel's cluster shape (2 CTAs) is compiled in (__cluster_dims__).
    rc = launch_ex(gemm_tcgen05_pair_kernel<DT, KB>, grid_workers * 2, pair_smem_bytes<DT>(), 1, stream, tmA, tmB, tmC, c,
                   m, n, k, out_scale, sk);
    if (rc != TRB_OK) return rc;
    TRB_CUDA(cudaGetLastError());
    if (info) {
        *info = LaunchInfo{};
        info->grid = grid_workers * 2;
        info->block = kThreads;
        info->splits = splits;
        info->pair = 1;
        info->tile_n = kPairN;
    }
    return TRB_OK;
}

// ------------------------------------------------------------------ float32 via 3xTF32
// A float32 GEMM on the tf32 tensor cores, accurate to ~fp32: each input
// x = hi + lo with hi = tf32(x), lo = tf32(x - hi) (x - hi is exact in fp32),
// and C = A_lo*B_hi + A_hi*B_lo + A_hi*B_hi (the dropped A_lo*B_lo term is
// ~2^-22 of a product).  The three products are ONE tf32 GEMM over K' = 3K:
//   A' = [A_lo | A_hi | A_hi]  (M x 3K),   B' = [B_hi ; B_lo ; B_hi]  (3K x N)
// (B^T storage: rows [B_hi | B_lo | B_hi]).  The small terms come first in K,
// so they accumulate into a small partial sum.  A' and B' live in a per-device
// grow-only buffer of 12 (MK + KN) bytes, built by one split pass per operand
// (the reference's float32 path is an fp32 rocWMMA kernel,
// mfu_gemm_highp.hip.hpp:39-218; its parity tolerance for fp32 is 1e-4).
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t t;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(x));
    return __uint_as_float(t);
}

// parts: bit j set = part j is hi, clear = lo.  `stacked`: parts are stacked
// rows x cols blocks (dst = 3 * rows x cols); otherwise parts are concatenated
// along each row (dst = rows x 3 * cols).  cols % 4 == 0.
__global__ void split3_tf32_kernel(const float4* __restrict__ src, float4* __restrict__ dst, uint64_t rows,
                                   uint64_t cols4, uint32_t parts, int stacked) {
    const uint64_t total = rows * cols4;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const float4 x = src[i];
        float4 hi, lo;
        hi.x = tf32_rna(x.x); lo.x = tf32_rna(x.x - hi.x);
        hi.y = tf32_rna(x.y); lo.y = tf32_rna(x.y - hi.y);
        hi.z = tf32_rna(x.z); lo.z = tf32_rna(x.z - hi.z);
        hi.w = tf32_rna(x.w); lo.w = tf32_rna(x.w - hi.w);
        const uint64_t r = i / cols4, c = i - r * cols4;
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const uint64_t o = stacked ? (uint64_t)part * total + i : r * 3 * cols4 + (uint64_t)part * cols4 + c;
            dst[o] = (parts >> part) & 1u ? hi : lo;
        }
    }
}

struct Fp32x3Workspace {
    float* buf = nullptr;
    size_t bytes = 0;
    std::mutex mu;
};
static Fp32x3Workspace g_fp32x3[64];

static int launch_fp32x3(int m, int n, int k, const void* a, const void* b, void* c, int splits, int cta_pair,
                         int tile_n, int b_kmajor, cudaStream_t stream, LaunchInfo* info) {
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) {
        set_error("device id %d out of range", dev);
        return TRB_ERR_ARGS;
    }
    const size_t a3 = (size_t)m * k * 3, b3 = (size_t)k * n * 3;
    Fp32x3Workspace& w = g_fp32x3[dev];
    std::lock_guard<std::mutex> lock(w.mu);
    if (w.bytes < (a3 + b3) * sizeof(float)) {
        if (w.buf) cudaFree(w.buf);
        w.buf = nullptr;
        w.bytes = 0;
        TRB_CUDA(cudaMalloc(&w.buf, (a3 + b3) * sizeof(float)));
        w.bytes = (a3 + b3) * sizeof(float);
    }
    float* ap = w.buf;
    float* bp = w.buf + a3;  // a3 * 4 bytes is a multiple of 16 (k % 4 == 0)
    const int grid = device_sm_count(dev) * 8;
    constexpr uint32_t kLoHiHi = 0b110, kHiLoHi = 0b101;
    split3_tf32_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4*>(a), reinterpret_cast<float4*>(ap),
                                                 (uint64_t)m, (uint64_t)k / 4, kLoHiHi, 0);
    TRB_CUDA(cudaGetLastError());
    if (b_kmajor)  // B^T rows (N x K) -> N x 3K
        split3_tf32_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4*>(b), reinterpret_cast<float4*>(bp),
                                                     (uint64_t)n, (uint64_t)k / 4, kHiLoHi, 0);
    else  // row-major K x N -> 3K x N
        split3_tf32_kernel<<<grid, 256, 0, stream>>>(static_cast<const float4*>(b), reinterpret_cast<float4*>(bp),
                                                     (uint64_t)k, (uint64_t)n / 4, kHiLoHi, 1);
    TRB_CUDA(cudaGetLastError());
    const int rc = b_kmajor ? launch_typed<TRB_TFLOAT32, true>(m, n, 3 * k, ap, bp, c, 1.0f, splits, cta_pair, tile_n, stream, info)
                            : launch_typed<TRB_TFLOAT32, false>(m, n, 3 * k, ap, bp, c, 1.0f, splits, cta_pair, tile_n, stream,
                                                                info);
    if (info) info->fp32x3 = 1;
    return rc;
}

int launch(int dtype, int m, int n, int k, const void* a, const void* b, void* c, float scale_a, float scale_b,
           int splits, int cta_pair, int b_kmajor, cudaStream_t stream, LaunchInfo* info, int tile_n) {
    if (m <= 0 || n <= 0 || k <= 0 || a == nullptr || b == nullptr || c == nullptr) {
        set_error("trb_gemm_launch: dimensions must be positive and pointers non-null");
        return TRB_ERR_ARGS;
    }
    const size_t es = dtype_size(dtype);
    if (!(dtype == TRB_BFLOAT16 || dtype == TRB_FLOAT16 || dtype == TRB_TFLOAT32 || dtype == TRB_FLOAT8_E4M3FN ||
          dtype == TRB_INT8 || dtype == TRB_FLOAT32 || dtype == TRB_FLOAT64)) {
        set_error("unsupported dtype for native MFU kernel: %s", dtype_name(dtype));
        return TRB_SKIPPED;
    }
    if (dtype == TRB_FLOAT64) return dgemm::launch(m, n, k, a, b, c, b_kmajor, stream, info);
    if (((size_t)k * es) % 16 != 0 || ((size_t)n * es) % 16 != 0) {
        set_error("trb_gemm_launch: k*elem and n*elem must be multiples of 16 bytes (k=%d n=%d elem=%zu)", k, n, es);
        return TRB_ERR_ALIGN;
    }
    if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15u) !=
        0) {
        set_error("trb_gemm_launch: A, B and C must be 16-byte aligned");
        return TRB_ERR_ALIGN;
    }
    if (splits < 0 && splits != -2 && splits != -4 && splits != -8) {
        set_error("trb_gemm_launch: splits must be >= 0, or -2 / -4 / -8 for cluster split-K (got %d)", splits);
        return TRB_ERR_ARGS;
    }
    if (dtype == TRB_FLOAT32) return launch_fp32x3(m, n, k, a, b, c, splits, cta_pair, tile_n, b_kmajor, stream, info);
    if (b_kmajor) {
        switch (dtype) {
            case TRB_BFLOAT16: return launch_typed<TRB_BFLOAT16, true>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
            case TRB_FLOAT16: return launch_typed<TRB_FLOAT16, true>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
            case TRB_TFLOAT32: return launch_typed<TRB_TFLOAT32, true>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
            case TRB_FLOAT8_E4M3FN:
                return launch_typed<TRB_FLOAT8_E4M3FN, true>(m, n, k, a, b, c, scale_a * scale_b, splits, cta_pair,
                                                             tile_n, stream, info);
            default: return launch_typed<TRB_INT8, true>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
        }
    }
    switch (dtype) {
        case TRB_BFLOAT16: return launch_typed<TRB_BFLOAT16, false>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
        case TRB_FLOAT16: return launch_typed<TRB_FLOAT16, false>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
        case TRB_TFLOAT32: return launch_typed<TRB_TFLOAT32, false>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
        case TRB_FLOAT8_E4M3FN:
            return launch_typed<TRB_FLOAT8_E4M3FN, false>(m, n, k, a, b, c, scale_a * scale_b, splits, cta_pair,
                                                          tile_n, stream, info);
        default: return launch_typed<TRB_INT8, false>(m, n, k, a, b, c, 1.0f, splits, cta_pair, tile_n, stream, info);
    }
}

// ------------------------------------------------------------------ no-allocation split-K
// Some callers cannot let a library call cudaMalloc: a host framework whose
// caching allocator has already reserved nearly all of HBM (a library
// cudaMalloc would then fail, or fragment memory the framework manages), or a
// latency-critical path that cannot absorb the device-wide synchronisation
// cudaMalloc / cudaFree may imply.  trb_gemm_launch_noalloc serves them: the
// same single-CTA split-K kernel as trb_gemm_launch, with its scratch (the
// per-tile arrival counters and the fp32 partials) in one fixed-size array in
// the library's device data instead of the grow-only cudaMalloc'd workspace.
// Each GPU that loads the library holds this array until the process exits.
constexpr size_t kNoAllocCounterBytes = 16u << 10;            // 4096 per-tile counters
constexpr size_t kNoAllocPartialBytes = 16u << 20;            // 16 MiB = 128 units of 128 x 256 fp32
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocScratch {
    bool ready = false;
    unsigned int* counters = nullptr;
    float* partials = nullptr;
};
static NoAllocScratch g_noalloc_scratch_ptr[64];
static std::mutex g_noalloc_mu;

// Host code cannot use g_noalloc_scratch's name as a device address (it names
// a host-side shadow); the device address comes from cudaGetSymbolAddress,
// resolved once per device while that device is current and cached for the
// life of the process.  A cudaDeviceReset (or any teardown of the primary
// context) while the library is in use reloads the module and can move the
// array, so the cached address would be stale; the header forbids it, as it
// would also invalidate the library's other per-device state.
static int noalloc_scratch(int dev, NoAllocScratch* out) {
    if (dev < 0 || dev >= 64) {
        set_error("trb_gemm_launch_noalloc: device id %d out of range", dev);
        return TRB_ERR_ARGS;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocScratch& s = g_noalloc_scratch_ptr[dev];
    if (!s.ready) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_error("trb_gemm_launch_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
            return TRB_ERR_CUDA;
        }
        s.counters = static_cast<unsigned int*>(p);
        s.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(p) + kNoAllocCounterBytes);
        s.ready = true;
    }
    *out = s;
    return TRB_OK;
}

template <int DT>
static int launch_noalloc_typed(int m, int n, int k, const void* a, const void* b, void* c, float out_scale,
                                int splits, cudaStream_t stream) {
    using Tr = Traits<DT>;
    constexpr int es = Tr::kEsize;
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    const long tiles = (long)((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
    const int num_kb = (int)(((long)k * es + kBKBytes - 1) / kBKBytes);
    if (splits <= 0) {
        // Automatic: choose_splits' count, cut to what the fixed scratch holds
        // (an automatic request never fails for lack of scratch).
        constexpr long kUnits = (long)(kNoAllocPartialBytes / (kBM * kBN * sizeof(float)));
        splits = choose_splits(tiles, num_kb, sms);
        if (tiles > (long)(kNoAllocCounterBytes / sizeof(unsigned int))) splits = 1;
        splits = (int)std::min<long>(splits, std::max<long>(1, kUnits / std::max<long>(tiles, 1)));
    }
    splits = std::max(1, std::min(splits, num_kb));
    const int kbps = (num_kb + splits - 1) / splits;
    splits = (num_kb + kbps - 1) / kbps;
    const size_t partial_bytes = (size_t)tiles * splits * kBM * kBN * sizeof(float);
    const size_t counter_bytes = (size_t)tiles * sizeof(unsigned int);
    if (splits > 1 && (partial_bytes > kNoAllocPartialBytes || counter_bytes > kNoAllocCounterBytes)) {
        set_error("trb_gemm_launch_noalloc: %dx%dx%d with %d K splits needs %zu bytes of split-K partials and %zu "
                  "bytes of counters; the fixed scratch holds %zu and %zu (at most 128 tile-splits of 128 x 256)",
                  m, n, k, splits, partial_bytes, counter_bytes, kNoAllocPartialBytes, kNoAllocCounterBytes);
        return TRB_ERR_ARGS;
    }
    NoAllocScratch scratch;
    int rc = noalloc_scratch(dev, &scratch);
    if (rc != TRB_OK) return rc;
    CUtensorMap tmA, tmB;
    rc = encode_2d(&tmA, a, es, (uint64_t)k, (uint64_t)m, kBKBytes / es, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TRB_OK) return rc;
    rc = encode_2d(&tmB, b, es, (uint64_t)n, (uint64_t)k, 128 / es, kBKBytes / es, Tr::BLayout::kTmaSwizzle);
    if (rc != TRB_OK) return rc;
    CUtensorMap tmC;
    rc = encode_2d(&tmC, c, out_esize<DT>(), (uint64_t)n, (uint64_t)m, 32, 32,
                   out_esize<DT>() == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TRB_OK) return rc;
    using Cfg = TileCfgFor<DT, 256, 1>;
    TRB_CUDA(cudaFuncSetAttribute(gemm_tcgen05_kernel<DT, false, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)Cfg::kSmem));
    // K rotation and raster as trb_gemm_launch_ex's single-CTA 128 x 256
    // kernel (launch_single), so the two agree bit for bit at equal splits.
    SplitK sk{splits, kbps, nullptr, nullptr, m <= kBM ? 1 : 0, raster_group(kBM, k, es), chain_kb<DT>()};
    if (splits > 1) {
        // The array keeps the previous call's contents: counters must start at zero.
        TRB_CUDA(cudaMemsetAsync(scratch.counters, 0, counter_bytes, stream));
        sk.ws = scratch.partials;
        sk.counters = scratch.counters;
    }
    const long units = tiles * splits;
    const int grid = (int)std::max<long>(1, std::min<long>(units, sms));
    gemm_tcgen05_kernel<DT, false, 256><<<grid, kThreads, Cfg::kSmem, stream>>>(tmA, tmB, tmC, c, m, n, k, out_scale,
                                                                             sk);
    TRB_CUDA(cudaGetLastError());
    return TRB_OK;
}

static int launch_noalloc(int dtype, int m, int n, int k, const void* a, const void* b, void* c, float scale_a,
                          float scale_b, int splits, cudaStream_t stream) {
    if (m <= 0 || n <= 0 || k <= 0 || a == nullptr || b == nullptr || c == nullptr || splits < 0) {
        set_error("trb_gemm_launch_noalloc: dimensions must be positive, pointers non-null, splits >= 0");
        return TRB_ERR_ARGS;
    }
    const size_t es = dtype_size(dtype);
    if (!(dtype == TRB_BFLOAT16 || dtype == TRB_FLOAT16 || dtype == TRB_TFLOAT32 || dtype == TRB_FLOAT8_E4M3FN ||
          dtype == TRB_INT8)) {
        set_error("unsupported dtype for native MFU kernel: %s", dtype_name(dtype));
        return TRB_SKIPPED;
    }
    if (((size_t)k * es) % 16 != 0 || ((size_t)n * es) % 16 != 0 ||
        ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15u)) {
        set_error("trb_gemm_launch_noalloc: k*elem and n*elem must be multiples of 16 bytes and A, B, C 16-byte aligned");
        return TRB_ERR_ALIGN;
    }
    switch (dtype) {
        case TRB_BFLOAT16: return launch_noalloc_typed<TRB_BFLOAT16>(m, n, k, a, b, c, 1.0f, splits, stream);
        case TRB_FLOAT16: return launch_noalloc_typed<TRB_FLOAT16>(m, n, k, a, b, c, 1.0f, splits, stream);
        case TRB_TFLOAT32: return launch_noalloc_typed<TRB_TFLOAT32>(m, n, k, a, b, c, 1.0f, splits, stream);
        case TRB_FLOAT8_E4M3FN:
            return launch_noalloc_typed<TRB_FLOAT8_E4M3FN>(m, n, k, a, b, c, scale_a * scale_b, splits, stream);
        default: return launch_noalloc_typed<TRB_INT8>(m, n, k, a, b, c, 1.0f, splits, stream);
    }
}

// ------------------------------------------------------------------ inputs
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// N(0,1) / sqrt(K) by Box-Muller from a counter hash of (seed, i).
__device__ __forceinline__ float normal_scaled(uint64_t seed, uint64_t i, float inv_sqrt_k) {
    const uint64_t z = mix64(seed * 0xD1B54A32D192ED03ull + i);
    const float u1 = ((float)(z >> 40) + 1.0f) * 0x1p-24f;  // (0, 1]
    const float u2 = (float)((z >> 16) & 0xFFFFFFu) * 0x1p-24f;
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2) * inv_sqrt_k;
}

__global__ void absmax_kernel(uint64_t n, uint64_t seed, float inv_sqrt_k, unsigned int* out_bits) {
    float m = 0.0f;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(normal_scaled(seed, i, inv_sqrt_k)));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));
}

__global__ void fill_gemm_kernel(void* data, int dtype, uint64_t n, uint64_t seed, float inv_sqrt_k,
                                 const unsigned int* absmax_bits) {
    const float inv_scale = absmax_bits ? 448.0f / __uint_as_float(*absmax_bits) : 1.0f;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        switch (dtype) {
            case TRB_BFLOAT16:
                static_cast<__nv_bfloat16*>(data)[i] = __float2bfloat16_rn(normal_scaled(seed, i, inv_sqrt_k));
                break;
            case TRB_FLOAT16:
                static_cast<__half*>(data)[i] = __float2half_rn(normal_scaled(seed, i, inv_sqrt_k));
                break;
            case TRB_FLOAT32: static_cast<float*>(data)[i] = normal_scaled(seed, i, inv_sqrt_k); break;
            case TRB_FLOAT64: static_cast<double*>(data)[i] = (double)normal_scaled(seed, i, inv_sqrt_k); break;
            case TRB_TFLOAT32: {
                uint32_t t;
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(normal_scaled(seed, i, inv_sqrt_k)));
                static_cast<uint32_t*>(data)[i] = t;
                break;
            }
            case TRB_FLOAT8_E4M3FN:
                static_cast<__nv_fp8_storage_t*>(data)[i] =
                    __nv_cvt_float_to_fp8(normal_scaled(seed, i, inv_sqrt_k) * inv_scale, __NV_SATFINITE, __NV_E4M3);
                break;
            case TRB_INT8: {
                const uint64_t z = mix64(seed * 0xD1B54A32D192ED03ull + i);
                static_cast<int8_t*>(data)[i] = (int8_t)((int)(z % 255ull) - 127);
                break;
            }
            default: break;
        }
    }
}

__global__ void round_tf32_kernel(uint32_t* data, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        uint32_t t;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(__uint_as_float(data[i])));
        data[i] = t;
    }
}

// Fills `data` (n elements) in the BASELINE distribution of `dtype`; for e4m3
// returns the per-tensor scale absmax / 448 in *scale_out.  `absmax_scratch`
// is one device word used by the e4m3 absmax reduction.
int fill_operand(void* data, int dtype, uint64_t n, int k, uint64_t seed, unsigned int* absmax_scratch,
                 float* scale_out, cudaStream_t stream) {
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    const int grid = device_sm_count(dev) * 8;
    const float inv_sqrt_k = 1.0f / sqrtf((float)k);
    *scale_out = 1.0f;
    if (dtype == TRB_FLOAT8_E4M3FN) {
        TRB_CUDA(cudaMemsetAsync(absmax_scratch, 0, sizeof(unsigned int), stream));
        absmax_kernel<<<grid, 256, 0, stream>>>(n, seed, inv_sqrt_k, absmax_scratch);
        TRB_CUDA(cudaGetLastError());
        fill_gemm_kernel<<<grid, 256, 0, stream>>>(data, dtype, n, seed, inv_sqrt_k, absmax_scratch);
        TRB_CUDA(cudaGetLastError());
        unsigned int bits = 0;
        TRB_CUDA(cudaMemcpyAsync(&bits, absmax_scratch, sizeof(bits), cudaMemcpyDeviceToHost, stream));
        TRB_CUDA(cudaStreamSynchronize(stream));
        float amax;
        memcpy(&amax, &bits, 4);
        *scale_out = amax / 448.0f;
        return TRB_OK;
    }
    fill_gemm_kernel<<<grid, 256, 0, stream>>>(data, dtype, n, seed, inv_sqrt_k, nullptr);
    TRB_CUDA(cudaGetLastError());
    return TRB_OK;
}

// Bounded-wait self-test: the failure path of every GEMM kernel's waits, made
// to run on purpose without a fault.  Warp 0 holds TMEM (as the GEMM kernels
// do) and its lane 0 waits, with the library's bounded wait and a short limit,
// for the first phase of an mbarrier that nothing ever arrives on; it gives
// up, records kErrSelfTestWait in the module's error word and raises the
// CTA's abort flag.  Warp 1's lane 0 waits on a second such barrier with the
// full kWaitTimeoutNs limit and returns as soon as it sees the abort flag --
// the path by which one stalled role releases the others.  No TMA, MMA or
// other asynchronous operation is in flight; TMEM is freed before exit.
__global__ void __launch_bounds__(64, 1) wait_probe_kernel(uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t never_bar[2];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&never_bar[0]), 1);
        mbar_init(smem_u32(&never_bar[1]), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_slot), 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        if (!mbar_wait(smem_u32(&never_bar[0]), 0, &abort_flag, limit_ns)) {
            atomicCAS(&g_gemm_error, 0, kErrSelfTestWait);
            abort_flag = 1;
        }
    } else if (threadIdx.x == 32) {
        if (!mbar_wait(smem_u32(&never_bar[1]), 0, &abort_flag)) atomicCAS(&g_gemm_error, 0, kErrEpilogueWait);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_slot, 32);
    }
}

int wait_probe(uint64_t limit_ns, cudaStream_t stream) {
    wait_probe_kernel<<<1, 64, 0, stream>>>(limit_ns);
    TRB_CUDA(cudaGetLastError());
    return TRB_OK;
}

int read_error(bool clear) {
    int v = 0;
    TRB_CUDA(cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)));
    if (clear) {
        const int zero = 0;
        TRB_CUDA(cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)));
    }
    return v;
}

}  // namespace gemm
}  // namespace trb

extern "C" int trb_gemm_launch(int dtype, int m, int n, int k, const void* a, const void* b, void* c, float scale_a,
                               float scale_b, void* stream) {
    trb::clear_error();
    return trb::gemm::launch(dtype, m, n, k, a, b, c, scale_a, scale_b, 0, -1, 0, static_cast<cudaStream_t>(stream),
                             nullptr);
}

extern "C" int trb_gemm_launch_ex(int dtype, int m, int n, int k, const void* a, const void* b, void* c, float scale_a,
                                  float scale_b, const trb_gemm_options* options, void* stream) {
    trb::clear_error();
    const trb_gemm_options defaults = {0, -1, TRB_B_ROW_MAJOR, 0};
    const trb_gemm_options& o = options ? *options : defaults;
    if (o.b_layout != TRB_B_ROW_MAJOR && o.b_layout != TRB_B_K_MAJOR) {
        trb::set_error("trb_gemm_launch_ex: unknown b_layout %d", o.b_layout);
        return TRB_ERR_ARGS;
    }
    return trb::gemm::launch(dtype, m, n, k, a, b, c, scale_a, scale_b, o.splits, o.cta_pair,
                             o.b_layout == TRB_B_K_MAJOR, static_cast<cudaStream_t>(stream), nullptr, o.tile_n);
}

extern "C" int trb_round_tf32(void* data, uint64_t count, void* stream) {
    trb::clear_error();
    if (data == nullptr || count == 0) {
        trb::set_error("trb_round_tf32: empty input");
        return TRB_ERR_ARGS;
    }
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    trb::gemm::round_tf32_kernel<<<trb::device_sm_count(dev) * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t*>(data), count);
    TRB_CUDA(cudaGetLastError());
    return TRB_OK;
}

extern "C" int trb_gemm_launch_noalloc(int dtype, int m, int n, int k, const void* a, const void* b, void* c,
                                       float scale_a, float scale_b, int splits, void* stream) {
    trb::clear_error();
    return trb::gemm::launch_noalloc(dtype, m, n, k, a, b, c, scale_a, scale_b, splits,
                                     static_cast<cudaStream_t>(stream));
}
