// gemm_fp64.cu -- float64 GEMM C = A * B on the B200's FP64 tensor path.
//
// Replaces mfma_gemm_highp_kernel<double> of the reference's mfu_hipblas
// executable (src/teamredbench/native/kernels/mfu_gemm_highp.hip.hpp:39-218)
// and torch.mm on float64 (src/teamredbench/benchmarks/mfu.py:229-234).  No
// tcgen05 MMA kind takes fp64; the FP64 tensor instruction on sm_100 is the
// warp-level DMMA, mma.sync.aligned.m8n8k4.row.col.f64 (256 FMAs per warp
// instruction; the same 64 FP64 FMAs per SM per clock as the CUDA cores, but
// one instruction and one operand fetch per 8 FMAs per lane).
//  * 256 threads per CTA compute a 128 x 128 tile; 8 warps in a 2 (M) x 4 (N)
//    grid, each warp 64 x 32 = 8 x 4 DMMA tiles, 64 fp64 accumulators per lane;
//  * K advances 32 at a time through a 3-stage cp.async ring (216 KiB; 16-byte
//    copies when the rows are 16-byte multiples and the pointers aligned, else
//    8-byte).  One CTA barrier per 32 K instead of per 16 measured 32.6 against
//    31.6 TFLOP/s at 8192^3;
//    out-of-range elements are zero-filled by the copy (src-size 0), and
//    out-of-range outputs are not stored, so any M, N, K works;
//  * A and B^T tiles are stored [row][32 + 4] doubles, row-major B tiles
//    [k][128 + 8]: the padding puts the 8 x 4 fragment of a warp's load in the
//    minimum two shared-memory wavefronts;
//  * either B layout: row-major K x N, or B^T stored N x K (K-major).
#include <algorithm>

#include "trb_common.cuh"

namespace trb {
namespace dgemm {

constexpr int kTile = 128;
constexpr int kBK = 32;
constexpr int kThreads = 256;
constexpr int kStages = 3;
constexpr int kKPad = kBK + 4;      // doubles per row of a k-contiguous tile
constexpr int kNPad = kTile + 8;    // doubles per k-row of an n-contiguous tile
constexpr int kTileKc = kTile * kKPad;  // k-contiguous tile, doubles
constexpr int kTileNc = kBK * kNPad;    // n-contiguous tile, doubles
constexpr int kStageDoubles = kTileKc + (kTileKc > kTileNc ? kTileKc : kTileNc);
constexpr size_t kSmemBytes = (size_t)kStages * kStageDoubles * sizeof(double);

__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, bool in_range, int bytes) {
    const int src_size = in_range ? bytes : 0;
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_size) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_size) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void dmma(double& d0, double& d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// Copy a 128-row x kBK-double tile of a k-contiguous matrix (rows of length K,
// leading dimension K) into smem [row][kKPad].  V = doubles per copy (2 or 1).
template <int V>
__device__ __forceinline__ void load_kc(uint32_t dst, const double* __restrict__ src, int row0, int rows, int k0,
                                        int K) {
    constexpr int kChunks = kTile * kBK / V;
#pragma unroll
    for (int i = 0; i < kChunks / kThreads; ++i) {
        const int c = threadIdx.x + i * kThreads;
        const int r = c / (kBK / V);
        const int kk = (c % (kBK / V)) * V;
        const int gr = row0 + r, gk = k0 + kk;
        const bool ok = gr < rows && gk < K;
        const double* p = ok ? src + (size_t)gr * K + gk : src;
        cp_async(dst + (uint32_t)((r * kKPad + kk) * 8), p, ok, V * 8);
    }
}

// Copy a kBK-k-row x 128-column tile of a row-major K x N matrix into smem [k][kNPad].
template <int V>
__device__ __forceinline__ void load_nc(uint32_t dst, const double* __restrict__ src, int k0, int K, int n0, int N) {
    constexpr int kChunks = kBK * kTile / V;
#pragma unroll
    for (int i = 0; i < kChunks / kThreads; ++i) {
        const int c = threadIdx.x + i * kThreads;
        const int kk = c / (kTile / V);
        const int nn = (c % (kTile / V)) * V;
        const int gk = k0 + kk, gn = n0 + nn;
        const bool ok = gk < K && gn < N;
        const double* p = ok ? src + (size_t)gk * N + gn : src;
        cp_async(dst + (uint32_t)((kk * kNPad + nn) * 8), p, ok, V * 8);
    }
}

template <bool KB, int V>
__global__ void __launch_bounds__(kThreads, 1)
    dgemm_kernel(const double* __restrict__ A, const double* __restrict__ B, double* __restrict__ C, int M, int N,
                 int K) {
    extern __shared__ __align__(16) double smem[];
    const uint32_t s0 = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;           // DMMA fragment coordinates
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
    const int ktiles = (K + kBK - 1) / kBK;

    auto stage_a = [&](int s) { return s0 + (uint32_t)(s * kStageDoubles * 8); };
    auto stage_b = [&](int s) { return s0 + (uint32_t)((s * kStageDoubles + kTileKc) * 8); };
    auto issue = [&](int kt) {
        const int s = kt % kStages;
        load_kc<V>(stage_a(s), A, m0, M, kt * kBK, K);
        if constexpr (KB)
            load_kc<V>(stage_b(s), B, n0, N, kt * kBK, K);
        else
            load_nc<V>(stage_b(s), B, kt * kBK, K, n0, N);
    };

    double acc[8][4][2];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < ktiles) issue(s);
        cp_async_commit();
    }
    for (int kt = 0; kt < ktiles; ++kt) {
        cp_async_wait<kStages - 2>();
        __syncthreads();  // tile kt landed for every thread; tile kt-1's slot is free
        if (kt + kStages - 1 < ktiles) issue(kt + kStages - 1);
        cp_async_commit();
        const double* sa = smem + (kt % kStages) * kStageDoubles;
        const double* sb = sa + kTileKc;
#pragma unroll
        for (int k4 = 0; k4 < kBK; k4 += 4) {
            double af[8], bf[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) af[i] = sa[(wm + i * 8 + g) * kKPad + k4 + t];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if constexpr (KB)
                    bf[j] = sb[(wn + j * 8 + g) * kKPad + k4 + t];
                else
                    bf[j] = sb[(k4 + t) * kNPad + wn + j * 8 + g];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma(acc[i][j][0], acc[i][j][1], af[i], bf[j]);
        }
    }
    cp_async_wait<0>();

    // D fragment: lane holds C[g][2t], C[g][2t + 1] of each 8 x 8 tile.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int gm = m0 + wm + i * 8 + g;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + wn + j * 8 + 2 * t;
            double* out = C + (size_t)gm * N + gn;
            if (V == 2 && gn + 1 < N) {
                *reinterpret_cast<double2*>(out) = make_double2(acc[i][j][0], acc[i][j][1]);
            } else {
                if (gn < N) out[0] = acc[i][j][0];
                if (gn + 1 < N) out[1] = acc[i][j][1];
            }
        }
    }
}

template <bool KB, int V>
static int launch_kernel(dim3 grid, const double* A, const double* B, double* C, int m, int n, int k,
                         cudaStream_t stream) {
    static bool attr_set[64] = {};
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attr_set[dev]) {
        TRB_CUDA(cudaFuncSetAttribute(dgemm_kernel<KB, V>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kSmemBytes));
        attr_set[dev] = true;
    }
    dgemm_kernel<KB, V><<<grid, kThreads, kSmemBytes, stream>>>(A, B, C, m, n, k);
    return TRB_OK;
}

int launch(int m, int n, int k, const void* a, const void* b, void* c, int b_kmajor, cudaStream_t stream,
           gemm::LaunchInfo* info) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                           reinterpret_cast<uintptr_t>(c);
    if ((addr & 7u) != 0) {
        set_error("trb_gemm_launch: float64 operands must be 8-byte aligned");
        return TRB_ERR_ALIGN;
    }
    const dim3 grid((n + kTile - 1) / kTile, (m + kTile - 1) / kTile);
    if (grid.y > 65535u) {
        set_error("trb_gemm_launch: float64 m too large (%d)", m);
        return TRB_ERR_ARGS;
    }
    // 16-byte copies and stores need 16-byte aligned pointers and even row lengths
    // (K for A and B^T, N for row-major B and for C).
    const bool vec2 = (addr & 15u) == 0 && k % 2 == 0 && n % 2 == 0;
    const double* A = static_cast<const double*>(a);
    const double* B = static_cast<const double*>(b);
    double* C = static_cast<double*>(c);
    int rc;
    if (b_kmajor)
        rc = vec2 ? launch_kernel<true, 2>(grid, A, B, C, m, n, k, stream)
                  : launch_kernel<true, 1>(grid, A, B, C, m, n, k, stream);
    else
        rc = vec2 ? launch_kernel<false, 2>(grid, A, B, C, m, n, k, stream)
                  : launch_kernel<false, 1>(grid, A, B, C, m, n, k, stream);
    if (rc != TRB_OK) return rc;
    TRB_CUDA(cudaGetLastError());
    if (info) {
        *info = gemm::LaunchInfo{};
        info->grid = (int)(grid.x * grid.y);
        info->block = kThreads;
        info->fp64 = 1;
        info->tile_n = kTile;
    }
    return TRB_OK;
}

}  // namespace dgemm
}  // namespace trb
