// gemm_fp64.cu -- float64 GEMM C = A * B on B200 CUDA cores.
//
// Replaces mfma_gemm_highp_kernel<double> of the reference's mfu_hipblas
// executable (src/teamredbench/native/kernels/mfu_gemm_highp.hip.hpp:39-218)
// and torch.mm on float64 (src/teamredbench/benchmarks/mfu.py:229-234).  No
// tcgen05 MMA kind takes fp64, so this is a register-tiled FMA kernel:
//  * 256 threads per CTA compute a 128 x 128 tile, each thread an 8 x 8 block
//    held as two 4 x 4 quadrants (rows ty*4 and 64 + ty*4, cols tx*4 and
//    64 + tx*4) so that shared-memory fragment reads are contiguous;
//  * K advances 8 at a time through a double-buffered shared-memory tile
//    (A stored transposed, k-major), the next tile prefetched into registers
//    while the current one is consumed;
//  * any M, N, K and either B layout (row-major K x N, or B^T stored N x K);
//    out-of-range elements load as 0 and out-of-range outputs are not stored.
// Accumulation is plain fp64 FMA in k order.
#include <algorithm>

#include "trb_common.cuh"

namespace trb {
namespace dgemm {

constexpr int kTile = 128;
constexpr int kBK = 8;
constexpr int kThreads = 256;

template <bool KB>
__global__ void __launch_bounds__(kThreads, 1)
    dgemm_kernel(const double* __restrict__ A, const double* __restrict__ B, double* __restrict__ C, int M, int N,
                 int K) {
    __shared__ __align__(16) double As[2][kBK][kTile];  // A^T tile: [k][m]
    __shared__ __align__(16) double Bs[2][kBK][kTile];  // B tile:   [k][n]
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;

    // global -> register staging: each thread moves 4 A and 4 B elements per K step
    // A: row (tid >> 1), k (tid & 1) * 4 .. +4
    const int a_r = tid >> 1, a_k = (tid & 1) * 4;
    // B (row-major): k (tid >> 5), n (tid & 31) * 4 .. +4 ; B^T: row n (tid >> 1), k (tid & 1) * 4 .. +4
    const int b_k = KB ? (tid & 1) * 4 : tid >> 5;
    const int b_n = KB ? tid >> 1 : (tid & 31) * 4;
    double ra[4], rb[4];

    auto load_tile = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int gm = m0 + a_r, gk = k0 + a_k + i;
            ra[i] = (gm < M && gk < K) ? A[(size_t)gm * K + gk] : 0.0;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (KB) {
                const int gn = n0 + b_n, gk = k0 + b_k + i;
                rb[i] = (gn < N && gk < K) ? B[(size_t)gn * K + gk] : 0.0;
            } else {
                const int gk = k0 + b_k, gn = n0 + b_n + i;
                rb[i] = (gk < K && gn < N) ? B[(size_t)gk * N + gn] : 0.0;
            }
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 4; ++i) As[buf][a_k + i][a_r] = ra[i];
        if constexpr (KB) {
#pragma unroll
            for (int i = 0; i < 4; ++i) Bs[buf][b_k + i][b_n] = rb[i];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) Bs[buf][b_k][b_n + i] = rb[i];
        }
    };

    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;

    const int ktiles = (K + kBK - 1) / kBK;
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int t = 0; t < ktiles; ++t) {
        const int buf = t & 1;
        if (t + 1 < ktiles) load_tile((t + 1) * kBK);
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            double a[8], b[8];
            const double2* ap = reinterpret_cast<const double2*>(&As[buf][kk][0]);
            const double2* bp = reinterpret_cast<const double2*>(&Bs[buf][kk][0]);
            const double2 a0 = ap[ty * 2], a1 = ap[ty * 2 + 1], a2 = ap[32 + ty * 2], a3 = ap[32 + ty * 2 + 1];
            const double2 b0 = bp[tx * 2], b1 = bp[tx * 2 + 1], b2 = bp[32 + tx * 2], b3 = bp[32 + tx * 2 + 1];
            a[0] = a0.x; a[1] = a0.y; a[2] = a1.x; a[3] = a1.y; a[4] = a2.x; a[5] = a2.y; a[6] = a3.x; a[7] = a3.y;
            b[0] = b0.x; b[1] = b0.y; b[2] = b1.x; b[3] = b1.y; b[4] = b2.x; b[5] = b2.y; b[6] = b3.x; b[7] = b3.y;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < ktiles) {
            store_tile(buf ^ 1);
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (gn < N) C[(size_t)gm * N + gn] = acc[i][j];
        }
    }
}

int launch(int m, int n, int k, const void* a, const void* b, void* c, int b_kmajor, cudaStream_t stream,
           gemm::LaunchInfo* info) {
    if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 7u) != 0) {
        set_error("trb_gemm_launch: float64 operands must be 8-byte aligned");
        return TRB_ERR_ALIGN;
    }
    const dim3 grid((n + kTile - 1) / kTile, (m + kTile - 1) / kTile);
    if (grid.y > 65535u) {
        set_error("trb_gemm_launch: float64 m too large (%d)", m);
        return TRB_ERR_ARGS;
    }
    const double* A = static_cast<const double*>(a);
    const double* B = static_cast<const double*>(b);
    double* C = static_cast<double*>(c);
    if (b_kmajor)
        dgemm_kernel<true><<<grid, kThreads, 0, stream>>>(A, B, C, m, n, k);
    else
        dgemm_kernel<false><<<grid, kThreads, 0, stream>>>(A, B, C, m, n, k);
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
