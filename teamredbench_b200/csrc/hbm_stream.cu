// hbm_stream.cu -- STREAM copy / scale / triad kernels for B200 (sm_100a).
//
// Replaces scale_kernel<T> / triad_kernel<T> and the hipMemcpyAsync copy of the
// reference's hbm_hip executable (src/teamredbench/native/kernels/
// hbm_bandwidth.hip.cpp:188-321, 373-386).  Arithmetic follows the reference's
// torch path (src/teamredbench/benchmarks/hbm.py:29-39) bit for bit; see
// include/trb_b200.h (trb_hbm_launch) for the per-dtype formulas.
//
// Two device paths:
//  * VEC  -- grid-stride loop; each thread keeps U independent 16-byte loads per
//            array in flight (ld.global.nc.L1::no_allocate) and writes with
//            st.global.cs (evict-first): the data set is far larger than L2.
//  * BULK -- TMA bulk copies: one producer thread streams 16 KiB chunks
//            global->shared with cp.async.bulk into a 4-stage mbarrier ring,
//            256 threads apply the op in shared memory, one thread writes the
//            chunk back with a bulk store.  Copy mode stores the landed chunk
//            directly (HBM -> SMEM -> HBM with no register traffic).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "trb_common.cuh"

namespace trb {
namespace hbm {

__device__ int g_hbm_error;  // device error word of this module (bounded waits)

// ------------------------------------------------------------------ element ops
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ uint32_t bf_pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 h2_unpack(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}
__device__ __forceinline__ uint32_t h2_pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Each op transforms one 16-byte vector (vec) or one element (elem, on the
// element's raw bits) -- the scalar form serves the ragged tail and unaligned
// pointers.  alpha_f is float(scale) (f32 and the scale of bf16/f16), or
// float(dt(scale)) for the bf16/f16 triad; alpha_d is the double scale.
struct OpCopy {
    static constexpr bool kAux = false;
    static constexpr bool kIsCopy = true;
    __device__ __forceinline__ uint4 vec(uint4 s, uint4) const { return s; }
    template <class T>
    __device__ __forceinline__ T elem(T s, T) const { return s; }
};

struct OpScaleF32 {
    static constexpr bool kAux = false, kIsCopy = false;
    float a;
    __device__ __forceinline__ uint4 vec(uint4 s, uint4) const {
        return make_uint4(__float_as_uint(__fmul_rn(__uint_as_float(s.x), a)),
                          __float_as_uint(__fmul_rn(__uint_as_float(s.y), a)),
                          __float_as_uint(__fmul_rn(__uint_as_float(s.z), a)),
                          __float_as_uint(__fmul_rn(__uint_as_float(s.w), a)));
    }
    __device__ __forceinline__ uint32_t elem(uint32_t s, uint32_t) const {
        return __float_as_uint(__fmul_rn(__uint_as_float(s), a));
    }
};

struct OpTriadF32 {
    static constexpr bool kAux = true, kIsCopy = false;
    float a;
    __device__ __forceinline__ uint32_t one(uint32_t b, uint32_t c) const {
        return __float_as_uint(__fmaf_rn(a, __uint_as_float(c), __uint_as_float(b)));
    }
    __device__ __forceinline__ uint4 vec(uint4 b, uint4 c) const {
        return make_uint4(one(b.x, c.x), one(b.y, c.y), one(b.z, c.z), one(b.w, c.w));
    }
    __device__ __forceinline__ uint32_t elem(uint32_t b, uint32_t c) const { return one(b, c); }
};

struct OpScaleF64 {
    static constexpr bool kAux = false, kIsCopy = false;
    double a;
    __device__ __forceinline__ unsigned long long one(unsigned long long s) const {
        return __double_as_longlong(__dmul_rn(__longlong_as_double(s), a));
    }
    __device__ __forceinline__ uint4 vec(uint4 s, uint4) const {
        unsigned long long lo = one((unsigned long long)s.x | ((unsigned long long)s.y << 32));
        unsigned long long hi = one((unsigned long long)s.z | ((unsigned long long)s.w << 32));
        return make_uint4((uint32_t)lo, (uint32_t)(lo >> 32), (uint32_t)hi, (uint32_t)(hi >> 32));
    }
    __device__ __forceinline__ unsigned long long elem(unsigned long long s, unsigned long long) const {
        return one(s);
    }
};

struct OpTriadF64 {
    static constexpr bool kAux = true, kIsCopy = false;
    double a;
    __device__ __forceinline__ unsigned long long one(unsigned long long b, unsigned long long c) const {
        return __double_as_longlong(__fma_rn(a, __longlong_as_double(c), __longlong_as_double(b)));
    }
    __device__ __forceinline__ uint4 vec(uint4 b, uint4 c) const {
        unsigned long long lo = one((unsigned long long)b.x | ((unsigned long long)b.y << 32),
                                    (unsigned long long)c.x | ((unsigned long long)c.y << 32));
        unsigned long long hi = one((unsigned long long)b.z | ((unsigned long long)b.w << 32),
                                    (unsigned long long)c.z | ((unsigned long long)c.w << 32));
        return make_uint4((uint32_t)lo, (uint32_t)(lo >> 32), (uint32_t)hi, (uint32_t)(hi >> 32));
    }
    __device__ __forceinline__ unsigned long long elem(unsigned long long b, unsigned long long c) const {
        return one(b, c);
    }
};

struct OpScaleBF16 {
    static constexpr bool kAux = false, kIsCopy = false;
    float a;
    __device__ __forceinline__ uint32_t two(uint32_t s) const {
        return bf_pack(__fmul_rn(bf_lo(s), a), __fmul_rn(bf_hi(s), a));
    }
    __device__ __forceinline__ uint4 vec(uint4 s, uint4) const {
        return make_uint4(two(s.x), two(s.y), two(s.z), two(s.w));
    }
    __device__ __forceinline__ uint16_t elem(uint16_t s, uint16_t) const {
        return (uint16_t)two((uint32_t)s);
    }
};

struct OpTriadBF16 {
    static constexpr bool kAux = true, kIsCopy = false;
    float a;  // float(bf16(scale))
    __device__ __forceinline__ uint32_t two(uint32_t b, uint32_t c) const {
        return bf_pack(__fmaf_rn(a, bf_lo(c), bf_lo(b)), __fmaf_rn(a, bf_hi(c), bf_hi(b)));
    }
    __device__ __forceinline__ uint4 vec(uint4 b, uint4 c) const {
        return make_uint4(two(b.x, c.x), two(b.y, c.y), two(b.z, c.z), two(b.w, c.w));
    }
    __device__ __forceinline__ uint16_t elem(uint16_t b, uint16_t c) const {
        return (uint16_t)two((uint32_t)b, (uint32_t)c);
    }
};

struct OpScaleF16 {
    static constexpr bool kAux = false, kIsCopy = false;
    float a;
    __device__ __forceinline__ uint32_t two(uint32_t s) const {
        float2 f = h2_unpack(s);
        return h2_pack(__fmul_rn(f.x, a), __fmul_rn(f.y, a));
    }
    __device__ __forceinline__ uint4 vec(uint4 s, uint4) const {
        return make_uint4(two(s.x), two(s.y), two(s.z), two(s.w));
    }
    __device__ __forceinline__ uint16_t elem(uint16_t s, uint16_t) const {
        return (uint16_t)two((uint32_t)s);
    }
};

struct OpTriadF16 {
    static constexpr bool kAux = true, kIsCopy = false;
    float a;  // float(f16(scale))
    __device__ __forceinline__ uint32_t two(uint32_t b, uint32_t c) const {
        float2 fb = h2_unpack(b), fc = h2_unpack(c);
        return h2_pack(__fmaf_rn(a, fc.x, fb.x), __fmaf_rn(a, fc.y, fb.y));
    }
    __device__ __forceinline__ uint4 vec(uint4 b, uint4 c) const {
        return make_uint4(two(b.x, c.x), two(b.y, c.y), two(b.z, c.z), two(b.w, c.w));
    }
    __device__ __forceinline__ uint16_t elem(uint16_t b, uint16_t c) const {
        return (uint16_t)two((uint32_t)b, (uint32_t)c);
    }
};

// ------------------------------------------------------------------ VEC path
// 1024 threads per CTA, two CTAs per SM (64 warps; <= 32 registers per thread,
// hence the launch bound).  Vectors per array per thread: 2 for triad (two
// input streams), 4 for copy / scale (one input stream, so the same bytes in
// flight per SM).  Measured on B200 for the fp32 triad against 512 x 4,
// 256/512 x 8, 1024 x 4/8, 768 x 4 and 256-bit (v8) loads: 7117 GB/s vs
// 7049 for 512 x 4 and <= 7080 for the others.
constexpr int kVecThreads = 1024;
template <class Op>
constexpr int vec_unroll() { return Op::kAux ? 2 : 4; }

// Elements [tail_begin, n) that do not fill a 16-byte vector, done by the last CTA.
template <class Op, class T>
__device__ __forceinline__ void tail_elems(T* dst, const T* src, const T* aux, uint64_t tail_begin, uint64_t n,
                                           const Op& op) {
    for (uint64_t i = tail_begin + threadIdx.x; i < n; i += blockDim.x)
        dst[i] = op.elem(src[i], Op::kAux ? aux[i] : T(0));
}

template <class Op, class T, int U>
__global__ void __launch_bounds__(kVecThreads, 2048 / kVecThreads) hbm_vec_kernel(T* __restrict__ dst, const T* __restrict__ src,
                                                              const T* __restrict__ aux, uint64_t n, Op op) {
    constexpr uint64_t kPerVec = 16 / sizeof(T);
    const uint64_t nvec = n / kPerVec;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    const uint4* a4 = reinterpret_cast<const uint4*>(aux);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    const uint64_t tile = (uint64_t)blockDim.x * U;
    for (uint64_t base = (uint64_t)blockIdx.x * tile; base < nvec; base += (uint64_t)gridDim.x * tile) {
        const uint64_t i0 = base + threadIdx.x;
        if (base + tile <= nvec) {
            uint4 s[U], a[U];
#pragma unroll
            for (int u = 0; u < U; ++u) s[u] = ld_stream(s4 + i0 + (uint64_t)u * blockDim.x);
            if constexpr (Op::kAux) {
#pragma unroll
                for (int u = 0; u < U; ++u) a[u] = ld_stream(a4 + i0 + (uint64_t)u * blockDim.x);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) st_stream(d4 + i0 + (uint64_t)u * blockDim.x, op.vec(s[u], a[u]));
        } else {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t i = i0 + (uint64_t)u * blockDim.x;
                if (i < nvec) {
                    uint4 sv = ld_stream(s4 + i);
                    uint4 av = sv;
                    if constexpr (Op::kAux) av = ld_stream(a4 + i);
                    st_stream(d4 + i, op.vec(sv, av));
                }
            }
        }
    }
    if (blockIdx.x == gridDim.x - 1) tail_elems(dst, src, aux, nvec * kPerVec, n, op);
}

// Unaligned pointers: plain per-element grid-stride loop.
template <class Op, class T>
__global__ void __launch_bounds__(256) hbm_scalar_kernel(T* dst, const T* src, const T* aux, uint64_t n, Op op) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dst[i] = op.elem(src[i], Op::kAux ? aux[i] : T(0));
}

// ------------------------------------------------------------------ BULK path
constexpr int kBulkStages = 4;
constexpr uint32_t kBulkChunk = 16384;  // bytes per array per stage
constexpr int kBulkCompute = 256;        // compute threads (warps 1..8); warp 0 = producer
constexpr int kBulkThreads = kBulkCompute + 32;

template <class Op>
constexpr size_t bulk_smem_bytes() {
    // input ring, aux ring (triad), output ring (scale/triad; copy stores the input ring)
    return (size_t)kBulkStages * kBulkChunk * (1 + (Op::kAux ? 1 : 0) + (Op::kIsCopy ? 0 : 1));
}

template <class Op, class T>
__global__ void __launch_bounds__(kBulkThreads, 1) hbm_bulk_kernel(T* __restrict__ dst, const T* __restrict__ src,
                                                                   const T* __restrict__ aux, uint64_t n, Op op) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kBulkStages];
    __shared__ __align__(8) uint64_t empty_bar[kBulkStages];
    __shared__ volatile int abort_flag;

    uint8_t* in_buf = smem;
    uint8_t* aux_buf = in_buf + (size_t)kBulkStages * kBulkChunk;
    uint8_t* out_buf = Op::kIsCopy ? in_buf : aux_buf + (Op::kAux ? (size_t)kBulkStages * kBulkChunk : 0);

    const uint64_t total_bytes = (n * sizeof(T)) & ~uint64_t(15);  // bulk-copyable prefix
    const uint64_t nchunks = (total_bytes + kBulkChunk - 1) / kBulkChunk;
    const uint64_t mine = nchunks > blockIdx.x ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kBulkStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const uint8_t* srcb = reinterpret_cast<const uint8_t*>(src);
    const uint8_t* auxb = reinterpret_cast<const uint8_t*>(aux);
    uint8_t* dstb = reinterpret_cast<uint8_t*>(dst);

    if (threadIdx.x < 32) {
        // ---- producer: one elected lane streams chunks into the ring
        if (threadIdx.x == 0) {
            uint64_t issued = 0;
            for (uint64_t j = 0; j < mine; ++j) {
                const int s = (int)(j % kBulkStages);
                const uint32_t ph = (uint32_t)((j / kBulkStages) & 1);
                if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u, &abort_flag)) {
                    atomicCAS(&g_hbm_error, 0, kErrBulkWait);
                    abort_flag = 1;
                    break;
                }
                const uint64_t c = blockIdx.x + j * gridDim.x;
                const uint64_t off = c * kBulkChunk;
                const uint32_t bytes = (uint32_t)(total_bytes - off < kBulkChunk ? total_bytes - off : kBulkChunk);
                mbar_arrive_expect_tx(smem_u32(&full_bar[s]), bytes * (Op::kAux ? 2u : 1u));
                bulk_load(smem_u32(in_buf + (size_t)s * kBulkChunk), srcb + off, bytes, smem_u32(&full_bar[s]));
                if constexpr (Op::kAux)
                    bulk_load(smem_u32(aux_buf + (size_t)s * kBulkChunk), auxb + off, bytes, smem_u32(&full_bar[s]));
                issued = j + 1;
            }
            // Drain: every issued load must land before the CTA may exit.
            const uint64_t first = issued > (uint64_t)kBulkStages ? issued - kBulkStages : 0;
            for (uint64_t j = first; j < issued; ++j) {
                const int s = (int)(j % kBulkStages);
                const uint32_t ph = (uint32_t)((j / kBulkStages) & 1);
                if (!mbar_wait(smem_u32(&full_bar[s]), ph, nullptr)) atomicCAS(&g_hbm_error, 0, kErrDrainWait);
            }
        }
    } else {
        // ---- compute warps
        const int t = threadIdx.x - 32;
        const bool storer = (t == 0);
        // Copy mode needs no compute: only the storer walks the ring.
        const uint64_t my_chunks = (Op::kIsCopy && !storer) ? 0 : mine;
        for (uint64_t j = 0; j < my_chunks; ++j) {
            const int s = (int)(j % kBulkStages);
            const uint32_t ph = (uint32_t)((j / kBulkStages) & 1);
            bool ok = mbar_wait(smem_u32(&full_bar[s]), ph, &abort_flag);
            if (!ok) {
                atomicCAS(&g_hbm_error, 0, kErrBulkWait);
                abort_flag = 1;
            }
            const uint64_t c = blockIdx.x + j * gridDim.x;
            const uint64_t off = c * kBulkChunk;
            const uint32_t bytes = (uint32_t)(total_bytes - off < kBulkChunk ? total_bytes - off : kBulkChunk);
            if constexpr (Op::kIsCopy) {
                if (!ok) break;
                bulk_store(dstb + off, smem_u32(in_buf + (size_t)s * kBulkChunk), bytes);
                bulk_commit();
                // Free the stage of the previous chunk once its store has read smem.
                bulk_wait_read<1>();
                if (j >= 1) mbar_arrive(smem_u32(&empty_bar[(j - 1) % kBulkStages]));
            } else {
                // The output slot s was last used by chunk j - S: its store must have read it.
                if (storer) bulk_wait_read<kBulkStages - 1>();
                // Uniform decision: every compute thread continues, or all stop together.
                if (!named_barrier_and(1, kBulkCompute, ok && !abort_flag)) break;
                const uint4* in4 = reinterpret_cast<const uint4*>(in_buf + (size_t)s * kBulkChunk);
                const uint4* ax4 = reinterpret_cast<const uint4*>(aux_buf + (size_t)s * kBulkChunk);
                uint4* out4 = reinterpret_cast<uint4*>(out_buf + (size_t)s * kBulkChunk);
                for (uint32_t v = t; v < bytes / 16; v += kBulkCompute) {
                    uint4 sv = in4[v];
                    uint4 av = sv;
                    if constexpr (Op::kAux) av = ax4[v];
                    out4[v] = op.vec(sv, av);
                }
                fence_proxy_async_smem();
                named_barrier(1, kBulkCompute);
                if (storer) {
                    bulk_store(dstb + off, smem_u32(out_buf + (size_t)s * kBulkChunk), bytes);
                    bulk_commit();
                    mbar_arrive(smem_u32(&empty_bar[s]));
                }
            }
        }
        if (storer) bulk_wait_all();
        // Ragged element tail (< 16 bytes), by the last CTA's compute threads.
        if (blockIdx.x == gridDim.x - 1) {
            const uint64_t tail_begin = total_bytes / sizeof(T);
            for (uint64_t i = tail_begin + t; i < n; i += kBulkCompute)
                dst[i] = op.elem(src[i], Op::kAux ? aux[i] : T(0));
        }
    }
}

// ------------------------------------------------------------------ host side
template <class Op, class T>
static int launch_op(int variant, T* dst, const T* src, const T* aux, uint64_t n, Op op, int blocks_per_sm,
                     cudaStream_t stream, LaunchShape* shape) {
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    if (sms <= 0) return TRB_ERR_CUDA;
    const bool aligned = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                           (Op::kAux ? reinterpret_cast<uintptr_t>(aux) : 0)) & 15u) == 0;
    if (!aligned) {
        const int grid = sms * 8;
        hbm_scalar_kernel<Op, T><<<grid, 256, 0, stream>>>(dst, src, aux, n, op);
        TRB_CUDA(cudaGetLastError());
        if (shape) *shape = {grid, 256, 8, TRB_HBM_VEC, "scalar_unaligned"};
        return TRB_OK;
    }
    if (variant == TRB_HBM_BULK) {
        constexpr size_t smem = bulk_smem_bytes<Op>();
        static bool attr_set[64] = {};
        if (dev < 64 && !attr_set[dev]) {
            TRB_CUDA(cudaFuncSetAttribute(hbm_bulk_kernel<Op, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
            attr_set[dev] = true;
        }
        const int bps = blocks_per_sm > 0 ? blocks_per_sm : 1;
        const uint64_t chunks = ((n * sizeof(T)) / kBulkChunk) + 1;
        const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * bps, chunks));
        hbm_bulk_kernel<Op, T><<<grid, kBulkThreads, smem, stream>>>(dst, src, aux, n, op);
        TRB_CUDA(cudaGetLastError());
        if (shape) *shape = {grid, kBulkThreads, bps, TRB_HBM_BULK, "tma_bulk_ring"};
        return TRB_OK;
    }
    // Default: one 16-byte-vector tile (kVecThreads * kVecUnroll vectors per
    // array) per CTA over the whole array -- the hardware block scheduler then
    // balances the stream across SMs dynamically, which measured faster on
    // B200 than any persistent grid-stride size (copy 6.92, triad 7.00 TB/s vs
    // <= 6.70 TB/s at 64 CTAs/SM).  blocks_per_sm > 0 caps the grid at
    // sms * blocks_per_sm (grid-stride), the reference's --blocks-per-cu knob.
    constexpr int kVecUnroll = vec_unroll<Op>();
    const uint64_t tiles = (n * sizeof(T) / 16 + (uint64_t)kVecThreads * kVecUnroll - 1) /
                           ((uint64_t)kVecThreads * kVecUnroll);
    const uint64_t cap = blocks_per_sm > 0 ? (uint64_t)sms * blocks_per_sm : tiles;
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>({cap, tiles, (uint64_t)INT32_MAX}));
    const int bps = blocks_per_sm > 0 ? blocks_per_sm : (int)((grid + sms - 1) / sms);
    hbm_vec_kernel<Op, T, kVecUnroll><<<grid, kVecThreads, 0, stream>>>(dst, src, aux, n, op);
    TRB_CUDA(cudaGetLastError());
    if (shape) *shape = {grid, kVecThreads, bps, TRB_HBM_VEC, "vec128_stream"};
    return TRB_OK;
}

static float host_round_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

static float host_round_f16(float f) { return __half2float(__float2half_rn(f)); }

// Resolves the tuned default for AUTO.
static int resolve_variant(int dtype, int mode, int variant) {
    (void)dtype;
    (void)mode;
    if (variant == TRB_HBM_AUTO) return TRB_HBM_VEC;
    return variant;
}

int launch(int dtype, int mode, void* dst, const void* src, const void* aux, uint64_t count, double scale,
           int variant, int blocks_per_sm, cudaStream_t stream, LaunchShape* shape) {
    if (count == 0 || dst == nullptr || src == nullptr) {
        set_error("trb_hbm_launch: empty count or null pointer");
        return TRB_ERR_ARGS;
    }
    if (mode == TRB_TRIAD && aux == nullptr) {
        set_error("trb_hbm_launch: triad needs aux");
        return TRB_ERR_ARGS;
    }
    if (mode < TRB_COPY || mode > TRB_TRIAD) {
        set_error("trb_hbm_launch: unknown mode %d", mode);
        return TRB_ERR_ARGS;
    }
    variant = resolve_variant(dtype, mode, variant);
    if (variant == TRB_HBM_MEMCPY) {
        if (mode != TRB_COPY) {
            set_error("unsupported variant memcpy for mode %d", mode);
            return TRB_SKIPPED;
        }
        const size_t es = dtype_size(dtype);
        if (es == 0) {
            set_error("unsupported dtype %d", dtype);
            return TRB_SKIPPED;
        }
        TRB_CUDA(cudaMemcpyAsync(dst, src, count * es, cudaMemcpyDeviceToDevice, stream));
        if (shape) *shape = {0, 0, 0, TRB_HBM_MEMCPY, "cudaMemcpyAsync_d2d"};
        return TRB_OK;
    }
    if (variant != TRB_HBM_VEC && variant != TRB_HBM_BULK) {
        set_error("unknown hbm variant %d", variant);
        return TRB_ERR_ARGS;
    }
    const float af = (float)scale;
    switch (dtype) {
    case TRB_FLOAT32: {
        auto* d = static_cast<uint32_t*>(dst);
        auto* s = static_cast<const uint32_t*>(src);
        auto* a = static_cast<const uint32_t*>(aux);
        if (mode == TRB_COPY) return launch_op(variant, d, s, a, count, OpCopy{}, blocks_per_sm, stream, shape);
        if (mode == TRB_SCALE) return launch_op(variant, d, s, a, count, OpScaleF32{af}, blocks_per_sm, stream, shape);
        return launch_op(variant, d, s, a, count, OpTriadF32{af}, blocks_per_sm, stream, shape);
    }
    case TRB_FLOAT64: {
        auto* d = static_cast<unsigned long long*>(dst);
        auto* s = static_cast<const unsigned long long*>(src);
        auto* a = static_cast<const unsigned long long*>(aux);
        if (mode == TRB_COPY) return launch_op(variant, d, s, a, count, OpCopy{}, blocks_per_sm, stream, shape);
        if (mode == TRB_SCALE)
            return launch_op(variant, d, s, a, count, OpScaleF64{scale}, blocks_per_sm, stream, shape);
        return launch_op(variant, d, s, a, count, OpTriadF64{scale}, blocks_per_sm, stream, shape);
    }
    case TRB_BFLOAT16: {
        auto* d = static_cast<uint16_t*>(dst);
        auto* s = static_cast<const uint16_t*>(src);
        auto* a = static_cast<const uint16_t*>(aux);
        if (mode == TRB_COPY) return launch_op(variant, d, s, a, count, OpCopy{}, blocks_per_sm, stream, shape);
        if (mode == TRB_SCALE)
            return launch_op(variant, d, s, a, count, OpScaleBF16{af}, blocks_per_sm, stream, shape);
        return launch_op(variant, d, s, a, count, OpTriadBF16{host_round_bf16(af)}, blocks_per_sm, stream, shape);
    }
    case TRB_FLOAT16: {
        auto* d = static_cast<uint16_t*>(dst);
        auto* s = static_cast<const uint16_t*>(src);
        auto* a = static_cast<const uint16_t*>(aux);
        if (mode == TRB_COPY) return launch_op(variant, d, s, a, count, OpCopy{}, blocks_per_sm, stream, shape);
        if (mode == TRB_SCALE)
            return launch_op(variant, d, s, a, count, OpScaleF16{af}, blocks_per_sm, stream, shape);
        return launch_op(variant, d, s, a, count, OpTriadF16{host_round_f16(af)}, blocks_per_sm, stream, shape);
    }
    case TRB_INT8: {
        if (mode != TRB_COPY) {
            set_error("unsupported dtype or mode for native HBM kernel: int8/%s", mode == TRB_SCALE ? "scale" : "triad");
            return TRB_SKIPPED;
        }
        auto* d = static_cast<uint8_t*>(dst);
        auto* s = static_cast<const uint8_t*>(src);
        return launch_op(variant, d, s, s, count, OpCopy{}, blocks_per_sm, stream, shape);
    }
    default:
        set_error("unsupported dtype or mode for native HBM kernel: %s", dtype_name(dtype));
        return TRB_SKIPPED;
    }
}

// ------------------------------------------------------------------ seeded fill
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// uniform[-1, 1) from a counter-based hash of (seed, index)
__global__ void fill_uniform_kernel(void* data, int dtype, uint64_t n, uint64_t seed) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t z = splitmix64(seed * 0xD1B54A32D192ED03ull + i);
        const float f = (float)(z >> 40) * 0x1p-23f - 1.0f;
        switch (dtype) {
            case TRB_FLOAT32: static_cast<float*>(data)[i] = f; break;
            case TRB_FLOAT64: static_cast<double*>(data)[i] = (double)(z >> 11) * 0x1p-52 - 1.0; break;
            case TRB_BFLOAT16: static_cast<__nv_bfloat16*>(data)[i] = __float2bfloat16_rn(f); break;
            case TRB_FLOAT16: static_cast<__half*>(data)[i] = __float2half_rn(f); break;
            case TRB_INT8: static_cast<int8_t*>(data)[i] = (int8_t)(z >> 56); break;
            default: break;
        }
    }
}

int fill_uniform(void* data, int dtype, uint64_t n, uint64_t seed, cudaStream_t stream) {
    int dev = 0;
    TRB_CUDA(cudaGetDevice(&dev));
    fill_uniform_kernel<<<device_sm_count(dev) * 8, 256, 0, stream>>>(data, dtype, n, seed);
    TRB_CUDA(cudaGetLastError());
    return TRB_OK;
}

int read_error(bool clear) {
    int v = 0;
    TRB_CUDA(cudaMemcpyFromSymbol(&v, g_hbm_error, sizeof(int)));
    if (clear) {
        const int zero = 0;
        TRB_CUDA(cudaMemcpyToSymbol(g_hbm_error, &zero, sizeof(int)));
    }
    return v;
}

}  // namespace hbm
}  // namespace trb

extern "C" int trb_hbm_launch(int dtype, int mode, void* dst, const void* src, const void* aux, uint64_t count,
                              double scale, int variant, int blocks_per_sm, void* stream) {
    trb::clear_error();
    return trb::hbm::launch(dtype, mode, dst, src, aux, count, scale, variant, blocks_per_sm,
                            static_cast<cudaStream_t>(stream), nullptr);
}
