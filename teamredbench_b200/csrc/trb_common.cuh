// trb_common.cuh -- shared host/device helpers for libtrb_b200 (sm_100a only).
//
// PTX wrappers for mbarriers, TMA (cp.async.bulk / cp.async.bulk.tensor), and
// the tcgen05 tensor-core / TMEM instructions, plus bounded waits and the
// per-thread error string of the C ABI.  No TMA load here uses
// a cluster-broadcast qualifier: the kernels run replicated on 1..8 GPUs.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/trb_b200.h"

namespace trb {

// ---------------------------------------------------------------- host errors
void set_error(const char* fmt, ...);
void clear_error();
int cuda_fail(cudaError_t err, const char* what);

#define TRB_CUDA(call)                                          \
    do {                                                        \
        cudaError_t trb_e_ = (call);                            \
        if (trb_e_ != cudaSuccess) return ::trb::cuda_fail(trb_e_, #call); \
    } while (0)

size_t dtype_size(int dtype);
const char* dtype_name(int dtype);
int device_sm_count(int device);

// Internal entry points shared between translation units.
namespace hbm {
struct LaunchShape {
    int grid = 0, block = 0, blocks_per_sm = 0, variant = 0;
    const char* impl = "";
};
int launch(int dtype, int mode, void* dst, const void* src, const void* aux, uint64_t count, double scale,
           int variant, int blocks_per_sm, cudaStream_t stream, LaunchShape* shape);
int fill_uniform(void* data, int dtype, uint64_t n, uint64_t seed, cudaStream_t stream);
int read_error(bool clear);
}  // namespace hbm

namespace gemm {
struct LaunchInfo {
    int grid = 0, block = 0, splits = 1, pair = 0, tile_n = 256;
    int fp32x3 = 0;   // float32 computed as three tf32 products
    int fp64 = 0;     // float64 DMMA kernel
    int swap = 0;     // swapped-operand skinny kernel (C^T = B^T A^T); tile_n = its MMA N
    int cluster = 1;  // > 1: K splits reduced inside a thread-block cluster of that size
};
// splits: 0 = automatic (split-K only for problems that leave SMs idle), >= 1 forced.
// cta_pair: < 0 automatic (pair, or narrow single-CTA tiles when skinny), 0 single-CTA, 2 CTA pair with
// 256 x 512 tiles (16-bit outputs, whole tiles), other > 0 CTA pair.
// b_kmajor: B is stored N x K (K-major) instead of the row-major K x N matrix.
// tile_n: 0 automatic; 64 / 128 / 256 force the single-CTA kernel at that tile
// width; < 0 forces the swapped-operand kernel (m <= 64): -1 with the
// workspace split-K of `splits` (0 = automatic), -2 / -4 / -8 with cluster
// split-K of that size.
int launch(int dtype, int m, int n, int k, const void* a, const void* b, void* c, float scale_a, float scale_b,
           int splits, int cta_pair, int b_kmajor, cudaStream_t stream, LaunchInfo* info, int tile_n = 0);
int fill_operand(void* data, int dtype, uint64_t n, int k, uint64_t seed, unsigned int* absmax_scratch,
                 float* scale_out, cudaStream_t stream);
int read_error(bool clear);
// Bounded-wait self-test kernel (see trb_selftest_bounded_wait).
int wait_probe(uint64_t limit_ns, cudaStream_t stream);
}  // namespace gemm

namespace dgemm {
// float64 C = A * B on the DMMA tensor path (no tcgen05 kind takes fp64); any m, n, k.
int launch(int m, int n, int k, const void* a, const void* b, void* c, int b_kmajor, cudaStream_t stream,
           gemm::LaunchInfo* info);
}  // namespace dgemm

// Bounded-wait budget for every spin inside the kernels (nanoseconds of
// %globaltimer).  A healthy wait lasts microseconds.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

// Device error codes written to a kernel's error word.
enum : int {
    kErrNone = 0,
    kErrProducerWait = 1,
    kErrMmaWait = 2,
    kErrEpilogueWait = 3,
    kErrDrainWait = 4,
    kErrBulkWait = 5,
    kErrSelfTestWait = 6,  // the bounded-wait self-test's deliberate give-up
};

#if defined(__CUDACC__)

// ---------------------------------------------------------------- device PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Suspend-time hint of the potentially blocking try_wait (ns): the waiting
// thread sleeps until the phase completes (it is woken at once) or the hint
// expires.  Without a hint the hardware picks its own window, which measured
// as a fixed ~0.5 us per pipeline step on B200.
constexpr uint32_t kTryWaitHintNs = 1000000u;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kTryWaitHintNs)
        : "memory");
    return ok != 0;
}

// Waits until the phase with the given parity has completed.  Gives up (returns
// false) after limit_ns (kWaitTimeoutNs in every library kernel; the bounded-wait
// self-test passes a few milliseconds), or early once *abort becomes non-zero.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort,
                                          uint64_t limit_ns = kWaitTimeoutNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort != nullptr && *abort) return false;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// 2-D tiled TMA load (no multicast) of the box at element coordinates (x, y).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// 2-D tiled TMA store of a shared-memory box to global element coordinates
// (x, y); completion is tracked by this thread's bulk async-groups
// (bulk_commit / bulk_wait_read / bulk_wait_all below).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 1-D bulk copy global -> shared (no multicast); bytes % 16 == 0, both 16-B aligned.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// 1-D bulk copy shared -> global, tracked by bulk async-groups of this thread.
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N of this thread's bulk groups may still be reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every bulk group of this thread has completed (its writes are performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy / tcgen05) reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ANDs a predicate over the participating threads, so
// that every participant takes the same branch afterwards.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %3, 0;\n\t"
        "barrier.cta.red.and.pred po, %1, %2, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(threads), "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

// ---- tcgen05 (5th-gen tensor cores, TMEM accumulators), cta_group::1 ----
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive once on `bar` when all prior tcgen05 async ops of this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], one instruction per kind.
#define TRB_DEFINE_MMA(NAME, KIND)                                                                         \
    __device__ __forceinline__ void NAME(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, \
                                         uint32_t accumulate) {                                           \
        asm volatile(                                                                                      \
            "{\n\t.reg .pred p;\n\t"                                                                       \
            "setp.ne.b32 p, %4, 0;\n\t"                                                                    \
            "tcgen05.mma.cta_group::1.kind::" KIND " [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),             \
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)                                          \
            : "memory");                                                                                   \
    }
TRB_DEFINE_MMA(mma_f16, "f16")
TRB_DEFINE_MMA(mma_tf32, "tf32")
TRB_DEFINE_MMA(mma_f8f6f4, "f8f6f4")
TRB_DEFINE_MMA(mma_i8, "i8")
#undef TRB_DEFINE_MMA

// ---- CTA pairs (clusters of 2) and tcgen05 cta_group::2 ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync_all, for work that can run between them.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kTryWaitHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (barriers that the peer CTA signals).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, const volatile int* abort) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (abort != nullptr && *abort) return false;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
    }
}
// Programmatic dependent launch.  wait: block until the grids this one
// depends on have completed and their memory is visible (a no-op without a
// programmatic dependency).  launch_dependents: allow the next grid in the
// stream to be scheduled (its own wait still orders its memory accesses).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Asynchronous 16-byte store into another CTA's shared memory; its bytes
// complete on `cluster_bar`, an mbarrier in the same destination CTA.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, uint4 v, uint32_t cluster_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     cluster_addr),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(cluster_bar)
                 : "memory");
}

// The pair's even CTA (rank 0) owns the barriers that both CTAs' TMA loads
// complete on; clearing bit 24 of a shared::cluster address selects it.
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;

// 2-D tiled TMA load whose completion is signalled on a barrier of either CTA
// of the pair (no multicast: each CTA loads only its own operand halves).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive on `bar` (same offset) in every CTA of `mask` when this thread's
// prior cta_group::2 tcgen05 ops complete.
__device__ __forceinline__ void tc_commit_pair_multicast(uint32_t bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                     "r"(bar),
                 "h"(mask)
                 : "memory");
}
#define TRB_DEFINE_MMA_PAIR(NAME, KIND)                                                                    \
    __device__ __forceinline__ void NAME(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, \
                                         uint32_t accumulate) {                                           \
        asm volatile(                                                                                      \
            "{\n\t.reg .pred p;\n\t"                                                                       \
            "setp.ne.b32 p, %4, 0;\n\t"                                                                    \
            "tcgen05.mma.cta_group::2.kind::" KIND " [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),             \
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)                                          \
            : "memory");                                                                                   \
    }
TRB_DEFINE_MMA_PAIR(mma_pair_f16, "f16")
TRB_DEFINE_MMA_PAIR(mma_pair_tf32, "tf32")
TRB_DEFINE_MMA_PAIR(mma_pair_f8f6f4, "f8f6f4")
TRB_DEFINE_MMA_PAIR(mma_pair_i8, "i8")
#undef TRB_DEFINE_MMA_PAIR

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 registers per thread -> 32 lanes x 32 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 16 registers per thread -> 32 lanes x 16 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// 32 lanes x 64 consecutive 32-bit TMEM columns -> 64 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
        "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
        "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
}
// 64 registers per thread -> 32 lanes x 64 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st_32x32b_x64(uint32_t taddr, const uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, "
        "%33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, "
        "%49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};"
        ::"r"(taddr),
          "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
          "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]),
          "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
          "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]),
          "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]),
          "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]),
          "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- streaming global accesses (data set >> L2) ----
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

#endif  // __CUDACC__

}  // namespace trb
