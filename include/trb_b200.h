/*
 * trb_b200.h -- C ABI of the TeamRedBench B200 native backend (libtrb_b200.so).
 *
 * The reference (Fangzhou-Ai/TeamRedBench) reaches its native kernels through a
 * subprocess: the runtime spawns a compiled executable with CLI flags and parses
 * the last stdout line as JSON (src/teamredbench/native/runtime.py:276-291).  This
 * library is the core behind that boundary: the launcher executables trb_hbm /
 * trb_mfu (teamredbench_b200/csrc/trb_native_main.cpp) keep the reference's
 * argv/JSON contract and call trb_hbm_run / trb_gemm_run; in-process callers
 * (ctypes, cgo, JNI ...) call the launch / host entry points directly.
 *
 * Conventions
 *  - Plain C types only; device pointers are void*, streams are void*
 *    (a cudaStream_t; NULL = the legacy default stream).
 *  - Return value: 0 = ok, > 0 = skipped (unsupported dtype / mode / shape; the
 *    reference's {"status": "skipped"} case), < 0 = error.  trb_last_error()
 *    returns a message for the calling thread's most recent non-zero status.
 *  - One call per device at a time per process; different devices may be driven
 *    from different threads.
 *  - Every kernel wait is bounded; a wait that gives up sets the device error
 *    word (trb_device_error) and the call returns TRB_ERR_DEVICE_TIMEOUT.
 */
#ifndef TRB_B200_H_
#define TRB_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRB_ABI_VERSION 1

/* Element types.  Names follow the reference's DTypeSpec names
 * (src/teamredbench/dtypes.py:16-31) plus "tfloat32" for the tf32 GEMM. */
typedef enum trb_dtype {
    TRB_FLOAT32 = 0,
    TRB_BFLOAT16 = 1,
    TRB_FLOAT16 = 2,
    TRB_FLOAT64 = 3,
    TRB_INT8 = 4,
    TRB_FLOAT8_E4M3FN = 5,
    TRB_TFLOAT32 = 6,
    TRB_INT32 = 7
} trb_dtype;

/* STREAM modes of the hbm benchmark (src/teamredbench/benchmarks/hbm.py:18-22). */
typedef enum trb_mode { TRB_COPY = 0, TRB_SCALE = 1, TRB_TRIAD = 2 } trb_mode;

/* HBM kernel variants. */
typedef enum trb_hbm_variant {
    TRB_HBM_AUTO = 0,   /* the tuned default for (dtype, mode) */
    TRB_HBM_VEC = 1,    /* grid-stride, 128-bit vector loads/stores with streaming cache hints */
    TRB_HBM_BULK = 2,   /* TMA bulk (cp.async.bulk) global->smem->global pipeline */
    TRB_HBM_MEMCPY = 3  /* copy mode only: cudaMemcpyAsync device-to-device (library comparison) */
} trb_hbm_variant;

/* Status codes (< 0). */
#define TRB_OK 0
#define TRB_SKIPPED 1
#define TRB_ERR_ARGS (-1)
#define TRB_ERR_CUDA (-2)
#define TRB_ERR_ALIGN (-3)
#define TRB_ERR_DEVICE_TIMEOUT (-4)
#define TRB_ERR_NO_DEVICE (-5)

typedef struct trb_result {
    double elapsed_s;        /* mean device seconds per iteration (CUDA events around the timed loop) */
    double moved_bytes;      /* hbm: algorithmic bytes per iteration (factor * count * element size) */
    double achieved_ops;     /* gemm: 2 * m * n * k per iteration */
    double h2d_bytes;        /* host entry points: bytes copied host->device per call */
    double d2h_bytes;        /* host entry points: bytes copied device->host per call */
    int32_t device_id;
    int32_t sm_count;
    int32_t grid;            /* CTAs launched */
    int32_t block;           /* threads per CTA */
    int32_t blocks_per_sm;
    int32_t variant;         /* trb_hbm_variant actually used (hbm) */
    int32_t device_error;    /* non-zero if a bounded device wait gave up */
    int32_t launches;        /* kernels this library launched inside the timed loop */
    int32_t split_k;         /* gemm: K splits used (1 = none) */
    int32_t reserved;
    char implementation[64]; /* short name of the kernel that ran */
} trb_result;

/* Arguments of one hbm case; mirrors the reference executable's flags
 * --dtype --mode --size-mib --warmup --iterations --device-id --scale
 * [--blocks-per-cu] (src/teamredbench/benchmarks/hbm.py:95-114). */
typedef struct trb_hbm_args {
    int32_t dtype;           /* trb_dtype: FLOAT32, BFLOAT16, FLOAT16, FLOAT64, or INT8 (copy only) */
    int32_t mode;            /* trb_mode */
    int32_t variant;         /* trb_hbm_variant */
    int32_t device_id;
    uint64_t size_bytes;     /* bytes per array; count = max(size_bytes / element size, 1) */
    int32_t warmup;
    int32_t iterations;
    double scale;            /* s in scale (a = s*c) and triad (a = b + s*c) */
    int32_t blocks_per_sm;   /* 0 = tuned default (the reference's --blocks-per-cu) */
    int32_t reserved;
} trb_hbm_args;

/* Arguments of one mfu case; mirrors --dtype --m --n --k --warmup --iterations
 * --device-id (src/teamredbench/benchmarks/mfu.py:107-125). */
/* Storage of the B operand of a GEMM. */
typedef enum trb_b_layout {
    TRB_B_ROW_MAJOR = 0,  /* B is the row-major K x N matrix (an MN-major tensor-core operand) */
    TRB_B_K_MAJOR = 1     /* B is stored transposed: row-major N x K (a K-major operand) */
} trb_b_layout;

typedef struct trb_gemm_args {
    int32_t dtype;           /* BFLOAT16, FLOAT16, TFLOAT32, FLOAT8_E4M3FN, INT8, FLOAT32 or FLOAT64 */
    int32_t m, n, k;
    int32_t warmup;
    int32_t iterations;
    int32_t device_id;
    int32_t b_layout;        /* trb_b_layout of the generated B (the reference packs B K-contiguous, untimed) */
} trb_gemm_args;

/* Kernel choices for trb_gemm_launch_ex. */
typedef struct trb_gemm_options {
    int32_t splits;          /* 0 = automatic split-K; >= 1 forces that many K splits (global workspace);
                                -2 / -4 / -8 = that many splits reduced inside a thread-block cluster */
    int32_t cta_pair;        /* < 0 automatic, 0 = single-CTA 128 x 256 tiles, 2 = CTA pair with 256 x 512 tiles
                                (bf16 / f16 / e4m3, whole tiles), other > 0 = CTA-pair 256 x 256 tiles */
    int32_t b_layout;        /* trb_b_layout */
    int32_t tile_n;          /* 0 = automatic; 64, 128 or 256 = single-CTA kernel with tiles of that width;
                                < 0 = swapped-operand kernel (C^T = B^T A^T, m <= 64) */
} trb_gemm_options;

/* ---- library ------------------------------------------------------------ */

/* Returns TRB_ABI_VERSION. */
int trb_abi_version(void);

/* Message for the calling thread's last non-zero status ("" if none). */
const char* trb_last_error(void);

/* Reads (and, if clear != 0, resets) the device error word of device_id.
 * Returns the word (>= 0) or a negative status. */
int trb_device_error(int device_id, int clear);

/* ---- HBM stream kernels ------------------------------------------------- */

/* Allocate three arrays, fill them with seeded uniform[-1,1) values, run
 * `warmup` untimed and `iterations` timed launches, report mean seconds per
 * launch.  Replaces run_kernel<T> of the reference's hbm_hip executable
 * (src/teamredbench/native/kernels/hbm_bandwidth.hip.cpp:323-426) and its
 * dtype dispatch (:458-480). */
int trb_hbm_run(const trb_hbm_args* args, trb_result* out);

/* One launch over caller-owned device arrays: dst[i] = op(src[i], aux[i]) for
 * i < count.  aux is read only in triad mode.  Arithmetic equals the
 * reference's torch path (hbm.py:29-39 `_run_mode`): copy is a byte copy;
 * scale = dt(float(src) * float(scale)); triad = fma(float(scale), aux, src)
 * for float32, fma(scale, aux, src) for float64, and
 * dt(fma(float(dt(scale)), float(aux), float(src))) for bf16/f16.
 * Pointers must be 16-byte aligned for the vector/bulk paths (unaligned
 * pointers take a scalar path).  Asynchronous on `stream`. */
int trb_hbm_launch(int dtype, int mode, void* dst, const void* src, const void* aux,
                   uint64_t count, double scale, int variant, int blocks_per_sm, void* stream);

/* Same operation over HOST arrays: copies src/aux to the device, runs the
 * kernel, copies dst back, all pipelined in chunks on internal streams; returns
 * after dst is written.  out->elapsed_s is the device-timed duration of the
 * whole call (copies included).  Pinned host memory gives full PCIe rate. */
int trb_hbm_host(int dtype, int mode, void* dst_host, const void* src_host, const void* aux_host,
                 uint64_t count, double scale, int device_id, trb_result* out);

/* ---- dense GEMM (tcgen05 / TMEM / TMA) ---------------------------------- */

/* Allocate A (m x k), B (k x n), C (m x n), fill with seeded values in the
 * BASELINE distributions, time `iterations` launches (after a warm-up they are
 * replayed from a CUDA graph captured once, so host launch work does not
 * enter the device-timed loop).  Replaces
 * run_low_precision_kernel / run_high_precision_kernel of the reference's
 * mfu_hipblas executable (src/teamredbench/native/kernels/mfu_gemm_lowp.hip.hpp:
 * 343-486, mfu_gemm_highp.hip.hpp:228-336) and its dispatch
 * (mfu_gemm.hip.cpp:4-25). */
int trb_gemm_run(const trb_gemm_args* args, trb_result* out);

/* One launch: C = A * B over caller-owned device arrays, all row-major:
 * A m x k, B k x n, C m x n.  Accumulate in fp32 (int32 for int8).  Output
 * element type: bf16 for bf16 and e4m3 inputs, f16 for f16, f32 for tf32 and
 * float32, f64 for float64, int32 for int8.  e4m3 results are multiplied by
 * scale_a * scale_b before rounding; other dtypes ignore the scales.  tf32
 * uses the upper 19 bits of each f32 input.  float32 runs on the tf32 tensor
 * cores as three products (x = hi + lo, C = A_lo B_hi + A_hi B_lo + A_hi B_hi;
 * one split pass per operand into a library workspace of 12 (mk + kn) bytes);
 * float64 runs on the DMMA tensor path (mma.sync m8n8k4 f64; no tcgen05 kind
 * takes fp64) and needs only 8-byte aligned pointers.  Others require k * elem % 16 == 0,
 * n * elem % 16 == 0 and 16-byte aligned pointers (TMA); any m, n, k > 0
 * otherwise.  Replaces
 * the reference's torch.mm(a, b, out=out) (src/teamredbench/benchmarks/mfu.py:
 * 229-234) and the native mfma_gemm_*_kernel launches. */
int trb_gemm_launch(int dtype, int m, int n, int k, const void* a, const void* b, void* c,
                    float scale_a, float scale_b, void* stream);

/* trb_gemm_launch with explicit kernel choices (options may be NULL: all automatic).
 *  splits:   >= 1 forces that many K splits (clamped to the number of 128-byte
 *            K blocks).  Splits > 1 use the library's per-device split-K
 *            workspace (fp32 partials and per-tile counters; the last CTA of a
 *            tile sums the partials in split order, so results are
 *            deterministic).  Automatic mode splits only problems whose output
 *            tiles leave more than half of the tile workers idle (e.g. the
 *            skinny M = 16 / 128 shapes).
 *  cta_pair: the CTA-pair kernel (tcgen05.mma.cta_group::2, 256 x 256 tiles)
 *            or the single-CTA kernel (128 x 256 tiles); automatic = the pair,
 *            except for skinny problems: M <= 64 takes the swapped-operand
 *            kernel (C^T = B^T A^T: 128 columns of C per tile, the rows of A as
 *            the MMA's N = 16, 32 or 64), and M <= 128 with few tiles takes
 *            narrow single-CTA tiles (128 x 64; 128 x 128 for 8-bit row-major B).
 *            cta_pair = 2 runs the CTA pair with 256 x 512 tiles (one A load
 *            per k-block feeds two MMAs: 25% fewer L2 -> SM bytes per FLOP) for
 *            bf16, f16 and e4m3 inputs without split-K; its results are
 *            bit-identical to the 256 x 256 pair's.
 *  b_layout: TRB_B_K_MAJOR reads b as B^T (row-major N x K).
 *  tile_n:   0 automatic; 64 / 128 / 256 force the single-CTA kernel with that
 *            tile width (8-bit row-major B: >= 128); < 0 forces the
 *            swapped-operand kernel (m <= 64).  Explicit cta_pair >= 0 also
 *            turns the automatic swapped choice off.
 *  splits < 0: cluster split-K -- the K splits of a tile run as one
 *            thread-block cluster (2, 4 or 8 CTAs, one tile each, every split
 *            owning >= 1 k-block) and are reduced through distributed shared
 *            memory in split order (bit-identical to the workspace split-K
 *            with the same count).  Swapped-operand or 128 x 256 single-CTA
 *            kernel.  Automatic for skinny problems whose tiles leave more
 *            than half of the SMs idle.
 * No reference counterpart: the reference's native GEMM has one tile shape
 * and no split-K (mfu_gemm_lowp.hip.hpp:423-431). */
int trb_gemm_launch_ex(int dtype, int m, int n, int k, const void* a, const void* b, void* c,
                       float scale_a, float scale_b, const trb_gemm_options* options, void* stream);

/* The split-K GEMM of trb_gemm_launch (single-CTA kernel, row-major B) for
 * callers that cannot let a library allocate device memory -- e.g. a host
 * framework whose caching allocator already holds nearly all of HBM, or a
 * latency-critical path that cannot absorb the synchronisation cudaMalloc /
 * cudaFree may imply.  It calls no cudaMalloc, cudaFree or allocating library
 * routine: its scratch (per-tile counters and fp32 partials) is one fixed
 * array in the library's device data, 16 KiB + 16 MiB, which every GPU that
 * loads the library holds until the process exits.
 *  - Limit: at most 128 tile-splits of 128 x 256 (e.g. M <= 128 with
 *    N * splits <= 32768) and 4096 output tiles; an explicit split count
 *    beyond that returns TRB_ERR_ARGS with the sizes in trb_last_error().
 *    splits = 0 takes the split count trb_gemm_launch_ex picks for the
 *    single-CTA 128 x 256 kernel (splits = 0, cta_pair = 0), lowered to what
 *    the array holds, so it never fails for lack of scratch (1 = no scratch
 *    used).  It does not run trb_gemm_launch's automatic kernel choice
 *    (CTA pair, cluster split-K, swapped operands).
 *  - The first call on a device resolves the array's device address
 *    (cudaGetSymbolAddress) with that device current and caches it; make that
 *    first call before any stream capture.  Do not cudaDeviceReset a device
 *    while the library is in use: the module reloads and the cached address
 *    (like the library's other per-device state) goes stale.
 *  - All calls share the one array and it keeps the last call's contents
 *    (the counters are cleared by every call); calls that overlap on the GPU
 *    (other streams, other threads) race.
 * No counterpart in the reference: its GEMM executables own all their memory. */
int trb_gemm_launch_noalloc(int dtype, int m, int n, int k, const void* a, const void* b, void* c,
                            float scale_a, float scale_b, int splits, void* stream);

/* Same GEMM over HOST arrays (copies in and out inside the call). */
int trb_gemm_host(int dtype, int m, int n, int k, const void* a_host, const void* b_host, void* c_host,
                  float scale_a, float scale_b, int device_id, trb_result* out);

/* Round f32 values in place on the device to tf32 (round to nearest, ties
 * away from zero; cvt.rna.tf32.f32).  Used to prepare tf32 GEMM inputs. */
int trb_round_tf32(void* data, uint64_t count, void* stream);

/* Self-test of the device-side failure detector: launches one small kernel
 * whose wait on an mbarrier that nothing arrives on gives up after limit_us
 * microseconds (1 .. 1e6) -- the same bounded wait, error word and CTA abort
 * flag every GEMM kernel uses, with a short limit instead of 2 s -- while a
 * second waiter, on the full limit, leaves as soon as it sees the abort flag.
 * Returns TRB_ERR_DEVICE_TIMEOUT with out->device_error = 6 (and
 * out->elapsed_s near limit_us) when the detector works; TRB_OK would mean
 * the wait did not give up.  No fault, trap or hang is involved, and the
 * context stays usable: the next launch runs normally.  Clears the error
 * words before and after.  No counterpart in the reference, whose native
 * kernels have no bounded waits and whose runner has no timeout
 * (src/teamredbench/native/runtime.py:281-287). */
int trb_selftest_bounded_wait(uint32_t limit_us, int device_id, trb_result* out);

#ifdef __cplusplus
}
#endif

#endif /* TRB_B200_H_ */
