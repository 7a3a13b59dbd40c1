// trb_native_main.cpp -- the reference's native-executable contract on top of
// libtrb_b200.so.  Built twice: -DTRB_BENCH_HBM -> trb_hbm, -DTRB_BENCH_MFU -> trb_mfu.
//
// Contract (src/teamredbench/native/runtime.py:249-291, docs/extending.md):
//   trb_hbm --dtype D --mode M --size-mib S --warmup W --iterations I --device-id G --scale X
//           [--blocks-per-cu B] [--variant auto|vec|bulk|memcpy]
//   trb_mfu --dtype D --m M --n N --k K --warmup W --iterations I --device-id G [--blocks-per-cu B]
//           [--b-layout auto|k_major|row_major]
//   The reference's native GEMM packs B into the layout its kernel reads best,
//   outside the timed loop (mfu_gemm_lowp.hip.hpp:396-409).  `auto` (default)
//   does the same for this library: B row-major for one row of output tiles
//   (m <= 128, the HBM-bound skinny kernels: bf16 M=16 / 128 at N = K = 8192
//   measured 8% / 5% faster than K-major), K-major otherwise (square shapes
//   within 0.5% either way; tf32 4.5% faster K-major).
// The last stdout line is one JSON object: {"status":"ok","raw_metrics":{...},"metadata":{...}},
// or {"status":"skipped","error":"..."} with exit status 0 for unsupported
// input and failures, as the reference executables do
// (src/teamredbench/native/kernels/hbm_bandwidth.hip.cpp:440-479).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/trb_b200.h"

namespace {

std::string json_escape(const char* s) {
    std::string out;
    for (; s && *s; ++s) {
        if (*s == '"' || *s == '\\') out += '\\';
        if (*s == '\n') {
            out += ' ';
            continue;
        }
        out += *s;
    }
    return out;
}

int emit_skipped(const char* error) {
    std::printf("{\"status\":\"skipped\",\"error\":\"%s\"}\n", json_escape(error).c_str());
    std::fflush(stdout);
    return 0;
}

int parse_dtype(const std::string& s) {
    if (s == "float32") return TRB_FLOAT32;
    if (s == "bfloat16") return TRB_BFLOAT16;
    if (s == "float16") return TRB_FLOAT16;
    if (s == "float64") return TRB_FLOAT64;
    if (s == "int8") return TRB_INT8;
    if (s == "float8_e4m3fn") return TRB_FLOAT8_E4M3FN;
    if (s == "tfloat32") return TRB_TFLOAT32;
    return -1;
}

bool parse_int(const char* s, long long* out) {
    char* end = nullptr;
    *out = std::strtoll(s, &end, 10);
    return end && *end == '\0' && end != s;
}

void print_common_metadata(const trb_result& r) {
    std::printf("\"implementation\":\"%s\",\"backend_library\":\"libtrb_b200\",\"device_id\":%d,\"sm_count\":%d,"
                "\"grid\":%d,\"threads_per_block\":%d,\"device_error\":%d",
                json_escape(r.implementation).c_str(), r.device_id, r.sm_count, r.grid, r.block, r.device_error);
}

}  // namespace

int main(int argc, char** argv) {
    std::string dtype = "float32";
    long long warmup = 10, iterations = 50, device_id = 0, blocks_per_cu = 0;
#if defined(TRB_BENCH_HBM)
    std::string mode = "copy", variant = "auto";
    long long size_mib = 1024;
    double scale = 1.0;
#else
    long long m = 4096, n = 4096, k = 4096;
    std::string b_layout = "auto";
#endif
    for (int i = 1; i < argc; ++i) {
        const std::string key = argv[i];
        if (i + 1 >= argc) return emit_skipped(("missing value for argument " + key).c_str());
        const char* value = argv[++i];
        long long iv = 0;
        bool ok = true;
        if (key == "--dtype") dtype = value;
        else if (key == "--warmup") ok = parse_int(value, &warmup);
        else if (key == "--iterations") ok = parse_int(value, &iterations);
        else if (key == "--device-id") ok = parse_int(value, &device_id);
        else if (key == "--blocks-per-cu") ok = parse_int(value, &blocks_per_cu);
#if defined(TRB_BENCH_HBM)
        else if (key == "--mode") mode = value;
        else if (key == "--size-mib") ok = parse_int(value, &size_mib);
        else if (key == "--scale") {
            char* end = nullptr;
            scale = std::strtod(value, &end);
            ok = end && *end == '\0' && end != value;
        } else if (key == "--variant") variant = value;
#else
        else if (key == "--m") ok = parse_int(value, &m);
        else if (key == "--n") ok = parse_int(value, &n);
        else if (key == "--k") ok = parse_int(value, &k);
        else if (key == "--b-layout") b_layout = value;
#endif
        else return emit_skipped(("unknown argument " + key).c_str());
        if (!ok) return emit_skipped(("invalid value for argument " + key).c_str());
        (void)iv;
    }
    if (warmup < 0 || iterations < 0) return emit_skipped("warmup and iterations must be non-negative");
    if (blocks_per_cu < 0) return emit_skipped("blocks-per-cu must be non-negative");
    const int dt = parse_dtype(dtype);
    trb_result r;
    std::memset(&r, 0, sizeof(r));

#if defined(TRB_BENCH_HBM)
    int md = mode == "copy" ? TRB_COPY : mode == "scale" ? TRB_SCALE : mode == "triad" ? TRB_TRIAD : -1;
    int var = variant == "auto" ? TRB_HBM_AUTO : variant == "vec" ? TRB_HBM_VEC : variant == "bulk" ? TRB_HBM_BULK
              : variant == "memcpy" ? TRB_HBM_MEMCPY : -1;
    if (dt < 0 || md < 0 || var < 0 || size_mib <= 0) {
        std::string msg = "unsupported dtype or mode for native HBM kernel: " + dtype + "/" + mode;
        if (var < 0) msg = "unknown --variant " + variant;
        if (size_mib <= 0) msg = "size-mib must be positive";
        return emit_skipped(msg.c_str());
    }
    trb_hbm_args a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dt;
    a.mode = md;
    a.variant = var;
    a.device_id = (int)device_id;
    a.size_bytes = (uint64_t)size_mib * 1024ull * 1024ull;
    a.warmup = (int)warmup;
    a.iterations = (int)iterations;
    a.scale = scale;
    a.blocks_per_sm = (int)blocks_per_cu;
    const int rc = trb_hbm_run(&a, &r);
    if (rc != TRB_OK) return emit_skipped(trb_last_error());
    std::printf("{\"status\":\"ok\",\"raw_metrics\":{\"elapsed_s\":%.9e,\"moved_bytes\":%.0f},\"metadata\":{",
                r.elapsed_s, r.moved_bytes);
    print_common_metadata(r);
    std::printf(",\"blocks_per_cu\":%d,\"variant\":\"%s\"}}\n", r.blocks_per_sm,
                r.variant == TRB_HBM_BULK ? "bulk" : r.variant == TRB_HBM_MEMCPY ? "memcpy" : "vec");
#else
    if (dt < 0) return emit_skipped(("unsupported dtype for native MFU kernel: " + dtype).c_str());
    if (m <= 0 || n <= 0 || k <= 0) return emit_skipped("matrix dimensions must be positive");
    trb_gemm_args a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dt;
    a.m = (int)m;
    a.n = (int)n;
    a.k = (int)k;
    a.warmup = (int)warmup;
    a.iterations = (int)iterations;
    a.device_id = (int)device_id;
    if (b_layout == "auto") b_layout = (m <= 128 && dt != TRB_TFLOAT32) ? "row_major" : "k_major";
    if (b_layout != "k_major" && b_layout != "row_major") return emit_skipped(("unknown --b-layout " + b_layout).c_str());
    a.b_layout = b_layout == "k_major" ? TRB_B_K_MAJOR : TRB_B_ROW_MAJOR;
    const int rc = trb_gemm_run(&a, &r);
    if (rc != TRB_OK) return emit_skipped(trb_last_error());
    std::printf("{\"status\":\"ok\",\"raw_metrics\":{\"elapsed_s\":%.9e,\"achieved_ops\":%.0f},\"metadata\":{",
                r.elapsed_s, r.achieved_ops);
    print_common_metadata(r);
    std::printf(",\"k_block_bytes\":128,\"split_k\":%d,\"b_layout\":\"%s\"}}\n", r.split_k, b_layout.c_str());
#endif
    std::fflush(stdout);
    return 0;
}
