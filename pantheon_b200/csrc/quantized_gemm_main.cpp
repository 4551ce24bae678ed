// quantized_gemm / llm_decode -- drop-in replacements for Pantheon's
// `quantized_gemm` and `llm_decode` workload binaries, running real quantized
// GEMMs / the W4A16 decode GEMV on the B200.  One source, two binaries: built
// with QG_DECODE_BINARY it is `llm_decode` (default --format w4a16, decode
// banner, also reports tokens/s), otherwise `quantized_gemm` (default int8).
//
// llm_decode's reference (kernels/llm_decode/llm_decode.cpp:59-115) has the
// same argv and flags; its `Throughput:` unit was tokens/s of a KV gather.
// Here the decode step is the weight-only projection, a stream over the
// weights, so `Throughput:` is GB/s (the runner derives MB/s per watt from a
// GB/s row, pantheon.py:3559) and tokens/s (rows x calls / s) is logged on an
// "  -> Tokens/s:" line.
//
// Process contract (kept from the reference):
//   argv   <device> <duration_s> <mem_pct> [--verify] [--inject_error]
//          [--block_size N] [--grid_size N] [--kernel_loops N] [--warmup_iters N]
//          [--sync_mode N]                       (ai_workload_template.h:351-356)
//          new: --format int8|fp8|nvfp4|w4a16, --m/--n/--k N, --seed S, --copies N
//          Unknown flags are ignored, as the reference's parser ignores them.
//   stdout "[PANTHEON] GPU <id>: ..." and "  -> ..." lines (kept in the runner's log),
//          "Throughput: <value> <unit>"          (ai_workload_template.h:377)
//          "Verification: PASS|FAIL (<n> mismatches)" and, per recorded
//          mismatch, an "[SDC FAULT]" line        (mma_virus.cpp:156-173,394-432)
//   exit   0 = ran and (if asked) verified; 1 = verification failed or the
//          workload could not run, reason on stderr (common.h:231-240,444-465).
// One process drives one GPU; the runner starts one per GPU with that GPU
// visible as device 0 (pantheon.py:3306-3336).
//
// Host side only: everything on the device goes through the C ABI of
// include/pantheon_qgemm.h.
#include "../../include/pantheon_qgemm.h"

#include <nvtx3/nvToolsExt.h>   // header-only; a no-op unless a profiler is attached

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>

namespace {

// NVTX ranges around the run's phases ("qg:fill", "qg:golden", "qg:warmup",
// "qg:timed", "qg:verify"), so a profiler can be pointed at the timed
// launches alone (ncu --nvtx --nvtx-include "qg:timed/").
struct Phase {
    explicit Phase(const char* name) { nvtxRangePushA(name); }
    ~Phase() { nvtxRangePop(); }
};

#ifdef QG_DECODE_BINARY
constexpr int kDefaultFormat = QG_FMT_W4A16;
constexpr const char* kWorkload = "LLM Decode";
constexpr const char* kFaultTag = "LLM_DECODE";
#else
constexpr int kDefaultFormat = QG_FMT_INT8;
constexpr const char* kWorkload = "Quantized GEMM";
constexpr const char* kFaultTag = "QUANTIZED_GEMM";
#endif

// Launch-knob clamps with the reference's bounds (common.h:248-311).
constexpr int kMaxKernelLoops = 1000000;

struct Options {
    int device = 0, duration = 1, mem_pct = 99;
    bool verify = false, inject = false;
    int kernel_loops = 0;        // GEMMs per timed batch; 0 = size a batch to ~200 ms
    int warmup_iters = 3;
    int format = kDefaultFormat;
    int m = 0, n = 0, k = 0, copies = 0;
    uint64_t seed = 1;
    bool seed_given = false;
};

const char* format_name(int f) {
    switch (f) {
        case QG_FMT_INT8: return "INT8 W8A8";
        case QG_FMT_FP8: return "FP8 e4m3 block-128";
        case QG_FMT_NVFP4: return "NVFP4 e2m1/ue4m3";
        case QG_FMT_W4A16: return "W4A16 group-128";
        default: return "?";
    }
}

int parse_format(const std::string& s) {
    if (s == "int8" || s == "i8") return QG_FMT_INT8;
    if (s == "fp8") return QG_FMT_FP8;
    if (s == "nvfp4" || s == "fp4") return QG_FMT_NVFP4;
    if (s == "w4a16") return QG_FMT_W4A16;
    return -1;
}

int fail(const std::string& why) {
    std::cerr << "[PANTHEON ERROR] " << why << std::endl;
    return 1;
}

int fail_ctx(qg_ctx* ctx, const char* what) {
    char buf[512];
    qg_last_error(ctx, buf, sizeof(buf));
    std::cerr << "[PANTHEON ERROR] " << what << ": " << buf << std::endl;
    if (ctx) qg_destroy(ctx);
    return 1;
}

} // namespace

int main(int argc, char* argv[]) {
    if (argc < 4) return 1;
    Options o;
    o.device = atoi(argv[1]);
    o.duration = atoi(argv[2]);
    o.mem_pct = atoi(argv[3]);
    for (int i = 4; i < argc; ++i) {
        std::string a(argv[i]);
        auto next = [&](void) -> const char* { return (i + 1 < argc) ? argv[++i] : nullptr; };
        if (a == "--verify") o.verify = true;
        else if (a == "--inject_error") o.inject = true;
        else if (a == "--kernel_loops") { if (const char* v = next()) o.kernel_loops = atoi(v); }
        else if (a == "--warmup_iters") { if (const char* v = next()) o.warmup_iters = atoi(v); }
        else if (a == "--block_size" || a == "--grid_size" || a == "--sync_mode") { next(); }
        else if (a == "--format") {
            if (const char* v = next()) {
                o.format = parse_format(v);
                if (o.format < 0) return fail(std::string("unknown --format ") + v);
            }
        }
        else if (a == "--m") { if (const char* v = next()) o.m = atoi(v); }
        else if (a == "--n") { if (const char* v = next()) o.n = atoi(v); }
        else if (a == "--k") { if (const char* v = next()) o.k = atoi(v); }
        else if (a == "--copies") { if (const char* v = next()) o.copies = atoi(v); }
        else if (a == "--seed") { if (const char* v = next()) { o.seed = strtoull(v, nullptr, 10); o.seed_given = true; } }
        // anything else: ignored, as in the reference
    }
    if (o.kernel_loops < 0) {
        std::cerr << "[PANTHEON] Warning: invalid kernel_loops " << o.kernel_loops << "; using auto." << std::endl;
        o.kernel_loops = 0;
    } else if (o.kernel_loops > kMaxKernelLoops) {
        std::cerr << "[PANTHEON] Warning: kernel_loops " << o.kernel_loops << " clamped to " << kMaxKernelLoops << "." << std::endl;
        o.kernel_loops = kMaxKernelLoops;
    }
    if (o.warmup_iters < 0) {
        std::cerr << "[PANTHEON] Warning: invalid warmup_iters " << o.warmup_iters << "; using 0." << std::endl;
        o.warmup_iters = 0;
    }
    if (o.duration < 0) o.duration = 0;
    o.mem_pct = o.mem_pct < 1 ? 1 : (o.mem_pct > 99 ? 99 : o.mem_pct);

    qg_cfg cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.format = o.format;
    cfg.m = o.m; cfg.n = o.n; cfg.k = o.k;
    cfg.out_type = QG_OUT_BF16;
    cfg.seed = o.seed;

    // Working-set sizing from --mem (ai_workload_template.h:359): operand copies
    // beyond the first only matter for the memory-bound GEMV, where they keep
    // each call streaming from HBM instead of L2.
    uint64_t free_b = 0, total_b = 0;
    if (qg_mem_info(o.device, &free_b, &total_b) != QG_OK) return fail_ctx(nullptr, "device query failed");
    const uint64_t budget = free_b / 100 * (uint64_t)o.mem_pct;
    cfg.copies = 1;
    uint64_t one = 0;
    if (qg_required_bytes(&cfg, &one) != QG_OK) return fail_ctx(nullptr, "bad configuration");
    if (o.copies > 0) cfg.copies = o.copies;
    else if (o.format == QG_FMT_W4A16) {
        uint64_t fit = one ? budget / one : 1;
        cfg.copies = (int)(fit < 1 ? 1 : (fit > 8 ? 8 : fit));
    }
    uint64_t need = 0;
    qg_required_bytes(&cfg, &need);
    if (need > free_b) {
        return fail("working set of " + std::to_string(need >> 20) + " MiB does not fit in " +
                    std::to_string(free_b >> 20) + " MiB of free device memory");
    }

    qg_ctx* ctx = nullptr;
    if (qg_create(&ctx, o.device, &cfg) != QG_OK) return fail_ctx(nullptr, "qg_create");
    const double ops = qg_ops_per_launch(ctx);
    const double bytes = qg_bytes_per_launch(ctx);
    const bool bw_metric = (o.format == QG_FMT_W4A16);

    std::cout << "[PANTHEON] GPU " << o.device << ": " << kWorkload << " (" << format_name(o.format)
              << (bw_metric ? " GEMV" : "") << ", sm_100a)" << std::endl;
    std::cout << "  -> Working Set:   " << (need >> 20) << " MiB (" << cfg.copies << " operand cop"
              << (cfg.copies == 1 ? "y" : "ies") << ")" << std::endl;
    std::cout << "  -> Work/Launch:   " << ops / 1e12 << " Tops, " << bytes / 1e6 << " MB" << std::endl;

    {
        Phase ph("qg:fill");
        if (qg_fill(ctx, o.seed) != QG_OK || qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "qg_fill");
    }
    {
        Phase ph("qg:golden");
        if (qg_golden(ctx) != QG_OK || qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "qg_golden");
    }

    // Warm-up, and a timing probe to size the batch (~200 ms per sync, as the
    // reference's vendor GEMM batches: vendor_gemm.h:560-571).
    auto t0 = std::chrono::high_resolution_clock::now();
    if (o.warmup_iters > 0) {
        Phase ph("qg:warmup");
        if (qg_run(ctx, o.warmup_iters, nullptr) != QG_OK || qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "warm-up");
    }
    double per_launch = std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - t0).count() /
                        (o.warmup_iters > 0 ? o.warmup_iters : 1);
    int loops = o.kernel_loops;
    if (loops == 0) {
        double l = per_launch > 0 ? 0.2 / per_launch : 1.0;
        loops = (int)(l < 1 ? 1 : (l > 100000 ? 100000 : l));
    }
    std::cout << "  -> Kernel Loops:  " << loops << std::endl;

    uint64_t mismatches = 0;
    double busy = 0.0;
    uint64_t launches = 0;
    auto start = std::chrono::high_resolution_clock::now();
    do {
        auto b0 = std::chrono::high_resolution_clock::now();
        {
            Phase ph("qg:timed");
            if (qg_run(ctx, loops, nullptr) != QG_OK) return fail_ctx(ctx, "qg_run");
            if (qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "kernel");
        }
        busy += std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - b0).count();
        launches += (uint64_t)loops;
        if (o.verify) {
            // Every batch is checked against the golden result, not only the last.
            uint64_t mm = 0;
            {
                Phase ph("qg:verify");
                if (qg_verify(ctx, &mm) != QG_OK) return fail_ctx(ctx, "qg_verify");
            }
            if (mm) {
                qg_mismatch log[8];
                int nlog = qg_mismatch_log(ctx, log, 8);
                for (int i = 0; i < nlog; ++i) {
                    printf("[SDC FAULT][%s] Output mismatch! Word: %llu | Exp: 0x%08x | Act: 0x%08x | XOR: 0x%08x\n", kFaultTag,
                           (unsigned long long)log[i].index, log[i].expected, log[i].actual, log[i].expected ^ log[i].actual);
                }
                fflush(stdout);
            }
            mismatches += mm;
        }
    } while (std::chrono::duration_cast<std::chrono::seconds>(std::chrono::high_resolution_clock::now() - start).count() <
             o.duration);

    const double rate = busy > 0 ? (bw_metric ? (bytes * (double)launches) / busy / 1e9 : (ops * (double)launches) / busy / 1e12) : 0.0;
    std::cout << "Throughput: " << rate << (bw_metric ? " GB/s" : " TOPS") << std::endl;
    if (bw_metric && busy > 0) {
        const double rows = o.m > 0 ? o.m : 1;   // the GEMV's default decode batch is one row
        std::cout << "  -> Tokens/s:      " << rows * (double)launches / busy << " (" << rows << " row"
                  << (rows == 1 ? "" : "s") << " per call)" << std::endl;
    }

    int exit_code = 0;
    if (o.verify) {
        if (o.inject) {
            std::cout << "[PANTHEON] Warning: SDC Fault Injection is ACTIVE!" << std::endl;
            if (qg_inject(ctx) != QG_OK) return fail_ctx(ctx, "qg_inject");
            uint64_t mm = 0;
            if (qg_verify(ctx, &mm) != QG_OK) return fail_ctx(ctx, "qg_verify");
            qg_mismatch log[8];
            int nlog = qg_mismatch_log(ctx, log, 8);
            for (int i = 0; i < nlog; ++i)
                printf("[SDC FAULT][%s] Output mismatch! Word: %llu | Exp: 0x%08x | Act: 0x%08x | XOR: 0x%08x\n", kFaultTag,
                       (unsigned long long)log[i].index, log[i].expected, log[i].actual, log[i].expected ^ log[i].actual);
            fflush(stdout);
            mismatches += mm;
        }
        std::cout << "  -> Mismatches:    " << mismatches << std::endl;
        std::cout << "Verification: " << (mismatches ? "FAIL" : "PASS") << " (" << mismatches << " mismatches)" << std::endl;
        exit_code = mismatches ? 1 : 0;
    }
    qg_destroy(ctx);
    return exit_code;
}
