// quantized_gemm / llm_decode / mma_virus -- drop-in replacements for
// Pantheon's `quantized_gemm`, `llm_decode` and `mma_virus` workload binaries,
// running real quantized GEMMs, the W4A16 decode GEMV, or the dense tensor
// furnace on the B200.  One source, three binaries:
//   default               `quantized_gemm` (default --format int8, TOPS)
//   QG_DECODE_BINARY      `llm_decode` (default --format w4a16, GB/s + tokens/s)
//   QG_MMA_VIRUS_BINARY   `mma_virus` (default --gemm_type bf16, TFLOPS)
//
// llm_decode's reference (kernels/llm_decode/llm_decode.cpp:59-115) has the
// same argv and flags; its `Throughput:` unit was tokens/s of a KV gather.
// Here the decode step is the weight-only projection, a stream over the
// weights, so `Throughput:` is GB/s (the runner derives MB/s per watt from a
// GB/s row, pantheon.py:3559) and tokens/s (rows x calls / s) is logged on an
// "  -> Tokens/s:" line.
//
// mma_virus's reference (kernels/mma_virus/mma_virus.cpp:181-441) drives a
// cuBLASLt GEMM chosen by the vendor-GEMM flags (kernels/common/vendor_gemm.h:
// 32-55: --gemm_type bf16|fp16|tf32|fp32|fp8|auto, --gemm_size, --gemm_m/n/k,
// --gemm_probe_ms, --gemm_margin, --gemm) and falls back to a WMMA loop.  Here
// the tensor-core formats run on this library's tcgen05 GEMMs and fp32 on its
// CUDA-core GEMM (the reference's fp32 type is an SGEMM too); the WMMA knobs
// (--block_size, --grid_size, --sync_mode, --mma_acc, --mma_groups,
// --mma_reuse, --init_pattern, --kernel_loops) are accepted and ignored, as
// the reference's vendor-GEMM path ignores them.
//
// Process contract (kept from the reference):
//   argv   <device> <duration_s> <mem_pct> [--verify] [--inject_error]
//          [--block_size N] [--grid_size N] [--kernel_loops N] [--warmup_iters N]
//          [--sync_mode N]                       (ai_workload_template.h:351-356)
//          new: --format int8|fp8|nvfp4|w4a16|bf16|fp16|tf32|e4m3|fp32, --m/--n/--k N,
//          --seed S, --copies N
//          Unknown flags are ignored, as the reference's parser ignores them.
//   stdout "[PANTHEON] GPU <id>: ..." and "  -> ..." lines (kept in the runner's log),
//          "Throughput: <value> <unit>"          (ai_workload_template.h:377)
//          "Verification: PASS|FAIL (<n> mismatches|errors)" and, per recorded
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

#include <dlfcn.h>
#include <strings.h>

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

#if defined(QG_MMA_VIRUS_BINARY)
constexpr int kDefaultFormat = QG_FMT_BF16;
constexpr const char* kWorkload = "MMA Virus";
constexpr const char* kFaultTag = "MMA_VIRUS";
constexpr bool kFurnace = true;
constexpr int kDefaultWarmup = 5;                // mma_virus.cpp:190
#elif defined(QG_DECODE_BINARY)
constexpr int kDefaultFormat = QG_FMT_W4A16;
constexpr const char* kWorkload = "LLM Decode";
constexpr const char* kFaultTag = "LLM_DECODE";
constexpr bool kFurnace = false;
constexpr int kDefaultWarmup = 3;
#else
constexpr int kDefaultFormat = QG_FMT_INT8;
constexpr const char* kWorkload = "Quantized GEMM";
constexpr const char* kFaultTag = "QUANTIZED_GEMM";
constexpr bool kFurnace = false;
constexpr int kDefaultWarmup = 3;
#endif

// Launch-knob clamps with the reference's bounds (common.h:248-311).
constexpr int kMaxKernelLoops = 1000000;
// Longest one timed batch (launches between two synchronisations and two
// verifications) may run, whatever --kernel_loops asks: a batch is the unit of
// verification and of the runner's progress, so it must stay well inside both
// the run's duration and the runner's duration*2+300 s kill (pantheon.py:4018).
constexpr double kMaxBatchSeconds = 1.0;
// Largest batch replayed as one CUDA graph (the W4A16 GEMV's ~200 ms batch is
// ~8,700 calls); larger batches of shorter launches run eagerly.
constexpr int kMaxGraphLaunches = 16384;

struct Options {
    int device = 0, duration = 1, mem_pct = 99;
    bool verify = false, inject = false;
    int kernel_loops = 0;        // launches per timed batch; 0 (flag absent) = size a batch to ~200 ms
    bool loops_given = false;
    int warmup_iters = kDefaultWarmup;
    int format = kDefaultFormat;
    bool format_given = false;
    int m = 0, n = 0, k = 0, copies = 0;
    uint64_t seed = 1;
    // vendor-GEMM flags of the tensor furnace (vendor_gemm.h:32-55)
    std::string gemm_type;
    int gemm_m = 8192, gemm_n = 8192, gemm_k = 8192;
    int probe_ms = 1500, margin_pct = 15;
};

bool is_dense(int f) {
    return f == QG_FMT_BF16 || f == QG_FMT_FP16 || f == QG_FMT_TF32 || f == QG_FMT_E4M3 || f == QG_FMT_FP32;
}

const char* format_name(int f) {
    switch (f) {
        case QG_FMT_INT8: return "INT8 W8A8";
        case QG_FMT_FP8: return "FP8 e4m3 block-128";
        case QG_FMT_NVFP4: return "NVFP4 e2m1/ue4m3";
        case QG_FMT_W4A16: return "W4A16 group-128";
        case QG_FMT_BF16: return "BF16";
        case QG_FMT_FP16: return "FP16";
        case QG_FMT_TF32: return "TF32";
        case QG_FMT_E4M3: return "FP8 (E4M3)";
        case QG_FMT_FP32: return "FP32";
        default: return "?";
    }
}

int parse_format(const std::string& s) {
    if (s == "int8" || s == "i8") return QG_FMT_INT8;
    if (s == "fp8") return QG_FMT_FP8;
    if (s == "nvfp4" || s == "fp4") return QG_FMT_NVFP4;
    if (s == "w4a16") return QG_FMT_W4A16;
    if (s == "bf16") return QG_FMT_BF16;
    if (s == "fp16") return QG_FMT_FP16;
    if (s == "tf32") return QG_FMT_TF32;
    if (s == "e4m3") return QG_FMT_E4M3;
    if (s == "fp32") return QG_FMT_FP32;
    return -1;
}

// --gemm_type names (case-insensitive, vendor_gemm.h:214-221); fp8 is the
// dense e4m3 GEMM here, as there.
int parse_gemm_type(const std::string& s) {
    if (!strcasecmp(s.c_str(), "bf16")) return QG_FMT_BF16;
    if (!strcasecmp(s.c_str(), "fp16")) return QG_FMT_FP16;
    if (!strcasecmp(s.c_str(), "tf32")) return QG_FMT_TF32;
    if (!strcasecmp(s.c_str(), "fp8")) return QG_FMT_E4M3;
    if (!strcasecmp(s.c_str(), "fp32")) return QG_FMT_FP32;
    return -1;
}

// Output type of each dense format: the operand type, fp32 for tf32, bf16 for
// fp8 (vendor_gemm.h:241).
int dense_out_type(int f) {
    return f == QG_FMT_FP16 ? QG_OUT_F16 : (f == QG_FMT_TF32 || f == QG_FMT_FP32) ? QG_OUT_F32 : QG_OUT_BF16;
}

int fail(const std::string& why) {
    std::cerr << "[PANTHEON ERROR] " << why << std::endl;
    return 1;
}

// A deliberate skip (common.h:444-460): the device cannot run this workload,
// which is not a failure of the device.
int skip(int device, const std::string& reason) {
    std::cout << "[PANTHEON] GPU " << device << ": Skipping " << kWorkload << " (" << reason << ")." << std::endl;
    std::cout << "Skipping: " << reason << std::endl;
    return 0;
}

int fail_ctx(qg_ctx* ctx, const char* what) {
    char buf[512];
    qg_last_error(ctx, buf, sizeof(buf));
    std::cerr << "[PANTHEON ERROR] " << what << ": " << buf << std::endl;
    if (ctx) qg_destroy(ctx);
    return 1;
}

// Board energy from NVML (read-only queries), loaded at run time so the
// binary runs where NVML is absent; the device is matched by PCI bus id.
struct EnergyMeter {
    void* lib = nullptr;
    void* dev = nullptr;
    int (*energy)(void*, unsigned long long*) = nullptr;

    bool open(int device) {
        lib = dlopen("libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
        if (!lib) return false;
        auto init = reinterpret_cast<int (*)(void)>(dlsym(lib, "nvmlInit_v2"));
        auto by_bus = reinterpret_cast<int (*)(const char*, void**)>(dlsym(lib, "nvmlDeviceGetHandleByPciBusId_v2"));
        energy = reinterpret_cast<int (*)(void*, unsigned long long*)>(dlsym(lib, "nvmlDeviceGetTotalEnergyConsumption"));
        if (!init || !by_bus || !energy || init() != 0) return false;
        char bus[64];
        if (qg_pci_bus_id(device, bus, sizeof(bus)) != QG_OK) return false;
        if (by_bus(bus, &dev) != 0) return false;
        unsigned long long probe = 0;
        return energy(dev, &probe) == 0;
    }
    bool millijoules(unsigned long long* out) const { return dev && energy(dev, out) == 0; }
};

// Shrink a dense shape, all three dimensions together, until one context of
// it fits in an eighth of free memory, keeping every dimension a multiple of
// 16 (vendor_gemm.h:414-424), so the furnace leaves memory to companion streams.
void fit_dense(qg_cfg& cfg, uint64_t free_b) {
    uint64_t need = 0;
    while ((cfg.m > 256 || cfg.n > 256 || cfg.k > 256) && qg_required_bytes(&cfg, &need) == QG_OK &&
           need > free_b / 8) {
        cfg.m = (cfg.m / 2) & ~15; cfg.n = (cfg.n / 2) & ~15; cfg.k = (cfg.k / 2) & ~15;
        if (cfg.m < 16) cfg.m = 16;
        if (cfg.n < 16) cfg.n = 16;
        if (cfg.k < 16) cfg.k = 16;
    }
}

qg_cfg dense_cfg(int fmt, int m, int n, int k, uint64_t seed) {
    qg_cfg c;
    memset(&c, 0, sizeof(c));
    c.format = fmt;
    c.m = m; c.n = n; c.k = k;
    c.out_type = dense_out_type(fmt);
    c.copies = 1;
    c.seed = seed;
    return c;
}

// --gemm_type auto: the formats are tried in a fixed order and the first one
// accepted is the default; each is run alone for probe_ms with its board
// energy read, and the default is replaced only by a format that draws more
// than margin_pct more power (the selection rule of vendor_gemm.h:426-505).
// Without a meter the default is used.
int pick_by_power(const Options& o, int m, int n, int k, uint64_t free_b) {
    static const int order[] = {QG_FMT_BF16, QG_FMT_FP16, QG_FMT_TF32, QG_FMT_E4M3, QG_FMT_FP32};
    EnergyMeter meter;
    const bool metered = o.probe_ms > 0 && meter.open(o.device);
    if (!metered) std::cout << "  -> No energy meter (or --gemm_probe_ms 0): the default order decides" << std::endl;
    int def = -1, best = -1;
    double def_w = 0.0, best_w = 0.0;
    for (int fmt : order) {
        qg_cfg c = dense_cfg(fmt, m, n, k, o.seed);
        fit_dense(c, free_b);
        qg_ctx* ctx = nullptr;
        if (qg_create(&ctx, o.device, &c) != QG_OK || qg_fill(ctx, o.seed) != QG_OK) {
            char buf[256];
            qg_last_error(ctx, buf, sizeof(buf));
            std::cout << "  -> Probe " << format_name(fmt) << ": skipped (" << buf << ")" << std::endl;
            if (ctx) qg_destroy(ctx);
            continue;
        }
        if (def < 0) def = fmt;
        if (!metered) { qg_destroy(ctx); break; }   // nothing to measure: first accepted wins
        bool ok = qg_run(ctx, 4, nullptr) == QG_OK && qg_synchronize(ctx) == QG_OK;
        unsigned long long e0 = 0, e1 = 0;
        auto t0 = std::chrono::high_resolution_clock::now();
        ok = ok && meter.millijoules(&e0);
        double dt = 0.0;
        while (ok && dt < o.probe_ms / 1000.0) {
            ok = qg_run(ctx, 8, nullptr) == QG_OK && qg_synchronize(ctx) == QG_OK;
            dt = std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - t0).count();
        }
        ok = ok && meter.millijoules(&e1) && e1 > e0 && dt > 0.0;
        const double watts = ok ? ((double)(e1 - e0) / 1000.0) / dt : 0.0;
        qg_destroy(ctx);
        std::cout << "  -> Probe " << format_name(fmt) << ": "
                  << (ok ? std::to_string((int)watts) + " W" : std::string("no energy reading")) << std::endl;
        if (!ok) continue;
        if (fmt == def) def_w = watts;
        if (best < 0 || watts > best_w) { best = fmt; best_w = watts; }
    }
    if (def < 0) return -1;
    int chosen = def;
    if (metered && def_w > 0.0 && best >= 0 && best != def && best_w > def_w * (1.0 + o.margin_pct / 100.0))
        chosen = best;
    std::cout << "  -> Selected " << format_name(chosen)
              << (chosen == def ? " (default order; no format ahead by " : " (ahead of the default by more than ")
              << o.margin_pct << "%)" << std::endl;
    return chosen;
}

void print_faults(qg_ctx* ctx) {
    qg_mismatch log[8];
    const int nlog = qg_mismatch_log(ctx, log, 8);
    for (int i = 0; i < nlog; ++i)
        printf("[SDC FAULT][%s] Output mismatch! Word: %llu | Exp: 0x%08x | Act: 0x%08x | XOR: 0x%08x\n", kFaultTag,
               (unsigned long long)log[i].index, log[i].expected, log[i].actual, log[i].expected ^ log[i].actual);
    // differences the launches of the batch found in their own results (qg_run's per-launch check)
    uint64_t words = 0, diffs = 0, launches = 0;
    if (qg_verify_detail(ctx, &words, &diffs, &launches) == QG_OK && diffs)
        printf("[SDC FAULT][%s] Per-launch check: %llu result segments differed from the golden run in a batch of "
               "%llu checked launches\n", kFaultTag, (unsigned long long)diffs, (unsigned long long)launches);
    fflush(stdout);
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
        else if (a == "--kernel_loops") { if (const char* v = next()) { o.kernel_loops = atoi(v); o.loops_given = true; } }
        else if (a == "--warmup_iters") { if (const char* v = next()) o.warmup_iters = atoi(v); }
        else if (a == "--block_size" || a == "--grid_size" || a == "--sync_mode" || a == "--mma_acc" ||
                 a == "--mma_groups" || a == "--mma_reuse" || a == "--init_pattern" || a == "--gemm") { next(); }
        else if (a == "--format") {
            if (const char* v = next()) {
                o.format = parse_format(v);
                o.format_given = true;
                if (o.format < 0) return fail(std::string("unknown --format ") + v);
            }
        }
        else if (a == "--gemm_type") { if (const char* v = next()) o.gemm_type = v; }
        else if (a == "--gemm_size") { if (const char* v = next()) o.gemm_m = o.gemm_n = o.gemm_k = atoi(v); }
        else if (a == "--gemm_m") { if (const char* v = next()) o.gemm_m = atoi(v); }
        else if (a == "--gemm_n") { if (const char* v = next()) o.gemm_n = atoi(v); }
        else if (a == "--gemm_k") { if (const char* v = next()) o.gemm_k = atoi(v); }
        else if (a == "--gemm_probe_ms") { if (const char* v = next()) o.probe_ms = atoi(v); }
        else if (a == "--gemm_margin") { if (const char* v = next()) o.margin_pct = atoi(v); }
        else if (a == "--m") { if (const char* v = next()) o.m = atoi(v); }
        else if (a == "--n") { if (const char* v = next()) o.n = atoi(v); }
        else if (a == "--k") { if (const char* v = next()) o.k = atoi(v); }
        else if (a == "--copies") { if (const char* v = next()) o.copies = atoi(v); }
        else if (a == "--seed") { if (const char* v = next()) o.seed = strtoull(v, nullptr, 10); }
        // anything else: ignored, as in the reference
    }
    if (kFurnace) {
        o.kernel_loops = 0;   // a WMMA knob there; the GEMM batch is sized to ~200 ms
        o.loops_given = false;
    } else if (o.loops_given && o.kernel_loops < 1) {
        std::cerr << "[PANTHEON] Warning: invalid kernel_loops " << o.kernel_loops << "; using 1." << std::endl;
        o.kernel_loops = 1;
    } else if (o.kernel_loops > kMaxKernelLoops) {
        std::cerr << "[PANTHEON] Warning: kernel_loops " << o.kernel_loops
                  << " would make a single batch effectively unbounded; clamping to " << kMaxKernelLoops << "."
                  << std::endl;
        o.kernel_loops = kMaxKernelLoops;
    }
    if (o.warmup_iters < 0) {
        std::cerr << "[PANTHEON] Warning: invalid warmup_iters " << o.warmup_iters << "; using 0." << std::endl;
        o.warmup_iters = 0;
    }
    if (o.duration < 0) o.duration = 0;
    o.mem_pct = o.mem_pct < 1 ? 1 : (o.mem_pct > 99 ? 99 : o.mem_pct);

    // vendor-GEMM option checks (vendor_gemm.h:510-535), before any device call
    const bool furnace = kFurnace && !o.format_given;
    const bool auto_type = furnace && !strcasecmp(o.gemm_type.c_str(), "auto");
    if (furnace) {
        if (!auto_type && !o.gemm_type.empty()) {
            o.format = parse_gemm_type(o.gemm_type);
            if (o.format < 0)
                return fail("Unknown --gemm_type '" + o.gemm_type + "'. Use auto, bf16, fp16, tf32, fp32 or fp8.");
        }
        if (o.gemm_m < 16 || o.gemm_n < 16 || o.gemm_k < 16) return fail("--gemm_m/n/k must each be at least 16.");
    }

    const int support = qg_device_check(o.device);
    if (support == QG_ERR_UNSUPPORTED) {
        char buf[512];
        qg_last_error(nullptr, buf, sizeof(buf));
        return skip(o.device, buf);
    }
    if (support != QG_OK) return fail_ctx(nullptr, "device query failed");
    uint64_t free_b = 0, total_b = 0;
    if (qg_mem_info(o.device, &free_b, &total_b) != QG_OK) return fail_ctx(nullptr, "device query failed");

    qg_cfg cfg;
    memset(&cfg, 0, sizeof(cfg));
    if (furnace) {
        const int m = (o.m > 0 ? o.m : o.gemm_m) & ~15;
        const int n = (o.n > 0 ? o.n : o.gemm_n) & ~15;
        const int k = (o.k > 0 ? o.k : o.gemm_k) & ~15;
        std::cout << "[PANTHEON] GPU " << o.device << ": Running MMA VIRUS (Physical Tensor Cores)..." << std::endl;
        if (auto_type) {
            std::cout << "[PANTHEON] Choosing the GEMM format by measured power (" << o.probe_ms << " ms each)..."
                      << std::endl;
            o.format = pick_by_power(o, m < 16 ? 16 : m, n < 16 ? 16 : n, k < 16 ? 16 : k, free_b);
            if (o.format < 0) return fail("no GEMM format could be brought up on this device");
        }
        cfg = dense_cfg(o.format, m < 16 ? 16 : m, n < 16 ? 16 : n, k < 16 ? 16 : k, o.seed);
        fit_dense(cfg, free_b);
    } else {
        cfg.format = o.format;
        cfg.m = o.m; cfg.n = o.n; cfg.k = o.k;
        cfg.out_type = is_dense(o.format) ? dense_out_type(o.format) : QG_OUT_BF16;
        cfg.seed = o.seed;
        cfg.copies = 1;
    }

    // Working-set sizing from --mem (ai_workload_template.h:359): operand copies
    // beyond the first only matter for the memory-bound GEMV, where they keep
    // each call streaming from HBM instead of L2.
    const uint64_t budget = free_b / 100 * (uint64_t)o.mem_pct;
    uint64_t one = 0;
    if (qg_required_bytes(&cfg, &one) != QG_OK) return fail_ctx(nullptr, "bad configuration");
    // Four weight sets (4 x 125 MB at configs[3], four times the 126 MB L2) are
    // enough to stream every call from HBM; more only spread the stream over
    // more pages (configs[3] M=1, 10 s runs: 8 sets 4925 GB/s, 4 sets 5048).
    if (o.copies > 0) cfg.copies = o.copies;
    else if (o.format == QG_FMT_W4A16) {
        uint64_t fit = one ? budget / one : 1;
        cfg.copies = (int)(fit < 1 ? 1 : (fit > 4 ? 4 : fit));
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
    const bool flops_metric = is_dense(o.format);
    const int rows = cfg.m > 0 ? cfg.m : (o.format == QG_FMT_W4A16 ? 1 : 0);

    if (furnace) {
        std::cout << "  -> Duration (s):  " << o.duration << std::endl;
        std::cout << "  -> Warmup Iters:  " << o.warmup_iters << std::endl;
        std::cout << "  -> Tensor Engine: " << (o.format == QG_FMT_FP32 ? "CUDA-core FP32 GEMM (" : "tcgen05 GEMM (")
                  << format_name(o.format) << " " << cfg.m << "x" << cfg.n << "x" << cfg.k << ", FP32 accumulate)"
                  << std::endl;
        std::cout << "  -> Verify Mode:   " << (o.verify ? "ON" : "OFF") << std::endl;
    } else {
        std::cout << "[PANTHEON] GPU " << o.device << ": " << kWorkload << " (" << format_name(o.format)
                  << (bw_metric ? " GEMV" : "") << ", sm_100a)" << std::endl;
    }
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
    {
        // The same arguments give the same golden result on every healthy GPU:
        // the runner compares this line across the GPUs of a run.
        uint64_t digest = 0;
        if (qg_golden_digest(ctx, 0, &digest) != QG_OK) return fail_ctx(ctx, "qg_golden_digest");
        char hex[24];
        snprintf(hex, sizeof(hex), "0x%016llx", (unsigned long long)digest);
        std::cout << "  -> Golden Digest: " << hex << std::endl;
    }

    // Warm-up, then a timing probe: without --kernel_loops it sizes the batch
    // (~200 ms per sync, as the reference's vendor GEMM batches:
    // vendor_gemm.h:560-571); with it, it caps the batch at kMaxBatchSeconds.
    // The probe runs after one untimed launch, so first-use costs do not
    // shrink the batch.
    int loops = o.kernel_loops;
    bool use_graph = false;
    {
        Phase ph("qg:warmup");
        if (o.warmup_iters > 0 && (qg_run(ctx, o.warmup_iters, nullptr) != QG_OK || qg_synchronize(ctx) != QG_OK))
            return fail_ctx(ctx, "warm-up");
        if (qg_run(ctx, 1, nullptr) != QG_OK || qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "warm-up");
        const int probe = 4;
        auto t0 = std::chrono::high_resolution_clock::now();
        if (qg_run(ctx, probe, nullptr) != QG_OK || qg_synchronize(ctx) != QG_OK) return fail_ctx(ctx, "warm-up");
        const double per = std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - t0).count() / probe;
        if (loops == 0) {
            const double l = per > 0 ? 0.2 / per : 1.0;
            loops = (int)(l < 1 ? 1 : (l > 100000 ? 100000 : l));
            // a whole number of operand-copy rotations: every batch then starts at
            // the same copy and replays one captured graph
            loops = (loops + cfg.copies - 1) / cfg.copies * cfg.copies;
        } else if (per > 0 && loops * per > kMaxBatchSeconds) {
            const double l = kMaxBatchSeconds / per;
            const int capped = (int)(l < 1 ? 1 : l);
            std::cerr << "[PANTHEON] Warning: kernel_loops " << loops << " would make one batch last "
                      << loops * per << " s; capping to " << capped << " (about " << kMaxBatchSeconds
                      << " s per batch)." << std::endl;
            loops = capped;
        }
        // A batch whose launches rotate through whole operand-copy cycles is
        // captured once as a CUDA graph (here, untimed) and replayed per batch;
        // other batch sizes would start at a different copy each time, and
        // batches of tiny launches would make graphs of too many nodes: those
        // run as eager launches.
        use_graph = loops % cfg.copies == 0 && loops <= kMaxGraphLaunches;
        if (use_graph && (qg_run_graph(ctx, loops, nullptr) != QG_OK || qg_synchronize(ctx) != QG_OK))
            return fail_ctx(ctx, "qg_run_graph");
    }
    uint64_t mismatches = 0;
    if (o.verify) {
        // the warm-up launches checked themselves too: collect what they found
        // before the timed batches, so every batch below reports its own launches
        uint64_t mm = 0;
        if (qg_verify(ctx, &mm) != QG_OK) return fail_ctx(ctx, "qg_verify");
        if (mm) print_faults(ctx);
        mismatches += mm;
    }
    std::cout << "  -> Kernel Loops:  " << loops << std::endl;
    std::cout << "  -> Batch Launch:  " << (use_graph ? "one CUDA graph per batch" : "eager launches") << std::endl;
    if (o.inject) std::cout << "[PANTHEON] Warning: SDC Fault Injection is ACTIVE!" << std::endl;
    std::cout << "[PANTHEON] Starting active telemetry phase..." << std::endl;

    double busy = 0.0;
    uint64_t launches = 0, checked = 0;
    auto start = std::chrono::high_resolution_clock::now();
    do {
        auto b0 = std::chrono::high_resolution_clock::now();
        {
            Phase ph("qg:timed");
            if ((use_graph ? qg_run_graph(ctx, loops, nullptr) : qg_run(ctx, loops, nullptr)) != QG_OK)
                return fail_ctx(ctx, "qg_run");
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
            if (mm) print_faults(ctx);
            mismatches += mm;
            uint64_t w = 0, d = 0, n = 0;
            if (qg_verify_detail(ctx, &w, &d, &n) == QG_OK) checked += n;
        }
    } while (std::chrono::duration_cast<std::chrono::seconds>(std::chrono::high_resolution_clock::now() - start).count() <
             o.duration);

    double rate = 0.0;
    if (busy > 0) rate = bw_metric ? (bytes * (double)launches) / busy / 1e9 : (ops * (double)launches) / busy / 1e12;
    std::cout << "Throughput: " << rate << (bw_metric ? " GB/s" : flops_metric ? " TFLOPS" : " TOPS") << std::endl;
    if (bw_metric && busy > 0) {
        std::cout << "  -> Tokens/s:      " << rows * (double)launches / busy << " (" << rows << " row"
                  << (rows == 1 ? "" : "s") << " per call)" << std::endl;
    }

    int exit_code = 0;
    if (o.verify) {
        if (o.inject) {
            if (qg_inject(ctx) != QG_OK) return fail_ctx(ctx, "qg_inject");
            uint64_t mm = 0;
            if (qg_verify(ctx, &mm) != QG_OK) return fail_ctx(ctx, "qg_verify");
            print_faults(ctx);
            mismatches += mm;
        }
        std::cout << "  -> Launches Checked: " << checked << " of " << launches
                  << " (each launch checks its own result against the golden run)" << std::endl;
        std::cout << "  -> Mismatches:    " << mismatches << std::endl;
        std::cout << "Verification: " << (mismatches ? "FAIL" : "PASS") << " (" << mismatches
                  << (kFurnace ? " errors)" : " mismatches)") << std::endl;
        exit_code = mismatches ? 1 : 0;
    }
    qg_destroy(ctx);
    return exit_code;
}
