// qg_capi.cu -- the context API of include/pantheon_qgemm.h: one workload
// instance per device (operands, outputs, golden results, verification
// counters), driven by the quantized_gemm binary, the Python wrapper and the
// benchmark.  The instance owns its device memory; the caller owns the handle.
#include "qg_common.cuh"
#include "qg_formats.cuh"

#include <cstdarg>
#include <cstdlib>
#include <new>
#include <string>
#include <vector>

struct qg_ctx {
    qg_cfg cfg{};
    int device = 0;
    qg::Layout layout{};
    std::vector<qg::CopyBuffers> copies;
    unsigned long long* counters = nullptr;   // [0] mismatching words, [1] log entries
    unsigned long long* launch_diffs = nullptr;   // per-launch check differences since the last qg_verify
    qg_mismatch* log = nullptr;
    int log_cap = 64;
    int next_copy = 0;
    bool golden_ready = false;
    uint64_t launches_checked = 0;            // launches run with the per-launch check since the last qg_verify
    uint64_t last_words = 0, last_launch_diffs = 0, last_launches = 0;   // split of the last qg_verify
    cudaStream_t stream = nullptr;            // internal stream for fill / golden / verify
    // Batches of qg_run_graph, captured once per (launches, first copy) and
    // replayed; dropped when qg_fill or qg_golden changes what a launch checks.
    struct GraphBatch {
        int iters;
        int start;
        cudaGraphExec_t exec;
    };
    std::vector<GraphBatch> graphs;
    std::string err;
};

namespace {

// Captured batches qg_run_graph keeps per context (each holds its own graph).
constexpr size_t kMaxGraphs = 16;

// Salt of the INT8 row checksums' terms in the golden digest (the output words' is 0).
constexpr uint64_t kCksumDigestSalt = 0xC2B2AE3D27D4EB4Full;

int fail(qg_ctx* c, int rc) {
    if (c) c->err = qg::last_error();
    return rc;
}

#define CTX_CUDA(c, call)                                                                       \
    do {                                                                                        \
        cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess) {                                                                \
            ::qg::set_error("%s failed: %s (%d)", #call, cudaGetErrorString(e_), (int)e_);     \
            return fail(c, QG_ERR_CUDA);                                                        \
        }                                                                                       \
    } while (0)

void drop_graphs(qg_ctx* c) {
    if (c->graphs.empty()) return;
    cudaDeviceSynchronize();   // no replay of these graphs may still be running
    for (auto& g : c->graphs) cudaGraphExecDestroy(g.exec);
    c->graphs.clear();
}

void free_ctx_memory(qg_ctx* c) {
    drop_graphs(c);
    for (auto& cp : c->copies) {
        for (int i = 0; i < qg::kMaxOperands; ++i)
            if (cp.op[i]) cudaFree(cp.op[i]);
        if (cp.out) cudaFree(cp.out);
        if (cp.golden) cudaFree(cp.golden);
        if (cp.cksum) cudaFree(cp.cksum);
        if (cp.golden_cksum) cudaFree(cp.golden_cksum);
        if (cp.scratch) cudaFree(cp.scratch);
        if (cp.check_fp) cudaFree(cp.check_fp);
    }
    c->copies.clear();
    if (c->counters) cudaFree(c->counters);
    if (c->launch_diffs) cudaFree(c->launch_diffs);
    if (c->log) cudaFree(c->log);
    c->counters = nullptr;
    c->launch_diffs = nullptr;
    c->log = nullptr;
}

// The per-launch check of a timed launch of copy `cp` (qg_check.cuh): GEMMs
// and the tcgen05 GEMV compare their fingerprints with the golden launch's,
// the CUDA-core and warp-MMA GEMVs compare their output words with the golden
// output.
// Nothing before qg_golden.
qg::LaunchCheck run_check(const qg_ctx* c, const qg::CopyBuffers& cp) {
    qg::LaunchCheck k;
    if (!c->golden_ready || !c->layout.check_bytes) return k;
    k.expect = static_cast<const uint32_t*>(cp.check_fp);
    k.count = c->launch_diffs;
    if (c->cfg.format == QG_FMT_W4A16) k.golden = cp.golden;
    return k;
}

uint64_t out_alloc_bytes(const qg::Layout& L) { return (L.out_bytes + 15) / 16 * 16; }

int alloc(void** p, uint64_t bytes) {
    if (bytes == 0) { *p = nullptr; return QG_OK; }
    QG_CUDA(cudaMalloc(p, (size_t)bytes));
    return QG_OK;
}

} // namespace

extern "C" {

int qg_required_bytes(const qg_cfg* cfg, uint64_t* bytes) {
    QG_CHECK_ARG(cfg && bytes, "qg_required_bytes: null argument");
    qg::Layout L;
    int rc = qg::layout_for(*cfg, &L);
    if (rc) return rc;
    const int copies = cfg->copies > 0 ? cfg->copies : 1;
    uint64_t per = 0;
    for (int i = 0; i < L.n_ops; ++i) per += L.op_bytes[i];
    per += 2 * out_alloc_bytes(L) + 2 * L.cksum_bytes + L.scratch_bytes + L.check_bytes;
    *bytes = per * (uint64_t)copies + 4096;
    return QG_OK;
}

int qg_create(qg_ctx** out, int device, const qg_cfg* cfg) {
    QG_CHECK_ARG(out && cfg, "qg_create: null argument");
    *out = nullptr;
    qg_ctx* c = new (std::nothrow) qg_ctx;
    if (!c) { qg::set_error("qg_create: out of host memory"); return QG_ERR_ARG; }
    c->cfg = *cfg;
    if (c->cfg.copies <= 0) c->cfg.copies = 1;
    c->device = device;
    int rc = qg::layout_for(c->cfg, &c->layout);
    if (rc) { delete c; return rc; }
    c->cfg.m = c->layout.M;
    c->cfg.n = c->layout.N;
    c->cfg.k = c->layout.K;
    if (cudaSetDevice(device) != cudaSuccess) {
        qg::set_error("qg_create: cudaSetDevice(%d) failed", device);
        delete c;
        return QG_ERR_CUDA;
    }
    qg::DeviceInfo* info = nullptr;
    if ((rc = qg::current_device_info(&info))) { delete c; return rc; }
    c->copies.resize((size_t)c->cfg.copies);
    const qg::Layout& L = c->layout;
    for (auto& cp : c->copies) {
        for (int i = 0; i < L.n_ops; ++i)
            if ((rc = alloc(&cp.op[i], L.op_bytes[i]))) goto oom;
        // Outputs are padded to whole 16-byte groups and zeroed, so the verifier
        // can compare whole 32-bit words even when a 2-byte output has an odd
        // element count (the padding stays zero in both copies).
        if ((rc = alloc(&cp.out, out_alloc_bytes(L)))) goto oom;
        if ((rc = alloc(&cp.golden, out_alloc_bytes(L)))) goto oom;
        if (cp.out && cudaMemset(cp.out, 0, out_alloc_bytes(L)) != cudaSuccess) { rc = QG_ERR_CUDA; goto oom; }
        if (cp.golden && cudaMemset(cp.golden, 0, out_alloc_bytes(L)) != cudaSuccess) { rc = QG_ERR_CUDA; goto oom; }
        if ((rc = alloc(&cp.cksum, L.cksum_bytes))) goto oom;
        if ((rc = alloc(&cp.golden_cksum, L.cksum_bytes))) goto oom;
        if ((rc = alloc(&cp.scratch, L.scratch_bytes))) goto oom;
        if ((rc = alloc(&cp.check_fp, L.check_bytes))) goto oom;
    }
    if ((rc = alloc(reinterpret_cast<void**>(&c->counters), 2 * sizeof(unsigned long long)))) goto oom;
    if ((rc = alloc(reinterpret_cast<void**>(&c->launch_diffs), sizeof(unsigned long long)))) goto oom;
    if (cudaMemset(c->launch_diffs, 0, sizeof(unsigned long long)) != cudaSuccess) { rc = QG_ERR_CUDA; goto oom; }
    if ((rc = alloc(reinterpret_cast<void**>(&c->log), sizeof(qg_mismatch) * (size_t)c->log_cap))) goto oom;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        qg::set_error("qg_create: cudaStreamCreate failed");
        rc = QG_ERR_CUDA;
        goto oom;
    }
    *out = c;
    return QG_OK;
oom:
    free_ctx_memory(c);
    delete c;
    return rc;
}

void qg_destroy(qg_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) { cudaStreamSynchronize(c->stream); cudaStreamDestroy(c->stream); }
    free_ctx_memory(c);
    delete c;
}

int qg_fill(qg_ctx* c, uint64_t seed) {
    QG_CHECK_ARG(c, "qg_fill: null context");
    CTX_CUDA(c, cudaSetDevice(c->device));
    // launches still running on a caller's stream read the operands rewritten here
    CTX_CUDA(c, cudaDeviceSynchronize());
    c->cfg.seed = seed;
    for (size_t i = 0; i < c->copies.size(); ++i) {
        int rc = qg::fill_copy(c->cfg, c->layout, c->copies[i], (int)i, seed, c->stream);
        if (rc) return fail(c, rc);
    }
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    c->golden_ready = false;
    drop_graphs(c);
    return QG_OK;
}

int qg_golden(qg_ctx* c) {
    QG_CHECK_ARG(c, "qg_golden: null context");
    CTX_CUDA(c, cudaSetDevice(c->device));
    // launches still running on a caller's stream write the outputs and row
    // checksums the golden launches write here
    CTX_CUDA(c, cudaDeviceSynchronize());
    for (auto& cp : c->copies) {
        qg::LaunchCheck record;   // the golden launch records its fingerprints for the later launches
        record.record = static_cast<uint32_t*>(cp.check_fp);
        int rc = qg::launch_copy(c->cfg, c->layout, cp, c->stream, 0u, record);
        if (rc) return fail(c, rc);
        CTX_CUDA(c, cudaMemcpyAsync(cp.golden, cp.out, c->layout.out_bytes, cudaMemcpyDeviceToDevice, c->stream));
        if (c->layout.cksum_bytes)
            CTX_CUDA(c, cudaMemcpyAsync(cp.golden_cksum, cp.cksum, c->layout.cksum_bytes, cudaMemcpyDeviceToDevice,
                                        c->stream));
    }
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    int st = qg_device_status(c->device);
    if (st) return fail(c, st);
    CTX_CUDA(c, cudaMemset(c->launch_diffs, 0, sizeof(unsigned long long)));
    c->launches_checked = 0;
    c->golden_ready = true;
    c->next_copy = 0;
    drop_graphs(c);
    return QG_OK;
}

int qg_run(qg_ctx* c, int iters, void* stream) {
    QG_CHECK_ARG(c && iters >= 0, "qg_run: bad argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < iters; ++i) {
        const qg::CopyBuffers& cp = c->copies[(size_t)c->next_copy];
        const qg::LaunchCheck chk = run_check(c, cp);
        // From the second launch on, the kernel before each GEMV on this stream
        // is the previous GEMV of this loop, which writes neither the weights
        // nor the activations: their first loads (and the activations'
        // quantisation) may start before the dependency wait.
        int rc = qg::launch_copy(c->cfg, c->layout, cp, s,
                                 i > 0 ? (QG_GEMV_WEIGHTS_CONST | QG_GEMV_ACTIVATIONS_CONST) : 0u, chk);
        if (rc) return fail(c, rc);
        if (chk.count) ++c->launches_checked;
        c->next_copy = (c->next_copy + 1) % (int)c->copies.size();
    }
    return QG_OK;
}

int qg_run_graph(qg_ctx* c, int iters, void* stream) {
    QG_CHECK_ARG(c && iters >= 0, "qg_run_graph: bad argument");
    if (iters == 0) return QG_OK;
    CTX_CUDA(c, cudaSetDevice(c->device));
    const int copies = (int)c->copies.size();
    const int start = c->next_copy;
    cudaGraphExec_t exec = nullptr;
    for (const auto& g : c->graphs)
        if (g.iters == iters && g.start == start) exec = g.exec;
    if (!exec) {
        // the same launches as qg_run's, captured from the context's own stream
        CTX_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed));
        int rc = QG_OK;
        for (int i = 0, copy = start; i < iters && rc == QG_OK; ++i, copy = (copy + 1) % copies) {
            const qg::CopyBuffers& cp = c->copies[(size_t)copy];
            rc = qg::launch_copy(c->cfg, c->layout, cp, c->stream,
                                 i > 0 ? (QG_GEMV_WEIGHTS_CONST | QG_GEMV_ACTIVATIONS_CONST) : 0u, run_check(c, cp));
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        if (rc != QG_OK || e != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            if (rc == QG_OK) {
                qg::set_error("qg_run_graph: stream capture failed: %s (%d)", cudaGetErrorString(e), (int)e);
                rc = QG_ERR_CUDA;
            }
            return fail(c, rc);
        }
        const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ei != cudaSuccess) {
            qg::set_error("qg_run_graph: cudaGraphInstantiate failed: %s (%d)", cudaGetErrorString(ei), (int)ei);
            return fail(c, QG_ERR_CUDA);
        }
        if (c->graphs.size() >= kMaxGraphs) {   // keep the most recent batches only
            CTX_CUDA(c, cudaDeviceSynchronize());   // the oldest may still be replaying
            cudaGraphExecDestroy(c->graphs.front().exec);
            c->graphs.erase(c->graphs.begin());
        }
        c->graphs.push_back({iters, start, exec});
    }
    CTX_CUDA(c, cudaGraphLaunch(exec, static_cast<cudaStream_t>(stream)));
    if (run_check(c, c->copies[(size_t)start]).count) c->launches_checked += (uint64_t)iters;
    c->next_copy = (int)((start + (long long)iters) % copies);
    return QG_OK;
}

int qg_verify(qg_ctx* c, uint64_t* mismatches) {
    QG_CHECK_ARG(c && mismatches, "qg_verify: null argument");
    QG_CHECK_ARG(c->golden_ready, "qg_verify: no golden result (call qg_golden first)");
    CTX_CUDA(c, cudaSetDevice(c->device));
    // Outputs written on another stream must be complete before the compare.
    CTX_CUDA(c, cudaDeviceSynchronize());
    CTX_CUDA(c, cudaMemsetAsync(c->counters, 0, 2 * sizeof(unsigned long long), c->stream));
    for (auto& cp : c->copies) {
        int rc = qg::verify_words(cp.out, cp.golden, (c->layout.out_bytes + 3) / 4, c->counters, c->log, c->log_cap, c->stream);
        if (rc) return fail(c, rc);
        if (c->layout.cksum_bytes) {
            rc = qg::verify_words(cp.cksum, cp.golden_cksum, c->layout.cksum_bytes / 4, c->counters, c->log, c->log_cap,
                                  c->stream);
            if (rc) return fail(c, rc);
        }
    }
    unsigned long long h[2] = {0, 0}, d = 0;
    CTX_CUDA(c, cudaMemcpyAsync(h, c->counters, sizeof(h), cudaMemcpyDeviceToHost, c->stream));
    CTX_CUDA(c, cudaMemcpyAsync(&d, c->launch_diffs, sizeof(d), cudaMemcpyDeviceToHost, c->stream));
    CTX_CUDA(c, cudaMemsetAsync(c->launch_diffs, 0, sizeof(d), c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    int st = qg_device_status(c->device);
    if (st) return fail(c, st);
    c->last_words = h[0];
    c->last_launch_diffs = d;
    c->last_launches = c->launches_checked;
    c->launches_checked = 0;
    *mismatches = h[0] + d;
    return QG_OK;
}

int qg_golden_digest(qg_ctx* c, int copy, uint64_t* digest) {
    QG_CHECK_ARG(c && digest && copy >= 0 && copy < (int)c->copies.size(), "qg_golden_digest: bad argument");
    QG_CHECK_ARG(c->golden_ready, "qg_golden_digest: no golden result (call qg_golden first)");
    CTX_CUDA(c, cudaSetDevice(c->device));
    const qg::CopyBuffers& cp = c->copies[(size_t)copy];
    // counters[0] is free outside qg_verify
    CTX_CUDA(c, cudaMemsetAsync(c->counters, 0, sizeof(unsigned long long), c->stream));
    int rc = qg::digest_words(cp.golden, (c->layout.out_bytes + 3) / 4, 0ull, c->counters, c->stream);
    if (!rc && c->layout.cksum_bytes)
        rc = qg::digest_words(cp.golden_cksum, c->layout.cksum_bytes / 4, kCksumDigestSalt, c->counters, c->stream);
    if (rc) return fail(c, rc);
    unsigned long long h = 0;
    CTX_CUDA(c, cudaMemcpyAsync(&h, c->counters, sizeof(h), cudaMemcpyDeviceToHost, c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    *digest = h;
    return QG_OK;
}

int qg_verify_detail(const qg_ctx* c, uint64_t* words, uint64_t* launch_diffs, uint64_t* launches_checked) {
    QG_CHECK_ARG(c && words && launch_diffs && launches_checked, "qg_verify_detail: null argument");
    *words = c->last_words;
    *launch_diffs = c->last_launch_diffs;
    *launches_checked = c->last_launches;
    return QG_OK;
}

int qg_flip_operand_bit(qg_ctx* c, int copy, int slot, uint64_t byte, int bit, void* stream) {
    QG_CHECK_ARG(c && copy >= 0 && copy < (int)c->copies.size(), "qg_flip_operand_bit: bad copy");
    QG_CHECK_ARG(slot >= 0 && slot < c->layout.n_ops && byte < c->layout.op_bytes[slot] && bit >= 0 && bit < 8,
                 "qg_flip_operand_bit: no byte %llu bit %d in operand slot %d", (unsigned long long)byte, bit, slot);
    QG_CHECK_ARG(!(c->cfg.format == QG_FMT_NVFP4 && slot == 4),
                 "qg_flip_operand_bit: the NVFP4 per-tensor scales are passed by value; flip another slot");
    CTX_CUDA(c, cudaSetDevice(c->device));
    int rc = qg::flip_bit_at(c->copies[(size_t)copy].op[slot], byte, bit, static_cast<cudaStream_t>(stream));
    return rc ? fail(c, rc) : QG_OK;
}

int qg_mismatch_log(qg_ctx* c, qg_mismatch* out, int cap) {
    QG_CHECK_ARG(c && (out || cap == 0), "qg_mismatch_log: null argument");
    CTX_CUDA(c, cudaSetDevice(c->device));
    unsigned long long h[2] = {0, 0};
    CTX_CUDA(c, cudaMemcpy(h, c->counters, sizeof(h), cudaMemcpyDeviceToHost));
    int n = (int)(h[1] < (unsigned long long)c->log_cap ? h[1] : (unsigned long long)c->log_cap);
    if (n > cap) n = cap;
    if (n > 0) CTX_CUDA(c, cudaMemcpy(out, c->log, sizeof(qg_mismatch) * (size_t)n, cudaMemcpyDeviceToHost));
    return n;
}

int qg_inject(qg_ctx* c) {
    QG_CHECK_ARG(c, "qg_inject: null context");
    CTX_CUDA(c, cudaSetDevice(c->device));
    CTX_CUDA(c, cudaDeviceSynchronize());
    int rc = qg::flip_bit(c->copies[0].out, c->stream);
    if (rc) return fail(c, rc);
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return QG_OK;
}

double qg_ops_per_launch(const qg_ctx* c) { return c ? c->layout.ops : 0.0; }
double qg_bytes_per_launch(const qg_ctx* c) { return c ? c->layout.bytes : 0.0; }

int qg_upload(qg_ctx* c, int copy, const void* const* host, void* stream) {
    QG_CHECK_ARG(c && host && copy >= 0 && copy < (int)c->copies.size(), "qg_upload: bad argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < c->layout.n_ops; ++i) {
        QG_CHECK_ARG(host[i], "qg_upload: null host operand %d", i);
        CTX_CUDA(c, cudaMemcpyAsync(c->copies[(size_t)copy].op[i], host[i], c->layout.op_bytes[i],
                                    cudaMemcpyHostToDevice, s));
    }
    if (c->cfg.format == QG_FMT_NVFP4) {
        // the launch passes the two per-tensor scales by value: take the uploaded ones
        const float* g = static_cast<const float*>(host[4]);
        c->copies[(size_t)copy].global_a = g[0];
        c->copies[(size_t)copy].global_b = g[1];
    }
    return QG_OK;
}

int qg_download(qg_ctx* c, int copy, void* host_out, void* stream) {
    QG_CHECK_ARG(c && host_out && copy >= 0 && copy < (int)c->copies.size(), "qg_download: bad argument");
    CTX_CUDA(c, cudaMemcpyAsync(host_out, c->copies[(size_t)copy].out, c->layout.out_bytes, cudaMemcpyDeviceToHost,
                                static_cast<cudaStream_t>(stream)));
    return QG_OK;
}

// Launch one GEMM on copy `copy` (used by the end-to-end path after qg_upload).
int qg_run_copy(qg_ctx* c, int copy, void* stream) {
    QG_CHECK_ARG(c && copy >= 0 && copy < (int)c->copies.size(), "qg_run_copy: bad argument");
    int rc = qg::launch_copy(c->cfg, c->layout, c->copies[(size_t)copy], static_cast<cudaStream_t>(stream));
    return rc ? fail(c, rc) : QG_OK;
}

int qg_tensor(qg_ctx* c, int copy, int slot, void** ptr, uint64_t* bytes) {
    QG_CHECK_ARG(c && ptr && copy >= 0 && copy < (int)c->copies.size(), "qg_tensor: bad argument");
    const qg::CopyBuffers& cp = c->copies[(size_t)copy];
    const qg::Layout& L = c->layout;
    void* p = nullptr;
    uint64_t b = 0;
    if (slot >= 0 && slot < L.n_ops) { p = cp.op[slot]; b = L.op_bytes[slot]; }
    else if (slot == 5) { p = cp.out; b = L.out_bytes; }
    else if (slot == 6) { p = cp.golden; b = L.out_bytes; }
    else if (slot == 7) { p = cp.cksum; b = L.cksum_bytes; }
    else { qg::set_error("qg_tensor: no slot %d for this format", slot); return QG_ERR_ARG; }
    *ptr = p;
    if (bytes) *bytes = b;
    return QG_OK;
}

int qg_last_error(const qg_ctx* c, char* buf, size_t len) {
    if (!buf || len == 0) return QG_ERR_ARG;
    const char* msg = (c && !c->err.empty()) ? c->err.c_str() : qg::last_error();
    snprintf(buf, len, "%s", msg);
    return QG_OK;
}

int qg_abi_version(void) { return QG_ABI_VERSION; }

int qg_synchronize(qg_ctx* c) {
    QG_CHECK_ARG(c, "qg_synchronize: null context");
    CTX_CUDA(c, cudaSetDevice(c->device));
    CTX_CUDA(c, cudaDeviceSynchronize());
    int st = qg_device_status(c->device);
    return st ? fail(c, st) : QG_OK;
}

int qg_mem_info(int device, uint64_t* free_bytes, uint64_t* total_bytes) {
    QG_CHECK_ARG(free_bytes && total_bytes, "qg_mem_info: null argument");
    QG_CUDA(cudaSetDevice(device));
    size_t f = 0, t = 0;
    QG_CUDA(cudaMemGetInfo(&f, &t));
    *free_bytes = f;
    *total_bytes = t;
    return QG_OK;
}

int qg_device_check(int device) {
    QG_CUDA(cudaSetDevice(device));
    qg::DeviceInfo* info = nullptr;
    return qg::current_device_info(&info);
}

int qg_pci_bus_id(int device, char* buf, int len) {
    QG_CHECK_ARG(buf && len >= 16, "qg_pci_bus_id: buffer of at least 16 bytes required");
    QG_CUDA(cudaDeviceGetPCIBusId(buf, len, device));
    return QG_OK;
}

} // extern "C"
