// vendor_gemm_check.cu -- TEST INFRASTRUCTURE, not part of the product.
//
// Holds this library's dense tensor-furnace GEMMs (the mma_virus replacement)
// to the reference's own furnace GEMM: the reference's PantheonGemm
// (kernels/common/vendor_gemm.h:197-360, cuBLASLt loaded by dlopen, "TN"
// operands, fp32 accumulate) is compiled from the reference's header where it
// lies, initialised at one shape and format (it allocates and fills its own
// operands with its own generator, vendor_gemm.h:184-191 and :293-310), and
// run once; then this library's GEMM of the same format runs on the SAME
// device operands, and the two outputs are compared element by element.
//
//   vendor_gemm_check <bf16|fp16|tf32|fp32|fp8> <m> <n> <k>
//
// Prints one JSON line: the format, shape, the largest relative difference
// |ours - ref| / max(|ref|, rms(ref)), the largest pure relative difference
// over elements with |ref| > rms/8, and how many elements differ beyond 1e-2
// of max(|ref|, rms).  Where the reference's GEMM cannot be brought up it
// prints {"unavailable": "<its reason>"} and exits 0.
//
// Layouts: the reference stores A as k x m read down k (our A[M,K], K
// contiguous), B as k x n read down k (our B[N,K]), and C column-major m x n
// (C[n][m]); ours is C[m][n] row-major, so element (i, j) is ref[j*m + i] and
// ours[i*n + j].
#include "vendor_gemm.h"
#include "../include/pantheon_qgemm.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

static float bf16_to_f32(uint16_t h) { uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f; }
static float f16_to_f32(uint16_t h) { return __half2float(*reinterpret_cast<const __half*>(&h)); }

int main(int argc, char** argv) {
    if (argc < 5) { fprintf(stderr, "usage: %s <bf16|fp16|tf32|fp32|fp8> <m> <n> <k>\n", argv[0]); return 2; }
    PantheonGemmType t;
    if (!PantheonGemm::parse_type(argv[1], &t)) { fprintf(stderr, "unknown type %s\n", argv[1]); return 2; }
    const int m = atoi(argv[2]), n = atoi(argv[3]), k = atoi(argv[4]);
    PantheonGemm g;
    if (!g.init(t, m, n, k)) {
        printf("{\"type\": \"%s\", \"unavailable\": \"%s\"}\n", argv[1], g.why.c_str());
        return 0;
    }
    if (!g.run(0) || cudaDeviceSynchronize() != cudaSuccess) { fprintf(stderr, "reference GEMM failed\n"); return 1; }

    const size_t nc = (size_t)m * n;
    const size_t ob = PantheonGemm::out_bytes(t);
    void* ours = nullptr;
    if (cudaMalloc(&ours, nc * ob) != cudaSuccess) { fprintf(stderr, "cudaMalloc failed\n"); return 1; }
    int rc;
    switch (t) {
        case GEMM_BF16: rc = qg_gemm_bf16(g.a, g.b, 1.0f, ours, QG_OUT_BF16, m, n, k, nullptr); break;
        case GEMM_FP16: rc = qg_gemm_f16(g.a, g.b, 1.0f, ours, QG_OUT_F16, m, n, k, nullptr); break;
        case GEMM_TF32: rc = qg_gemm_tf32(g.a, g.b, 1.0f, ours, QG_OUT_F32, m, n, k, nullptr); break;
        case GEMM_FP32: rc = qg_gemm_f32(g.a, g.b, 1.0f, ours, QG_OUT_F32, m, n, k, nullptr); break;
        default: rc = qg_gemm_e4m3(g.a, g.b, 1.0f, ours, QG_OUT_BF16, m, n, k, nullptr); break;
    }
    if (rc != QG_OK || cudaDeviceSynchronize() != cudaSuccess || qg_device_status(0) != QG_OK) {
        char buf[256];
        qg_last_error(nullptr, buf, sizeof(buf));
        fprintf(stderr, "our GEMM failed: %s\n", buf);
        return 1;
    }
    std::vector<uint8_t> hr(nc * ob), ho(nc * ob);
    cudaMemcpy(hr.data(), g.c, nc * ob, cudaMemcpyDeviceToHost);
    cudaMemcpy(ho.data(), ours, nc * ob, cudaMemcpyDeviceToHost);
    auto val = [&](const std::vector<uint8_t>& v, size_t idx) -> double {
        if (ob == 4) { float f; memcpy(&f, &v[idx * 4], 4); return f; }
        uint16_t h;
        memcpy(&h, &v[idx * 2], 2);
        return t == GEMM_FP16 ? f16_to_f32(h) : bf16_to_f32(h);
    };
    double ss = 0.0;
    for (size_t i = 0; i < nc; ++i) { const double r = val(hr, i); ss += r * r; }
    const double rms = std::sqrt(ss / (double)nc);
    double max_rel = 0.0, max_pure = 0.0;
    size_t over = 0, nonfinite = 0;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            const double r = val(hr, (size_t)j * m + i), o = val(ho, (size_t)i * n + j);
            if (!std::isfinite(r) || !std::isfinite(o)) { ++nonfinite; continue; }
            const double d = std::fabs(o - r);
            const double rel = d / std::fmax(std::fabs(r), rms);
            if (rel > max_rel) max_rel = rel;
            if (rel > 1e-2) ++over;
            if (std::fabs(r) > rms / 8) max_pure = std::fmax(max_pure, d / std::fabs(r));
        }
    printf("{\"type\": \"%s\", \"m\": %d, \"n\": %d, \"k\": %d, \"rms\": %.6g, \"max_rel\": %.6g, "
           "\"max_rel_above_rms_8\": %.6g, \"over_1e-2\": %zu, \"nonfinite\": %zu}\n",
           argv[1], m, n, k, rms, max_rel, max_pure, over, nonfinite);
    cudaFree(ours);
    g.release();
    return 0;
}
