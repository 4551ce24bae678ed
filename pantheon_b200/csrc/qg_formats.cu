// qg_formats.cu -- per-format layout, generation and launch for the context API.
//
// Format defaults are the workload configurations: INT8 W8A8 at M=N=K=8192
// with bf16 output; FP8 block-128 at M=N=8192, K=16384; NVFP4 at 16384^3;
// W4A16 at M=1, K=8192, N=28672; the dense tensor-furnace formats at 8192^3.  Tensor ids give every tensor of every copy
// its own generator stream: id = 8 * copy + slot.
#include "qg_formats.cuh"

namespace qg {

static int out_elem_bytes(int out_type) { return (out_type == QG_OUT_BF16 || out_type == QG_OUT_F16) ? 2 : 4; }

uint32_t dense_elem_bytes(int fmt) {
    switch (fmt) {
        case QG_FMT_BF16: case QG_FMT_FP16: return 2;
        case QG_FMT_TF32: case QG_FMT_FP32: return 4;
        case QG_FMT_E4M3: return 1;
        default: return 0;
    }
}

int layout_for(const qg_cfg& cfg, Layout* L) {
    Layout l;
    l.format = cfg.format;
    l.out_type = cfg.out_type;
    switch (cfg.format) {
        case QG_FMT_INT8: {
            l.M = cfg.m > 0 ? cfg.m : 8192;
            l.N = cfg.n > 0 ? cfg.n : 8192;
            l.K = cfg.k > 0 ? cfg.k : 8192;
            QG_CHECK_ARG(l.K % 16 == 0 && l.K <= 131072, "INT8: K=%d must be a multiple of 16 and <= 131072", l.K);
            QG_CHECK_ARG(l.out_type == QG_OUT_BF16 || l.out_type == QG_OUT_F32 || l.out_type == QG_OUT_S32,
                         "INT8: bad out_type %d", l.out_type);
            l.n_ops = 4;
            l.op_bytes[0] = (uint64_t)l.M * l.K;
            l.op_bytes[1] = (uint64_t)l.N * l.K;
            l.op_bytes[2] = 4ull * l.M;
            l.op_bytes[3] = 4ull * l.N;
            l.out_bytes = (uint64_t)l.M * l.N * out_elem_bytes(l.out_type);
            l.cksum_bytes = 4ull * l.M;
            l.check_bytes = 4ull * gemm_i8_check_slots(l.M, l.N);
            l.ops = 2.0 * l.M * (double)l.N * l.K;
            l.bytes = (double)(l.op_bytes[0] + l.op_bytes[1] + l.op_bytes[2] + l.op_bytes[3] + l.out_bytes + l.cksum_bytes);
            break;
        }
        case QG_FMT_FP8: {
            l.M = cfg.m > 0 ? cfg.m : 8192;
            l.N = cfg.n > 0 ? cfg.n : 8192;
            l.K = cfg.k > 0 ? cfg.k : 16384;
            QG_CHECK_ARG(l.K % 128 == 0, "FP8: K=%d must be a multiple of 128", l.K);
            QG_CHECK_ARG(l.out_type == QG_OUT_BF16 || l.out_type == QG_OUT_F32, "FP8: bad out_type %d", l.out_type);
            l.n_ops = 4;                                                   // A, B, sa, sb
            l.op_bytes[0] = (uint64_t)l.M * l.K;
            l.op_bytes[1] = (uint64_t)l.N * l.K;
            l.op_bytes[2] = 4ull * l.M * (l.K / 128);
            l.op_bytes[3] = 4ull * ((l.N + 127) / 128) * (l.K / 128);
            l.out_bytes = (uint64_t)l.M * l.N * out_elem_bytes(l.out_type);
            l.check_bytes = 4ull * gemm_fp8_check_slots(l.M, l.N);
            l.ops = 2.0 * l.M * (double)l.N * l.K;
            l.bytes = (double)(l.op_bytes[0] + l.op_bytes[1] + l.op_bytes[2] + l.op_bytes[3] + l.out_bytes);
            break;
        }
        case QG_FMT_NVFP4: {
            l.M = cfg.m > 0 ? cfg.m : 16384;
            l.N = cfg.n > 0 ? cfg.n : 16384;
            l.K = cfg.k > 0 ? cfg.k : 16384;
            QG_CHECK_ARG(l.K % 256 == 0, "NVFP4: K=%d must be a multiple of 256", l.K);
            QG_CHECK_ARG(l.out_type == QG_OUT_BF16 || l.out_type == QG_OUT_F32, "NVFP4: bad out_type %d", l.out_type);
            l.n_ops = 5;                                                   // A, sfa, B, sfb, global scales
            l.op_bytes[0] = (uint64_t)l.M * l.K / 2;
            l.op_bytes[1] = nvfp4_sf_bytes(l.M, l.K);
            l.op_bytes[2] = (uint64_t)l.N * l.K / 2;
            l.op_bytes[3] = nvfp4_sf_bytes(l.N, l.K);
            l.op_bytes[4] = 16;
            l.out_bytes = (uint64_t)l.M * l.N * out_elem_bytes(l.out_type);
            l.check_bytes = 4ull * gemm_nvfp4_check_slots(l.M, l.N);
            l.scratch_bytes = 16;
            l.ops = 2.0 * l.M * (double)l.N * l.K;
            l.bytes = (double)(l.op_bytes[0] + l.op_bytes[1] + l.op_bytes[2] + l.op_bytes[3] + l.out_bytes);
            break;
        }
        case QG_FMT_W4A16: {
            l.M = cfg.m > 0 ? cfg.m : 1;
            l.N = cfg.n > 0 ? cfg.n : 28672;
            l.K = cfg.k > 0 ? cfg.k : 8192;
            QG_CHECK_ARG(l.K % 128 == 0, "W4A16: K=%d must be a multiple of 128", l.K);
            QG_CHECK_ARG(l.N % 4 == 0, "W4A16: N=%d must be a multiple of 4", l.N);
            QG_CHECK_ARG(l.out_type == QG_OUT_BF16 || l.out_type == QG_OUT_F32, "W4A16: bad out_type %d", l.out_type);
            l.n_ops = 4;
            l.op_bytes[0] = 2ull * l.M * l.K;                  // X bf16
            l.op_bytes[1] = (uint64_t)l.K / 8 * l.N * 4;       // W packed int4
            l.op_bytes[2] = (uint64_t)l.K / 128 * l.N * 2;     // S fp16
            l.op_bytes[3] = (uint64_t)l.K / 128 * l.N * 2;     // Z fp16
            l.out_bytes = (uint64_t)l.M * l.N * out_elem_bytes(l.out_type);
            l.scratch_bytes = gemv_w4a16_workspace_bytes(l.M, l.N, l.K, 148);
            // per-launch check of the tensor-core chunks: one fingerprint per (16-row chunk, column)
            l.check_bytes = 4ull * (uint64_t)((l.M + 15) / 16) * (uint64_t)l.N;
            l.ops = 2.0 * l.M * (double)l.N * l.K;
            l.bytes = (double)(l.op_bytes[0] + l.op_bytes[1] + l.op_bytes[2] + l.op_bytes[3] + l.out_bytes);
            break;
        }
        case QG_FMT_BF16:
        case QG_FMT_FP16:
        case QG_FMT_TF32:
        case QG_FMT_E4M3:
        case QG_FMT_FP32: {
            // The tensor furnace: C = A B^T at 8192^3 by default, as the
            // reference's vendor GEMM (vendor_gemm.h:38).
            const uint32_t eb = dense_elem_bytes(cfg.format);
            l.M = cfg.m > 0 ? cfg.m : 8192;
            l.N = cfg.n > 0 ? cfg.n : 8192;
            l.K = cfg.k > 0 ? cfg.k : 8192;
            QG_CHECK_ARG(((uint64_t)l.K * eb) % 16 == 0, "dense GEMM: K=%d must make 16-byte rows", l.K);
            QG_CHECK_ARG(l.out_type == QG_OUT_BF16 || l.out_type == QG_OUT_F16 || l.out_type == QG_OUT_F32,
                         "dense GEMM: bad out_type %d", l.out_type);
            l.n_ops = 2;
            l.op_bytes[0] = (uint64_t)l.M * l.K * eb;
            l.op_bytes[1] = (uint64_t)l.N * l.K * eb;
            l.out_bytes = (uint64_t)l.M * l.N * out_elem_bytes(l.out_type);
            // the fp32 CUDA-core GEMM has no per-launch check: its output is compared per batch only
            if (cfg.format != QG_FMT_FP32) l.check_bytes = 4ull * gemm_i8_check_slots(l.M, l.N);
            l.ops = 2.0 * l.M * (double)l.N * l.K;
            l.bytes = (double)(l.op_bytes[0] + l.op_bytes[1] + l.out_bytes);
            break;
        }
        default:
            set_error("format %d is not available in this build", cfg.format);
            return QG_ERR_ARG;
    }
    QG_CHECK_ARG(l.M > 0 && l.N > 0 && l.K > 0, "empty shape %dx%dx%d", l.M, l.N, l.K);
    *L = l;
    return QG_OK;
}

int fill_copy(const qg_cfg& cfg, const Layout& L, CopyBuffers& cp, int copy_index, uint64_t seed, cudaStream_t s) {
    const uint32_t base = 8u * (uint32_t)copy_index;
    int rc = QG_OK;
    switch (cfg.format) {
        case QG_FMT_INT8:
            if ((rc = gen_i8(cp.op[0], L.op_bytes[0], seed, base + 0, s))) return rc;
            if ((rc = gen_i8(cp.op[1], L.op_bytes[1], seed, base + 1, s))) return rc;
            if ((rc = gen_uniform(cp.op[2], (uint64_t)L.M, 0.001f, 0.01f, seed, base + 2, s))) return rc;
            if ((rc = gen_uniform(cp.op[3], (uint64_t)L.N, 0.001f, 0.01f, seed, base + 3, s))) return rc;
            return QG_OK;
        case QG_FMT_FP8:
            return gen_fp8(cp.op[0], cp.op[2], cp.op[1], cp.op[3], L.M, L.N, L.K, seed, base, s);
        case QG_FMT_NVFP4: {
            float* g = static_cast<float*>(cp.op[4]);
            if ((rc = gen_nvfp4(cp.op[0], cp.op[1], cp.op[2], cp.op[3], g, cp.scratch, L.M, L.N, L.K, seed, base, s)))
                return rc;
            float h[2] = {1.0f, 1.0f};
            QG_CUDA(cudaMemcpyAsync(h, g, sizeof(h), cudaMemcpyDeviceToHost, s));
            QG_CUDA(cudaStreamSynchronize(s));
            cp.global_a = h[0];
            cp.global_b = h[1];
            return QG_OK;
        }
        case QG_FMT_W4A16:
            if (cp.scratch) QG_CUDA(cudaMemsetAsync(cp.scratch, 0, L.scratch_bytes, s));
            return gen_w4a16(cp.op[0], cp.op[1], cp.op[2], cp.op[3], L.M, L.N, L.K, seed, base, s);
        case QG_FMT_BF16:
        case QG_FMT_FP16:
        case QG_FMT_TF32:
        case QG_FMT_E4M3:
        case QG_FMT_FP32: {
            const uint32_t eb = dense_elem_bytes(cfg.format);
            if ((rc = gen_dense(cfg.format, cp.op[0], L.op_bytes[0] / eb, seed, base + 0, s))) return rc;
            return gen_dense(cfg.format, cp.op[1], L.op_bytes[1] / eb, seed, base + 1, s);
        }
        default:
            set_error("format %d is not available in this build", cfg.format);
            return QG_ERR_ARG;
    }
}

int launch_copy(const qg_cfg& cfg, const Layout& L, const CopyBuffers& cp, cudaStream_t s, unsigned int gemv_flags,
                const LaunchCheck& chk) {
    switch (cfg.format) {
        case QG_FMT_INT8:
            return gemm_i8(cp.op[0], cp.op[1], cp.op[2], cp.op[3], cp.out, L.out_type, cp.cksum, L.M, L.N, L.K, s, chk);
        case QG_FMT_FP8:
            return gemm_fp8(cp.op[0], cp.op[1], cp.op[2], cp.op[3], cp.out, L.out_type, L.M, L.N, L.K, s, chk);
        case QG_FMT_NVFP4:
            return gemm_nvfp4(cp.op[0], cp.op[1], cp.op[2], cp.op[3], cp.global_a, cp.global_b, cp.out, L.out_type,
                              L.M, L.N, L.K, s, chk);
        case QG_FMT_W4A16:
            return gemv_w4a16(cp.op[0], cp.op[1], cp.op[2], cp.op[3], cp.out, L.out_type, L.M, L.N, L.K, cp.scratch,
                              L.scratch_bytes, s, gemv_flags, chk);
        case QG_FMT_BF16:
        case QG_FMT_FP16:
        case QG_FMT_TF32:
        case QG_FMT_E4M3:
            return gemm_dense_format(cfg.format, cp.op[0], cp.op[1], 1.0f, cp.out, L.out_type, L.M, L.N, L.K, s, chk);
        case QG_FMT_FP32:
            return gemm_f32(cp.op[0], cp.op[1], 1.0f, cp.out, L.out_type, L.M, L.N, L.K, s);
        default:
            set_error("format %d is not available in this build", cfg.format);
            return QG_ERR_ARG;
    }
}

} // namespace qg
