// qg_formats.cuh -- per-format buffer layout, operand generation and launch,
// shared by the context API; plus the internal entry points of each kernel file.
#pragma once

#include "qg_common.cuh"
#include "qg_check.cuh"

namespace qg {

constexpr int kMaxOperands = 5;

// Sizes of one operand set and its results for a given configuration.
struct Layout {
    int format = 0;
    int M = 0, N = 0, K = 0;
    int out_type = QG_OUT_BF16;
    int n_ops = 0;
    uint64_t op_bytes[kMaxOperands] = {};
    uint64_t out_bytes = 0;
    uint64_t cksum_bytes = 0;
    uint64_t scratch_bytes = 0;
    uint64_t check_bytes = 0;   // per-launch check fingerprints of one copy (GEMMs; 0 for the GEMV)
    double ops = 0.0;     // useful arithmetic per launch (2 M N K)
    double bytes = 0.0;   // algorithmic bytes moved per launch
    float global_a = 1.0f, global_b = 1.0f;   // NVFP4 per-tensor scales
};

// Device buffers of one operand copy.
struct CopyBuffers {
    void* op[kMaxOperands] = {};
    void* out = nullptr;
    void* golden = nullptr;
    void* cksum = nullptr;
    void* golden_cksum = nullptr;
    void* scratch = nullptr;
    void* check_fp = nullptr;   // golden fingerprints of the per-launch check (GEMMs)
    float global_a = 1.0f, global_b = 1.0f;
};

int layout_for(const qg_cfg& cfg, Layout* L);
int fill_copy(const qg_cfg& cfg, const Layout& L, CopyBuffers& cp, int copy_index, uint64_t seed, cudaStream_t s);
// `gemv_flags` (QG_GEMV_WEIGHTS_CONST | QG_GEMV_ACTIVATIONS_CONST, or 0) is passed to the W4A16 GEMV; `chk`
// makes the launch record (golden) or check its own output (qg_check.cuh).
int launch_copy(const qg_cfg& cfg, const Layout& L, const CopyBuffers& cp, cudaStream_t s, unsigned int gemv_flags = 0,
                const LaunchCheck& chk = LaunchCheck{});

// Kernel entry points (one per kernel file).  A default LaunchCheck checks nothing.
int gemm_i8(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type, void* row_cksum,
            int M, int N, int K, cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{});
// Fingerprint slots of one launch's per-launch check (qg_check.cuh), per kernel family.
uint64_t gemm_i8_check_slots(int M, int N);      // INT8 and the dense furnace kinds
uint64_t gemm_fp8_check_slots(int M, int N);
uint64_t gemm_nvfp4_check_slots(int M, int N);
int gen_i8(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s);
int gen_dense(int fmt, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s);
// Dense tensor-furnace GEMM of a QG_FMT_BF16 / FP16 / TF32 / E4M3 workload.
int gemm_dense_format(int fmt, const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                      cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{});
uint32_t dense_elem_bytes(int fmt);
int gemm_f32(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
             cudaStream_t stream);
int gen_uniform(void* out, uint64_t n, float lo, float hi, uint64_t seed, uint32_t tensor_id, cudaStream_t s);
int gen_normal(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s);
int gen_fp8(void* A, void* SA, void* B, void* SB, int M, int N, int K, uint64_t seed, uint32_t tid0, cudaStream_t s);
int gemm_fp8(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type, int M, int N, int K,
             cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{});
uint64_t nvfp4_sf_bytes(int R, int K);
int gen_nvfp4(void* A, void* SFA, void* B, void* SFB, float* gscales, void* work, int M, int N, int K, uint64_t seed,
              uint32_t tid0, cudaStream_t s);
int gemm_nvfp4(const void* A, const void* SFA, const void* B, const void* SFB, float ga, float gb, void* C,
               int out_type, int M, int N, int K, cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{});
int gen_w4a16(void* X, void* W, void* S, void* Z, int M, int N, int K, uint64_t seed, uint32_t tid0, cudaStream_t s);
uint64_t gemv_w4a16_workspace_bytes(int M, int N, int K, int sm_count);
// `chk.expect` (when set) is the golden output, compared word for word by the writer of each output.
// With `tickets` the split-K tickets live there (zero on entry, left zero) and the
// workspace holds only the rest (gemv_w4a16_workspace_bytes minus the tickets).
int gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int M, int N, int K,
               void* workspace, uint64_t workspace_bytes, cudaStream_t stream, unsigned int flags,
               const LaunchCheck& chk = LaunchCheck{}, unsigned int* tickets = nullptr);
int verify_words(const void* actual, const void* expected, uint64_t nwords, void* counters, void* log, int log_cap,
                 cudaStream_t s);
// Adds the digest of nwords 32-bit words (qg_verify.cu) to the uint64 at `out`.
int digest_words(const void* words, uint64_t nwords, uint64_t salt, void* out, cudaStream_t s);
int flip_bit(void* word, cudaStream_t s);
int flip_bit_at(void* base, uint64_t byte, int bit, cudaStream_t s);

} // namespace qg
