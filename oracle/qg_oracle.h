/*
 * qg_oracle.h -- CPU restatement of the quantized-GEMM workload's arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load this code, and only as the
 * checker or as the timed CPU baseline.  Nothing in pantheon_b200/ links,
 * loads or calls it.
 *
 * What it restates, and how it is pinned
 *   The reference (Pantheon 1.2.5) has no INT8/FP8/NVFP4/W4A16 arithmetic:
 *   kernels/quantized_gemm/quantized_gemm.cpp:1-2 selects kind 3 of the
 *   synthetic loop in kernels/common/ai_workload_template.h:157-177, an
 *   integer hash loop with no matrices.  Parity with the reference's NUMERICS
 *   is therefore unpinned; what the reference does pin is the workload
 *   contract (argv, output lines, exit codes, verify/inject semantics), and
 *   the tests pin that against the reference's MOCK binary built from its own
 *   sources (oracle/Makefile -> oracle/_ref/).
 *   The arithmetic here follows the formats' published definitions and the
 *   configuration text of the workload (INT8 exact INT32 accumulate with
 *   fp32 per-row/per-column scales; FP8 e4m3 with fp32 1x128 / 128x128 block
 *   scales promoted per 128-wide K block; NVFP4 e2m1 with ue4m3 scales per 16
 *   along K and an fp32 per-tensor scale; W4A16 int4 with fp16 scale and zero
 *   per group of 128 along K).  Its format conversions and integer GEMM are
 *   pinned against independent implementations (numpy integer matmul,
 *   torch's float8_e4m3fn / bfloat16 / float16 casts) by
 *   tests/golden/make_golden.py and tests/test_oracle.py.
 *   Conventions kept from the reference: TN layout with fp32 accumulate
 *   (kernels/common/vendor_gemm.h:276-279,334-337); golden computed once and
 *   compared bitwise (kernels/mma_virus/mma_virus.cpp:156-173,331-337).
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).  The
 * -ffp-contract=off flag matters: the fp32 expressions below are evaluated
 * one rounding at a time, the same way the CUDA kernels evaluate them with
 * __fmul_rn / __fadd_rn.
 */
#ifndef QG_ORACLE_H
#define QG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- counter-based generator (splitmix64, Steele/Lea/Flood 2014) ---------- */
uint64_t qgo_splitmix64(uint64_t z);
uint64_t qgo_hash64(uint64_t seed, uint32_t tensor_id, uint64_t index);
int8_t   qgo_i8_from_hash(uint64_t h);
float    qgo_uniform_from_hash(uint64_t h, float lo, float hi);
float    qgo_normal_from_hash(uint64_t h);
float    qgo_logf(float x);

void qgo_gen_i8(int8_t* out, uint64_t n, uint64_t seed, uint32_t tensor_id);
void qgo_gen_uniform_f32(float* out, uint64_t n, float lo, float hi, uint64_t seed, uint32_t tensor_id);
void qgo_gen_normal_f32(float* out, uint64_t n, uint64_t seed, uint32_t tensor_id);

/* ---- format conversions (round to nearest even) -------------------------- */
uint16_t qgo_f32_to_bf16(float x);
float    qgo_bf16_to_f32(uint16_t b);
uint16_t qgo_f32_to_f16(float x);
float    qgo_f16_to_f32(uint16_t h);
uint8_t  qgo_f32_to_e4m3(float x);          /* satfinite: |x| > 448 -> +-448 */
float    qgo_e4m3_to_f32(uint8_t v);
uint8_t  qgo_f32_to_e2m1(float x);          /* 4-bit code, satfinite at +-6 */
float    qgo_e2m1_to_f32(uint8_t v);

/* ---- INT8 W8A8 ----------------------------------------------------------- */
uint32_t qgo_cksum_weight(uint32_t m, uint32_t n);

/* Rows `rows[0..nrows)` (all rows when rows == NULL, nrows == M) of
 * C = out(f32(acc) * sa[m] * sb[n]).  C is indexed by the row's position in
 * `rows` (compact); acc (optional) receives the INT32 accumulators, row_cksum
 * (optional) the per-row checksum. out_type 0 = bf16 (uint16), 1 = f32, 2 = s32. */
void qgo_gemm_i8(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                 int M, int N, int K, const int32_t* rows, int nrows,
                 int out_type, void* C, int32_t* acc, uint32_t* row_cksum);

/* ---- FP8 e4m3 with 1x128 (A) / 128x128 (B) fp32 block scales ------------- */
void qgo_quant_fp8_rows(const float* X, int R, int K, uint8_t* Q, float* S);     /* S[R, K/128] */
void qgo_quant_fp8_blocks(const float* X, int R, int K, uint8_t* Q, float* S);   /* S[R/128, K/128] */
void qgo_gemm_fp8_b128(const uint8_t* A, const uint8_t* B, const float* sa, const float* sb,
                       int M, int N, int K, const int32_t* rows, int nrows,
                       int out_type, void* C);

/* ---- NVFP4 ----------------------------------------------------------------
 * Q packed two codes per byte along K (low nibble = even k), SF ue4m3 [R, K/16]
 * (row-major, plain layout), G = per-tensor fp32 scale. */
float qgo_nvfp4_global_scale(const float* X, uint64_t n);
void  qgo_quant_nvfp4(const float* X, int R, int K, float G, uint8_t* Q, uint8_t* SF);
void  qgo_gemm_nvfp4(const uint8_t* A, const uint8_t* SFA, float GA,
                     const uint8_t* B, const uint8_t* SFB, float GB,
                     int M, int N, int K, const int32_t* rows, int nrows,
                     int out_type, void* C);

/* ---- W4A16 GEMV / skinny GEMM ---------------------------------------------
 * X bf16 [M,K]; W packed uint32 [K/8, N] (nibble j of word (k/8, n) is
 * code u(k=8*(k/8)+j, n), value q = u - 8); S, Z fp16 [K/128, N];
 * Y[m,n] = sum_k X[m,k] * (q[k,n] - Z[k/128,n]) * S[k/128,n]. */
void qgo_gen_w4a16(uint16_t* X, uint32_t* W, uint16_t* S, uint16_t* Z, int M, int N, int K,
                   uint64_t seed, uint32_t tid0);
void qgo_gemv_w4a16(const uint16_t* X, const uint32_t* W, const uint16_t* S, const uint16_t* Z,
                    int M, int N, int K, const int32_t* cols, int ncols,
                    int out_type, void* Y);

/* ---- verification ---------------------------------------------------------- */
uint64_t qgo_count_mismatch_u32(const uint32_t* a, const uint32_t* b, uint64_t n);
/* max over i of |y_i - r_i| / max(|r_i|, rms(r)) for bf16 (kind 0) or f32 (kind 1) arrays */
double   qgo_max_rel_err(const void* y, const void* r, uint64_t n, int kind);

/* number of OpenMP threads the oracle uses */
int qgo_threads(void);
void qgo_set_threads(int n);

/* ---- tensor-furnace (dense) GEMMs ------------------------------------------ */
#define QGO_FMT_BF16 4
#define QGO_FMT_FP16 5
#define QGO_FMT_TF32 6
#define QGO_FMT_E4M3 7
#define QGO_FMT_FP32 8
uint32_t qgo_f32_to_tf32_bits(float x);   /* nearest even at 10 mantissa bits, low 13 bits zero */
float    qgo_dense_value(uint64_t h);     /* j / 32768 - 1, j = h >> 48 */
void     qgo_gen_dense(int fmt, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id);
/* kind 1 bf16, 2 e4m3, 3 fp16, 4 tf32 (fp32 words), 5 fp32; out_type 0 bf16, 1 f32, 3 fp16 */
void qgo_gemm_dense(int kind, const void* A, const void* B, float alpha, int M, int N, int K,
                    const int32_t* rows, int nrows, int out_type, void* C);

#ifdef __cplusplus
}
#endif
#endif
