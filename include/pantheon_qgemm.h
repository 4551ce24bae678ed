/*
 * pantheon_qgemm.h -- C ABI of the B200-native quantized-GEMM stress workload.
 *
 * This library is what sits behind the `quantized_gemm` workload binary that
 * Pantheon's runner launches once per GPU.  The reference implementation of
 * that binary is the synthetic harness in
 *   kernels/quantized_gemm/quantized_gemm.cpp:1-2  (kind 3 of)
 *   kernels/common/ai_workload_template.h:351-380  (main: argv, warm-up,
 *                                                   timed loop, verify, exit)
 * and the entry points below replace, one for one, the pieces of that harness
 * (cited beside each declaration).  The process contract (argv in; the
 * "Throughput:" / "Verification:" lines and the exit code out) is kept by the
 * binary built from pantheon_b200/csrc/quantized_gemm_main.cpp on top of this
 * ABI.
 *
 * Conventions
 *   - Plain C types only.  Device pointers are `const void*` / `void*`; a CUDA
 *     stream is passed as `void*` (a cudaStream_t, NULL = legacy stream).
 *   - Every int-returning call returns QG_OK (0) on success, a negative value
 *     for a CUDA / argument error, and a positive value when a kernel's
 *     bounded wait expired (QG_ERR_DEVICE_TIMEOUT); the context is then still
 *     usable and qg_last_error() says where.  No call aborts the process.
 *   - Layouts are row-major with the contraction dimension K contiguous for
 *     both operands ("TN": A[M,K], B[N,K]), as the reference vendor GEMM uses
 *     (kernels/common/vendor_gemm.h:276-279,334-337).
 *   - Built for sm_100a only.  There is no CPU fallback: on a machine without
 *     a B200 every compute call fails with QG_ERR_CUDA.
 */
#ifndef PANTHEON_QGEMM_H
#define PANTHEON_QGEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QG_ABI_VERSION 1

#if defined(__GNUC__)
#define QG_API __attribute__((visibility("default")))
#else
#define QG_API
#endif

/* Return codes. */
#define QG_OK                  0
#define QG_ERR_ARG            -1   /* bad argument, unsupported shape or format */
#define QG_ERR_CUDA           -2   /* a CUDA runtime call failed (no device, OOM, fault) */
#define QG_ERR_UNSUPPORTED    -3   /* device is not sm_100 */
#define QG_ERR_DEVICE_TIMEOUT  1   /* a kernel's bounded mbarrier/TMEM wait expired */

/* Operand formats (the `--format` flag of the workload binary). */
#define QG_FMT_INT8   0   /* INT8 x INT8 -> INT32, fp32 per-row/per-col scales   */
#define QG_FMT_FP8    1   /* FP8 e4m3, 1x128 (A) and 128x128 (B) fp32 block scales */
#define QG_FMT_NVFP4  2   /* e2m1 + ue4m3 per 16 along K + fp32 per-tensor scale   */
#define QG_FMT_W4A16  3   /* bf16 activations x int4 weights, fp16 scale/zero per 128 */
/* Dense tensor-furnace formats (the mma_virus workload; C = A B^T, fp32 accumulate,
 * operands uniform on [-1, 1) rounded to the format). */
#define QG_FMT_BF16   4   /* bf16 x bf16 */
#define QG_FMT_FP16   5   /* fp16 x fp16 */
#define QG_FMT_TF32   6   /* tf32 x tf32 (stored as fp32 words) */
#define QG_FMT_E4M3   7   /* e4m3 x e4m3, unscaled */
#define QG_FMT_FP32   8   /* fp32 x fp32 on the CUDA cores (the furnace's fp32 type) */

/* Output element types. */
#define QG_OUT_BF16   0
#define QG_OUT_F32    1
#define QG_OUT_S32    2   /* raw INT32 accumulators (INT8 only) */
#define QG_OUT_F16    3   /* fp16 (dense formats only) */

/* Workload configuration for a context. Zero fields take the format default. */
typedef struct qg_cfg {
    int32_t  format;     /* QG_FMT_* */
    int32_t  m, n, k;    /* GEMM: C[m,n] = A[m,k] B[n,k]^T ; W4A16: Y[m,n] = X[m,k] W[k,n] */
    int32_t  out_type;   /* QG_OUT_BF16 (default) or QG_OUT_F32 */
    int32_t  copies;     /* rotating operand sets (>= 1); each has its own output and golden */
    uint64_t seed;       /* generator seed (tensor ids keep A and B on separate streams) */
} qg_cfg;

typedef struct qg_ctx qg_ctx;

/* One recorded verification mismatch (first few are kept, as the reference's
 * device fault log does: kernels/common/fault_log.h:36-50). */
typedef struct qg_mismatch {
    uint64_t index;      /* output word index */
    uint32_t expected;   /* golden word */
    uint32_t actual;     /* observed word */
} qg_mismatch;

/* ---------------------------------------------------------------- context API */

/* Allocate every device buffer of one workload instance on `device`.
 * Replaces: the cudaMalloc block of ai_workload_template.h:361-366 and the
 * working-set sizing at :359. */
QG_API int  qg_create(qg_ctx** out, int device, const qg_cfg* cfg);

/* Bytes of device memory a context with this configuration allocates
 * (used by the binary's --mem sizing). */
QG_API int  qg_required_bytes(const qg_cfg* cfg, uint64_t* bytes);

/* Fill all operand copies from the counter-based generator (after waiting for
 * all work on the device, so no launch still reads the old operands).
 * Replaces: ai_initialize (ai_workload_template.h:85-94) and
 *           pantheon_gemm_fill (kernels/common/vendor_gemm.h:184-191). */
QG_API int  qg_fill(qg_ctx* ctx, uint64_t seed);

/* Run every copy once and keep the outputs (and INT8 row checksums) as the
 * golden result of this run (after waiting for all work on the device, so no
 * earlier launch on another stream still writes the outputs).
 * Replaces: the golden GEMM + D2D copy of kernels/mma_virus/mma_virus.cpp:331-337. */
QG_API int  qg_golden(qg_ctx* ctx);

/* Launch `iters` GEMMs (or GEMVs), rotating over the operand copies, on `stream`.
 * After qg_golden every launch also checks itself (all formats but fp32): a GEMM
 * folds the output words of each row segment it stores (256 columns for INT8
 * and the dense tensor formats, 128 for FP8 and NVFP4; INT8 also folds its
 * INT32 accumulators) into a fingerprint and compares it with the one the
 * golden launch recorded; the GEMV compares every output word it writes with
 * the golden output (13-16 rows: per-column fingerprints, like the GEMMs).
 * Differences are counted on the device for qg_verify, so a corruption in any
 * launch of a batch is seen, not only in the last.  W4A16 launches after the
 * first pass QG_GEMV_WEIGHTS_CONST | QG_GEMV_ACTIVATIONS_CONST: the kernel
 * ahead is the previous GEMV, which writes neither.
 * Replaces: the ai_workload_kernel launch of the timed loop
 *           (ai_workload_template.h:370). Asynchronous. */
QG_API int  qg_run(qg_ctx* ctx, int iters, void* stream);

/* qg_run as a CUDA graph: the batch of `iters` launches is captured once per
 * (iters, the copy it starts at) from the context's own stream, instantiated,
 * and replayed on `stream` (NULL: the legacy default stream) with one
 * cudaGraphLaunch, so a batch costs the host one call however many launches
 * it holds.  Same launches, flags, checks and copy rotation as qg_run; the
 * captured batches are dropped by qg_fill and qg_golden.  Asynchronous.
 * Replaces: the timed batch of vendor_gemm.h:560-571 (launches between syncs). */
QG_API int  qg_run_graph(qg_ctx* ctx, int iters, void* stream);

/* Compare every copy's latest output (and checksums) with the golden result on
 * the device; `*mismatches` receives the number of differing 32-bit words plus
 * the differences the per-launch checks of qg_run counted since the previous
 * qg_verify (qg_verify_detail gives the two apart).
 * Replaces: ai_verify_output (ai_workload_template.h:343-349) and
 *           verify_mma_kernel (kernels/mma_virus/mma_virus.cpp:156-173). Synchronous. */
QG_API int  qg_verify(qg_ctx* ctx, uint64_t* mismatches);

/* The parts of the last qg_verify: differing output words of the final
 * compare, differences found by the per-launch checks (row segments of a GEMM,
 * output elements of the GEMV), and how many launches ran with a check.
 * Replaces: the error count of verify_mma_kernel (mma_virus.cpp:156-173), split by source. */
QG_API int  qg_verify_detail(const qg_ctx* ctx, uint64_t* words, uint64_t* launch_diffs,
                             uint64_t* launches_checked);

/* A 64-bit digest of copy `copy`'s golden result (after qg_golden): the sum
 * mod 2^64 of splitmix64(i * 0x9E3779B97F4A7C15 + w_i + salt) over the golden
 * output's 32-bit words w_i (salt 0, the output padded to whole words with
 * zeros) and, for INT8, its golden row checksums (salt 0xC2B2AE3D27D4EB4F).
 * Processes given the same format, shape, output type and seed compute the
 * same golden result on every healthy GPU, so the runner can compare the
 * digests of all GPUs of a run: a GPU whose digest differs from the others'
 * computed a wrong golden result (a silent data corruption that the per-GPU
 * compare against its own golden cannot see).  Synchronous.
 * Replaces: nothing in the reference (its golden never leaves the GPU); it
 * lets the runner compare the GPUs of one run with each other, with no
 * collective between them. */
QG_API int  qg_golden_digest(qg_ctx* ctx, int copy, uint64_t* digest);

/* Flip bit `bit` (0-7) of byte `byte` of operand `slot` (qg_tensor's slots
 * 0..3, or 0..3 of NVFP4's five) of copy `copy`, on `stream`, so the launches
 * that read it compute a wrong result; flipping it again restores the operand.
 * Used to show that the per-launch check catches a corruption in one launch of
 * a batch that later launches overwrite.
 * Replaces: the input corruption of --inject_error (ai_workload_template.h:90-92). */
QG_API int  qg_flip_operand_bit(qg_ctx* ctx, int copy, int slot, uint64_t byte, int bit, void* stream);

/* Copy out up to `cap` recorded mismatches of the last qg_verify; returns how many. */
QG_API int  qg_mismatch_log(qg_ctx* ctx, qg_mismatch* out, int cap);

/* Flip one bit of copy 0's output, so the next qg_verify must fail.
 * Replaces: --inject_error (ai_workload_template.h:90-92) and
 *           pantheon_gemm_flip_bit (kernels/common/vendor_gemm.h:193-195). */
QG_API int  qg_inject(qg_ctx* ctx);

/* Useful work of one launch: 2*M*N*K integer or floating-point operations
 * (GEMMs), or the algorithmic bytes moved (W4A16). */
QG_API double qg_ops_per_launch(const qg_ctx* ctx);
QG_API double qg_bytes_per_launch(const qg_ctx* ctx);

/* Copy the context's operands from / its output to HOST memory (pinned or
 * pageable), on `stream`; used for the end-to-end path.  The host layouts are
 * the device layouts described under the direct entry points below.
 * host_operands holds one pointer per operand of the format, in the order of
 * qg_tensor's slots: 2 for the dense formats (A, B), 4 for INT8 / FP8 (A, B,
 * sa, sb) and W4A16 (X, W, S, Z), 5 for NVFP4 (A, sfa, B, sfb, and the two
 * fp32 per-tensor scales, which the next launch of that copy uses). */
QG_API int  qg_upload(qg_ctx* ctx, int copy, const void* const* host_operands, void* stream);
QG_API int  qg_download(qg_ctx* ctx, int copy, void* host_out, void* stream);

/* Device pointers of copy `copy`'s tensors (for tests and the bench):
 * slot 0..4 = operands in the order of the direct entry point of the format,
 * slot 5 = output, slot 6 = golden output, slot 7 = row checksums. */
QG_API int  qg_tensor(qg_ctx* ctx, int copy, int slot, void** ptr, uint64_t* bytes);

/* Launch one GEMM (or GEMV) on copy `copy` (end-to-end path: qg_upload,
 * qg_run_copy, qg_download). Asynchronous.  No per-launch check: the operands
 * are the caller's, so the golden result need not apply to them. */
QG_API int  qg_run_copy(qg_ctx* ctx, int copy, void* stream);

/* Wait for all work on the context's device; returns QG_ERR_DEVICE_TIMEOUT if
 * a kernel's bounded wait expired. Replaces the per-launch hipDeviceSynchronize
 * of the timed loop (ai_workload_template.h:370). */
QG_API int  qg_synchronize(qg_ctx* ctx);

/* Free and total device memory of `device` (the --mem sizing input,
 * ai_workload_template.h:359). */
QG_API int  qg_mem_info(int device, uint64_t* free_bytes, uint64_t* total_bytes);

/* PCI bus id of `device` ("0000:1b:00.0"), for matching the device in NVML
 * (CUDA and NVML ordinals can differ).  Replaces: the cudaDeviceGetPCIBusId
 * call of the energy meter (kernels/common/vendor_gemm.h:383-404). */
QG_API int  qg_pci_bus_id(int device, char* buf, int len);

/* QG_ABI_VERSION of the loaded library. */
QG_API int  qg_abi_version(void);

/* Last error message of this context (or of the library when ctx is NULL). */
QG_API int  qg_last_error(const qg_ctx* ctx, char* buf, size_t len);

QG_API void qg_destroy(qg_ctx* ctx);

/* ---------------------------------------------------------------- direct entry points
 * Stateless kernels over caller-owned device memory (all asynchronous on `stream`).
 * They replace the per-kind body of ai_workload_kernel
 * (ai_workload_template.h:157-177, kind 3 "Quantized GEMM") with real GEMMs. */

/* INT8 W8A8:  C[m,n] = out( f32(sum_k A[m,k]*B[n,k]) * sa[m] * sb[n] )
 *   A int8 [M,K], B int8 [N,K] (K contiguous, K % 16 == 0), sa fp32 [M], sb fp32 [N];
 *   out_type QG_OUT_BF16 / QG_OUT_F32 / QG_OUT_S32 (raw accumulators, scales ignored).
 *   row_checksums (optional, uint32 [M]) receives
 *   sum_n (uint32)acc[m,n] * qg_cksum_weight(m,n)  (mod 2^32), a bit-exact
 *   fingerprint of the INT32 accumulators. */
QG_API int  qg_gemm_i8(const void* A, const void* B, const void* sa, const void* sb,
                void* C, int out_type, void* row_checksums,
                int M, int N, int K, void* stream);

/* Tensor-furnace GEMMs (the mma_virus workload): C = out(alpha * A B^T) with
 * fp32 accumulation on the tcgen05 tensor cores, A [M,K], B [N,K] K-contiguous;
 *   qg_gemm_bf16: bf16 operands (K % 8 == 0)
 *   qg_gemm_f16:  fp16 operands (K % 8 == 0)
 *   qg_gemm_tf32: fp32 words read as tf32 (the MMA uses the top 19 bits; K % 4 == 0)
 *   qg_gemm_e4m3: e4m3 bytes (K % 16 == 0)
 * out_type QG_OUT_BF16, QG_OUT_F16 or QG_OUT_F32.  M >= 256 runs on CTA pairs.
 * Replaces: the cuBLASLt bf16 / fp16 / tf32 / fp8 GEMMs of the tensor furnace
 *   (kernels/common/vendor_gemm.h:279-360, driven by kernels/mma_virus/mma_virus.cpp:264-282)
 *   and its WMMA fallback (mma_virus.cpp:57-135). */
QG_API int  qg_gemm_bf16(const void* A, const void* B, float alpha, void* C, int out_type,
                         int M, int N, int K, void* stream);
QG_API int  qg_gemm_f16(const void* A, const void* B, float alpha, void* C, int out_type,
                        int M, int N, int K, void* stream);
QG_API int  qg_gemm_tf32(const void* A, const void* B, float alpha, void* C, int out_type,
                         int M, int N, int K, void* stream);
QG_API int  qg_gemm_e4m3(const void* A, const void* B, float alpha, void* C, int out_type,
                         int M, int N, int K, void* stream);
/* The same product with fp32 operands on the CUDA cores (fp32 FMAs, no tf32
 * rounding): K % 4 == 0, A, B, C 16-byte aligned; out_type bf16, f16 or f32.
 * Replaces: cuBLASLt's SGEMM of the furnace's fp32 type
 *   (kernels/common/vendor_gemm.h:296-316, R_32F operands with COMPUTE_32F). */
QG_API int  qg_gemm_f32(const void* A, const void* B, float alpha, void* C, int out_type,
                        int M, int N, int K, void* stream);

/* FP8 e4m3 with fp32 block scales:
 *   C[m,n] = out( sum_kb P_kb[m,n] * sa[m,kb] * sb[n/128,kb] ),
 *   P_kb = sum over the 128-deep K block kb of A[m,k] B[n,k] (tensor cores, fp32),
 *   promoted in fp32 in K-block order as acc = fma(P_kb, sa*sb, acc).
 *   A e4m3 [M,K], B e4m3 [N,K] (K contiguous, K % 128 == 0); sa fp32 [M, K/128]
 *   (1x128 blocks), sb fp32 [ceil(N/128), K/128] (128x128 blocks);
 *   out_type QG_OUT_BF16 or QG_OUT_F32.
 * Replaces: the per-kind body of ai_workload_kernel (ai_workload_template.h:157-177);
 *   the reference's only FP8 GEMM is cuBLASLt e4m3 without block scales
 *   (kernels/common/vendor_gemm.h:311-327). */
QG_API int  qg_gemm_fp8_b128(const void* A, const void* B, const void* sa, const void* sb,
                             void* C, int out_type, int M, int N, int K, void* stream);

/* NVFP4: C[m,n] = out( ga*gb * sum_k (qa[m,k] sfa[m,k/16]) (qb[n,k] sfb[n,k/16]) ),
 *   tensor cores (tcgen05.mma kind::mxf4nvf4, block 16), fp32 accumulate.
 *   A, B: e2m1 codes packed two per byte along K (low nibble = even k),
 *   [M, K/2] and [N, K/2] bytes, K % 256 == 0.
 *   sfa, sfb: ue4m3 scale bytes (one per 16 elements along K) in the atom
 *   layout: one 512-byte atom per (128-row block, 64-element K chunk), atoms
 *   ordered [row block][K/64]; inside an atom row r's four scales are bytes
 *   (r%32)*16 + ((r/32)%4)*4 + 0..3 (qg_nvfp4_sf_bytes gives the size).
 *   ga, gb: per-tensor fp32 scales.  out_type QG_OUT_BF16 or QG_OUT_F32.
 * Replaces: the per-kind body of ai_workload_kernel (ai_workload_template.h:157-177)
 *   for configs[4]; the reference has no FP4 GEMM. */
QG_API int  qg_gemm_nvfp4(const void* A, const void* sfa, const void* B, const void* sfb,
                          float ga, float gb, void* C, int out_type, int M, int N, int K, void* stream);
QG_API int  qg_nvfp4_sf_bytes(int rows, int K, uint64_t* bytes);

/* W4A16 group-128 decode GEMV / skinny GEMM (1 row on the CUDA cores, 2-12
 * rows on warp MMAs, 13-16 rows on tcgen05, more rows in chunks of 16):
 *   Y[m,n] = sum_k X[m,k] * (q[k,n] - Z[k/128,n]) * S[k/128,n],  q = u - 8
 *   X bf16 [M,K]; W uint32 [K/8, N] with nibble j of word (k8, n) = u(8*k8+j, n)
 *   in [0,15]; S, Z fp16 [K/128, N]; Y bf16 or fp32 [M,N] (out_type).
 *   K % 128 == 0, N % 4 == 0; X, W, Y 16-byte and S, Z 8-byte aligned.
 *   `workspace` (qg_gemv_w4a16_workspace_bytes) holds the split-K partials,
 *   the tcgen05 path's quantised activations and the per-column-block
 *   tickets: it must be zero-filled before its first use, and every call
 *   leaves its tickets zero, ready for the next call (calls sharing one
 *   workspace must not overlap on the GPU).
 * Replaces: the decode kernel of the llm_decode path
 *   (kernels/llm_decode/llm_decode.cpp:28-46, a KV gather + FMA chain). */
QG_API int  qg_gemv_w4a16_workspace_bytes(int M, int N, int K, uint64_t* bytes);
QG_API int  qg_gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y,
                          int out_type, int M, int N, int K,
                          void* workspace, uint64_t workspace_bytes, void* stream);

/* qg_gemv_w4a16 with flags.  QG_GEMV_WEIGHTS_CONST: the kernel that precedes
 * this call on `stream` does not write W, S or Z (a decode loop over fixed
 * weights, e.g. the previous GEMV call); the 1-row and 2-12-row kernels then
 * issue their first weight loads before waiting for that kernel to finish,
 * overlapping the previous call's tail.  Other bits are rejected with
 * QG_ERR_ARG.
 * No counterpart in the reference. */
#define QG_GEMV_WEIGHTS_CONST 1u
/* QG_GEMV_ACTIVATIONS_CONST: the kernel that precedes this call on `stream`
 * does not write X (a loop of GEMVs over one activation set, such as the
 * workload's timed loop; not a decode step, whose X the layer before just
 * wrote).  The 2-12-row kernel then quantises its activations before waiting
 * for that kernel, overlapping the previous call's tail; the 13-16-row path's
 * pre-pass quantises them before its wait (and stores them after it); and the
 * 1-row kernel, when QG_GEMV_WEIGHTS_CONST is set too, stages its
 * activations, scales and zero points before the wait.  Either, both or
 * neither flag may be set. */
#define QG_GEMV_ACTIVATIONS_CONST 2u
QG_API int  qg_gemv_w4a16_ex(const void* X, const void* W, const void* S, const void* Z, void* Y,
                             int out_type, int M, int N, int K, void* workspace, uint64_t workspace_bytes,
                             unsigned int flags, void* stream);

/* qg_gemv_w4a16 without a caller-provided workspace, for callers that cannot
 * allocate device memory where they call it (a process whose device-memory
 * budget is already claimed, or a latency-critical decode path where an
 * allocation is not acceptable).  No counterpart in the reference.
 * Scratch comes from a 16 MiB array compiled into the library, which every GPU
 * that loads the library holds until the process exits: its first 256 KiB
 * hold the split-K tickets of every call, the rest the partial sums and
 * prepared activations.  Shapes whose workspace (qg_gemv_w4a16_workspace_bytes)
 * does not fit are rejected with QG_ERR_ARG (configs[3], M <= 16, K = 8192,
 * N = 28672, fits).  The call allocates nothing and clears nothing: every call
 * leaves its tickets zero, and everything else it reads it wrote first; the
 * first call on a device zeroes the ticket region once, on `stream`.  All
 * calls share the one array per device, so calls that overlap on the GPU
 * (other streams, other threads) race: serialise them.  The first call on a
 * device also looks up the array's device address; make that first call
 * before any stream capture. */
QG_API int  qg_gemv_w4a16_noalloc(const void* X, const void* W, const void* S, const void* Z, void* Y,
                                  int out_type, int M, int N, int K, void* stream);

/* Whether this library's kernels can run on `device`: QG_OK on an sm_100
 * (B200) device, QG_ERR_UNSUPPORTED on any other GPU (the message names its
 * architecture), QG_ERR_CUDA when there is no usable device.  The binaries
 * turn QG_ERR_UNSUPPORTED into the runner's deliberate skip ("Skipping:
 * <reason>" on stdout, exit 0).
 * Replaces: the platform checks before pantheon_skip (kernels/common/common.h:444-460). */
QG_API int  qg_device_check(int device);

/* Bounded-wait status of the most recent kernel on this device (QG_OK or
 * QG_ERR_DEVICE_TIMEOUT); clears the flag. Synchronous. */
QG_API int  qg_device_status(int device);

/* qg_device_status with its detail: `site` = (kernel id << 16) | wait site of
 * the first wait that gave up (0 = none), `waits_expired` = how many waits gave
 * up, `ctas_drained` = how many CTAs then let their copies and MMAs in flight
 * land, freed their TMEM and returned.  Any pointer may be NULL; clears all three.
 * Replaces: the CHECK / fault-log reporting of a kernel that failed
 *           (kernels/common/common.h:231-240, kernels/common/fault_log.h:36-50). */
QG_API int  qg_device_status_detail(int device, uint32_t* site, uint32_t* waits_expired,
                                    uint32_t* ctas_drained);

/* Fault drill of the bounded waits (no GPU fault, no hang): one INT8 GEMM
 * (bf16 out, M < 256, the single-CTA kernel) whose producers stop before K
 * block `withhold_kb` (< 4) of their first tile, with every wait limited to
 * `wait_ns` (1e5 .. 2e9 ns).  The wait for the withheld block expires; each CTA
 * records the site, drains and frees its TMEM and returns, so the call ends
 * after about `wait_ns` and qg_device_status_detail then reports
 * QG_ERR_DEVICE_TIMEOUT with ctas_drained = the grid's CTAs.  The device and
 * the process stay usable for the next launch.  For tests of the failure path.
 * No counterpart in the reference (its kernels have no bounded waits). */
QG_API int  qg_fault_drill_i8(const void* A, const void* B, const void* sa, const void* sb, void* C,
                              int M, int N, int K, uint64_t wait_ns, int withhold_kb, void* stream);

/* Compare two word arrays on the device.  `count` is a device uint64[2]:
 * count[0] += number of differing 32-bit words, count[1] += number of
 * differences seen for logging; the first `log_cap` differences are written to
 * `log` (device qg_mismatch array).  Arrays must be 16-byte aligned.
 * Replaces: ai_verify_output (ai_workload_template.h:343-349). */
QG_API int  qg_verify_words(const void* actual, const void* expected, uint64_t nwords,
                     void* count, void* log, int log_cap, void* stream);

/* Counter-based generator (identical arithmetic to the CPU restatement in the
 * test oracle): out[i] = uniform int8 in [-127,127] from (seed, tensor_id, i).
 * Replaces: ai_initialize's hash fill (ai_workload_template.h:85-94). */
QG_API int  qg_gen_i8(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream);
/* out[i] = lo + (hi-lo) * u(seed, tensor_id, i), fp32. */
QG_API int  qg_gen_uniform_f32(void* out, uint64_t n, float lo, float hi,
                        uint64_t seed, uint32_t tensor_id, void* stream);
/* out[i] = standard normal deviate (seed, tensor_id, i), fp32. */
QG_API int  qg_gen_normal_f32(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream);
/* Dense tensor-furnace operands (format QG_FMT_BF16 / FP16 / TF32 / E4M3 / FP32):
 * out[i] = fmt_rn(j / 32768 - 1), j = top 16 bits of hash(seed, tensor_id, i);
 * bf16 / fp16 / e4m3 (saturating) round to nearest even; tf32 is the fp32
 * word rounded to nearest even at 10 mantissa bits, low 13 bits zero; fp32
 * keeps the value as it is (exact).
 * Replaces: pantheon_gemm_fill (kernels/common/vendor_gemm.h:184-191), whose
 * operands are uniform on [-1, 1) in steps of 2^-15. */
QG_API int  qg_gen_dense(int format, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream);
/* FP8 operands of configs[2]: values N(0,1) (A: tensor tid0, B: tid0+2), each
 * block (A 1x128, B 128x128) scaled so its absmax maps to 448:
 * q = e4m3_rn_satfinite(x * (448/absmax)), scale = absmax/448 (fp32). */
QG_API int  qg_gen_fp8(void* A, void* sa, void* B, void* sb, int M, int N, int K,
                       uint64_t seed, uint32_t tid0, void* stream);
/* NVFP4 operands of configs[4]: values N(0,1) (A: tensor tid0, B: tid0+2);
 * per-tensor scale g = absmax/(448*6) -> gscales[0..1] (device fp32);
 * per 16 along K an ue4m3 scale sf = e4m3(blockmax/6/g); codes
 * q = e2m1(x / (sf*g)).  `work` is 8 bytes of device scratch. */
QG_API int  qg_gen_nvfp4(void* A, void* sfa, void* B, void* sfb, void* gscales, void* work,
                         int M, int N, int K, uint64_t seed, uint32_t tid0, void* stream);
/* W4A16 operands of configs[3]: X bf16 [M,K] = bf16(N(0,1)); W packed as in
 * qg_gemv_w4a16 with u uniform in [0,15] (q uniform in [-8,7]);
 * S fp16 = f16(U[0.005, 0.02]), Z fp16 = f16(U[-0.5, 0.5]) per (group, n).
 * Tensor ids: X = tid0, W = tid0+1, S = tid0+2, Z = tid0+3. */
QG_API int  qg_gen_w4a16(void* X, void* W, void* S, void* Z, int M, int N, int K,
                         uint64_t seed, uint32_t tid0, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PANTHEON_QGEMM_H */
