// qg_gemm_i8.cu -- INT8 x INT8 -> INT32 GEMM on the sm_100a tensor cores
// (tcgen05.mma kind::i8), with the fp32 per-row / per-column dequant epilogue.
//
// Replaces the body of the reference's "Quantized GEMM" workload kernel
// (kernels/common/ai_workload_template.h:157-177, kind 3), which is a synthetic
// integer hash loop, with the GEMM the workload is named after:
//     C[m,n] = out( f32(sum_k A[m,k] B[n,k]) * sa[m] * sb[n] )
//
// Structure (one persistent CTA per SM, 256 threads):
//   warp 0      TMA producer: A 128x128 and B 256x128 int8 tiles per stage,
//               128-byte swizzled, into a 4-stage shared-memory ring.
//   warp 1      MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=32) per stage
//               into a TMEM accumulator; tcgen05.commit frees the stage.
//   warp 2      TMEM allocator (512 columns = two 128x256 s32 accumulators,
//               so the epilogue of tile i overlaps the mainloop of tile i+1).
//   warps 4-7   epilogue: tcgen05.ld 32 columns at a time, convert, scale,
//               round, store, and fold the INT32 accumulators into a per-row
//               checksum (a bit-exact fingerprint of the integer result).
// Every barrier wait is bounded (qg_ptx.cuh); on expiry the kernel records
// the site in the device status word, drains its in-flight copies and MMAs,
// frees TMEM and returns.
#include "qg_common.cuh"
#include "qg_check.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qg {
namespace i8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;            // bytes of K per stage = one 128-byte swizzle row (128 int8 / 64 bf16)
constexpr int UMMA_K = 32;         // bytes of K per tcgen05.mma (32 int8 / 16 bf16 / 32 e4m3)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;   // 16 KB
constexpr int B_BYTES = BN * BK;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = BN;       // s32 accumulator columns per buffer
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int THREADS = 256;
constexpr int EPI_WARP0 = 4;

// Operand kinds these kernels run.  The mainloops are the same for all of
// them (128-byte K rows per stage, 32-byte K steps per MMA: 32 int8 / 16
// bf16 or fp16 / 8 tf32 / 32 e4m3 elements); the MMA instruction, its
// descriptor and the epilogue differ.
//   KIND_I8    s8 x s8 -> s32, epilogue f32(acc) * sa[m] * sb[n], row checksums
//   KIND_BF16  bf16 x bf16 -> f32, epilogue acc * alpha          (tensor furnace)
//   KIND_E4M3  e4m3 x e4m3 -> f32, epilogue acc * alpha          (tensor furnace)
//   KIND_F16   fp16 x fp16 -> f32, epilogue acc * alpha          (tensor furnace)
//   KIND_TF32  tf32 x tf32 -> f32, epilogue acc * alpha          (tensor furnace;
//              operands are fp32 words, the MMA reads their top 19 bits)
enum : int { KIND_I8 = 0, KIND_BF16 = 1, KIND_E4M3 = 2, KIND_F16 = 3, KIND_TF32 = 4 };
__host__ __device__ constexpr int elem_bytes(int kind) {
    return (kind == KIND_BF16 || kind == KIND_F16) ? 2 : kind == KIND_TF32 ? 4 : 1;
}
// Tile rasterisation: consecutive tiles walk group_m row-tiles (sharing B tiles
// in L2) before moving to the next columns.  Measured at 8192^3 on the pair
// kernel (DRAM bytes read per launch): INT8 16 / 8 / 32 row-tiles 222 / 337 /
// 652 MB; BF16 8 / 16 / 4 / 32 row-tiles 1.09 / 1.25 / 1.44 / 2.05 GB, and 8
// was also the fastest for the 2-byte kinds.  TF32 (4-byte rows, a slower MMA)
// ran faster at 16 than at 4 (709 against 668 TFLOP/s).
__host__ __device__ constexpr int group_m(int kind) { return elem_bytes(kind) == 2 ? 8 : 16; }
__host__ __device__ constexpr uint32_t kind_idesc(int kind, uint32_t M, uint32_t N) {
    return kind == KIND_I8     ? make_idesc(/*s32*/ 2, /*s8*/ 1, /*s8*/ 1, M, N)
           : kind == KIND_BF16 ? make_idesc(/*f32*/ 1, /*bf16*/ 1, /*bf16*/ 1, M, N)
           : kind == KIND_F16  ? make_idesc(/*f32*/ 1, /*f16*/ 0, /*f16*/ 0, M, N)
           : kind == KIND_TF32 ? make_idesc(/*f32*/ 1, /*tf32*/ 2, /*tf32*/ 2, M, N)
                               : make_idesc(/*f32*/ 1, /*e4m3*/ 0, /*e4m3*/ 0, M, N);
}
template <int KIND>
__device__ __forceinline__ void umma_kind(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if constexpr (KIND == KIND_I8) umma_i8(d, a, b, idesc, acc);
    else if constexpr (KIND == KIND_BF16 || KIND == KIND_F16) umma_f16(d, a, b, idesc, acc);
    else if constexpr (KIND == KIND_TF32) umma_tf32(d, a, b, idesc, acc);
    else umma_f8(d, a, b, idesc, acc);
}
template <int KIND>
__device__ __forceinline__ void umma_kind_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if constexpr (KIND == KIND_I8) umma_i8_pair(d, a, b, idesc, acc);
    else if constexpr (KIND == KIND_BF16 || KIND == KIND_F16) umma_f16_pair(d, a, b, idesc, acc);
    else if constexpr (KIND == KIND_TF32) umma_tf32_pair(d, a, b, idesc, acc);
    else umma_f8_pair(d, a, b, idesc, acc);
}

// Barrier block that follows the operand ring in shared memory.
struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

// Status sites: kernel id 1 (INT8 GEMM) in the high half.
constexpr uint32_t SITE_PRODUCER = 0x00010001u;
constexpr uint32_t SITE_MMA_FULL = 0x00010002u;
constexpr uint32_t SITE_MMA_TMEM = 0x00010003u;
constexpr uint32_t SITE_EPI = 0x00010004u;

struct Params {
    int M, N, K;
    const float* sa;
    const float* sb;
    void* C;
    uint32_t* row_cksum;
    DeviceStatus* status;
    float alpha;            // output scale of the f32-accumulating kinds
    LaunchCheck chk;        // per-launch check: one fingerprint per (row, 256-column tile)
    // Fault drill (qg_fault_drill_i8, single-CTA kernel only): every bounded wait
    // gives up after wait_ns, and the producer of each CTA stops before the
    // withhold_kb-th K block of its first tile, so the MMA's wait for it expires.
    uint64_t wait_ns = QG_WAIT_LIMIT_NS;
    int withhold_kb = -1;
};

// Fingerprint slot of row m, column tile nt (qg_check.cuh).
__device__ __forceinline__ uint64_t seg_index(int m, int nt, int N) {
    return (uint64_t)m * (uint64_t)((N + BN - 1) / BN) + (uint64_t)nt;
}

template <int GROUP_M>
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
    const int group = GROUP_M * tiles_n;
    const int g = t / group;
    const int first_m = g * GROUP_M;
    const int gm = min(tiles_m - first_m, GROUP_M);
    const int r = t - g * group;
    mt = first_m + r % gm;
    nt = r / gm;
}

__device__ __forceinline__ uint32_t cksum_weight(uint32_t m, uint32_t n) {
    return (m * 0x9E3779B1u + n * 0x85EBCA77u) | 1u;
}

// One 32-column chunk of an accumulator row: checksum fold, then the s32 /
// dequantised f32 / bf16 store (ragged edges handled per element).
// `fold` (uniform: a golden or checked launch) adds every stored output word,
// times its odd weight, to `ofp`; the INT8 kind then also folds its
// accumulators into `ck` (the row checksum's fold) even without row checksums.
template <int KIND, int OUT>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], int m, int n0, bool row_ok, float sam,
                                               const Params& p, uint32_t& ck, bool fold, uint32_t& ofp) {
    if (!row_ok || n0 >= p.N) return;
    const bool full_chunk = (n0 + 32 <= p.N);
    if (KIND == KIND_I8 && (p.row_cksum || fold)) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (full_chunk || n0 + i < p.N) ck += r[i] * cksum_weight((uint32_t)m, (uint32_t)(n0 + i));
    }
    if (OUT == QG_OUT_S32) {
        int32_t* dst = static_cast<int32_t*>(p.C) + (size_t)m * p.N + n0;
        if (full_chunk && (p.N % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<uint4*>(dst + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) dst[i] = (int32_t)r[i];
        }
        if (fold) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (full_chunk || n0 + i < p.N) ofp = ofp * kCheckMul + r[i];
        }
        return;
    }
    float f[32];
    if constexpr (KIND != KIND_I8) {
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __fmul_rn(__uint_as_float(r[i]), p.alpha);
    } else if (full_chunk) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + i));
            f[i + 0] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[i + 0]), sam), s4.x);
            f[i + 1] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[i + 1]), sam), s4.y);
            f[i + 2] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[i + 2]), sam), s4.z);
            f[i + 3] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[i + 3]), sam), s4.w);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float sbn = (n0 + i < p.N) ? __ldg(p.sb + n0 + i) : 0.0f;
            f[i] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[i]), sam), sbn);
        }
    }
    if (OUT == QG_OUT_F32) {
        float* dst = static_cast<float*>(p.C) + (size_t)m * p.N + n0;
        if (full_chunk && (p.N % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) dst[i] = f[i];
        }
        if (fold) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (full_chunk || n0 + i < p.N) ofp = ofp * kCheckMul + __float_as_uint(f[i]);
        }
    } else if (OUT == QG_OUT_F16) {
        __half* dst = static_cast<__half*>(p.C) + (size_t)m * p.N + n0;
        if (full_chunk && (p.N % 8) == 0) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
#pragma unroll
            for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<uint4*>(dst + 2 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
            if (fold) {
#pragma unroll
                for (int i = 0; i < 16; ++i) ofp = ofp * kCheckMul + w[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) {
                    const __half h = __float2half_rn(f[i]);
                    dst[i] = h;
                    if (fold) ofp = ofp * kCheckMul + (uint32_t)__half_as_ushort(h);
                }
        }
    } else {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.C) + (size_t)m * p.N + n0;
        if (full_chunk && (p.N % 8) == 0) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
#pragma unroll
            for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<uint4*>(dst + 2 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
            if (fold) {
#pragma unroll
                for (int i = 0; i < 16; ++i) ofp = ofp * kCheckMul + w[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(f[i]);
                    dst[i] = h;
                    if (fold) ofp = ofp * kCheckMul + (uint32_t)__bfloat16_as_ushort(h);
                }
        }
    }
}

template <int KIND, int OUT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment: the 128-byte swizzle pattern is a function of the
    // address bits, and the UMMA descriptors assume base offset 0.
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tiles_m = (p.M + BM - 1) / BM;
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int nk = (p.K * elem_bytes(KIND) + BK - 1) / BK;   // 128-byte K blocks

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&bars->full[s], 1); mbar_init(&bars->empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&bars->tmem_full[a], 1); mbar_init(&bars->tmem_empty[a], 4 * 32); }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort_flag = &bars->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ producer
        uint32_t stage = 0, phase = 0;
        uint32_t armed = 0, armed_phase = 0;   // bitmasks over stages, for the abort drain
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            for (int kb = 0; kb < nk; ++kb) {
                if (kb == p.withhold_kb && t == (int)blockIdx.x) { ok = false; break; }   // fault drill only
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PRODUCER, p.wait_ns)) { ok = false; break; }
                mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
                tma_load_2d(sA + stage * A_BYTES, &tmA, &bars->full[stage], kb * BK, mt * BM);
                tma_load_2d(sB + stage * B_BYTES, &tmB, &bars->full[stage], kb * BK, nt * BN);
                armed |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok) {
            // Let every copy already issued land before the CTA's shared memory goes away.
            for (int s = 0; s < STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t IDESC = kind_idesc(KIND, BM, BN);
        uint32_t stage = 0, phase = 0;
        bool ok = true, issued = false;
        int iter = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++iter) {
            const uint32_t acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            if (!mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.status, SITE_MMA_TMEM, p.wait_ns)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_MMA_FULL, p.wait_ns)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
                const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k) {
                    const uint64_t ad = make_sdesc_kmajor_sw128(a_addr + k * UMMA_K);
                    const uint64_t bd = make_sdesc_kmajor_sw128(b_addr + k * UMMA_K);
                    umma_kind<KIND>(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
                }
                issued = true;
                umma_commit(&bars->empty[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) umma_commit(&bars->tmem_full[acc]);
        }
        if (!ok && issued) {
            // Wait for the MMAs already in flight before TMEM is released.
            umma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - EPI_WARP0;               // TMEM lane quarter of this warp
        const int row = ew * 32 + lane;
        const bool fold = p.chk.record != nullptr || p.chk.expect != nullptr;
        int iter = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++iter) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            const uint32_t acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&bars->tmem_full[acc], acc_phase, abort_flag, p.status, SITE_EPI, p.wait_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();

            const int m = mt * BM + row;
            const bool row_ok = m < p.M;
            const float sam = (KIND == KIND_I8 && OUT != QG_OUT_S32 && row_ok) ? __ldg(p.sa + m) : 0.0f;
            uint32_t ck = 0, ofp = 0;
            const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + acc * ACC_COLS;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait_regs(r);
                epilogue_chunk<KIND, OUT>(r, m, nt * BN + c, row_ok, sam, p, ck, fold, ofp);
            }
            tc_fence_before();
            mbar_arrive(&bars->tmem_empty[acc]);
            if (p.row_cksum && row_ok) atomicAdd(p.row_cksum + m, ck);
            if (fold) check_segment(p.chk, row_ok, seg_index(m, nt, p.N), ck + ofp);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
        if (lane == 0 && *abort_flag) atomicAdd(&p.status->drained, 1u);   // gave up, drained, TMEM freed
    }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (M >= 256): a cluster of two CTAs computes 256x256 tiles
// with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32) issued by the even
// CTA.  Each CTA loads its own 128 rows of A and its own 128 rows (half) of B
// per K block, 32 KB instead of the single-CTA kernel's 48 KB, which relieves
// the operand stream into shared memory that bounds the single-CTA kernel;
// each CTA's TMEM holds its 128 rows of the 256-column accumulator and its
// epilogue is the single-CTA one.  Protocol:
//   * both CTAs' copies complete on the even CTA's `full` barrier (the even
//     producer arms it with both CTAs' bytes); the odd producer paces itself
//     on its own `empty` barrier;
//   * the MMA thread commits `empty` and `tmem_full` to both CTAs (one plain
//     commit per CTA, no multicast);
//   * each epilogue warp of either CTA arrives on the even CTA's `tmem_empty`;
//   * TMEM is allocated and freed by warp 2 of both CTAs (cta_group::2), and a
//     cluster barrier keeps both CTAs alive until the last MMA has landed.
constexpr int P_STAGES = 6;
constexpr int PA_BYTES = BM * BK;                 // 16 KB: this CTA's A rows
constexpr int PB_BYTES = (BN / 2) * BK;           // 16 KB: this CTA's half of B
constexpr int P_STAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
constexpr int P_EPI_WARPS = 4;

template <int KIND, int OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + P_STAGES * PA_BYTES;
    struct PBarriers {
        uint64_t full[P_STAGES];
        uint64_t empty[P_STAGES];
        uint64_t tmem_full[2];
        uint64_t tmem_empty[2];
        uint64_t drain;
        uint32_t tmem_base;
        int abort;
    };
    PBarriers* bars = reinterpret_cast<PBarriers*>(smem + P_STAGES * P_STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int nk = (p.K * elem_bytes(KIND) + BK - 1) / BK;   // 128-byte K blocks
    const int pair = blockIdx.x >> 1;
    const int pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) { mbar_init(&bars->full[s], 1); mbar_init(&bars->empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&bars->tmem_full[a], 1); mbar_init(&bars->tmem_empty[a], 2 * P_EPI_WARPS); }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 2) {
        tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    // both CTAs' barriers initialised and TMEM allocated before anyone signals the other
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort_flag = &bars->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        uint32_t stage = 0, phase = 0;
        uint32_t armed = 0, armed_phase = 0;
        bool ok = true;
        for (int t = pair; t < tiles && ok; t += pairs) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PRODUCER, p.wait_ns)) { ok = false; break; }
                if (leader) mbar_arrive_expect_tx(&bars->full[stage], 2 * P_STAGE_BYTES);
                const uint32_t full_leader = mapa_shared(smem_u32(&bars->full[stage]), 0);
                tma_load_2d_pair(sA + stage * PA_BYTES, &tmA, full_leader, kb * BK, mt * 2 * BM + (int)rank * BM);
                tma_load_2d_pair(sB + stage * PB_BYTES, &tmB, full_leader, kb * BK, nt * BN + (int)rank * (BN / 2));
                armed |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok && leader) {
            // copies of both CTAs complete on these barriers: let them land
            for (int s = 0; s < P_STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        constexpr uint32_t IDESC = kind_idesc(KIND, 2 * BM, BN);
        uint32_t stage = 0, phase = 0;
        bool ok = true, issued = false;
        int iter = 0;
        for (int t = pair; t < tiles && ok; t += pairs, ++iter) {
            const uint32_t acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            if (!mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.status, SITE_MMA_TMEM, p.wait_ns)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_MMA_FULL, p.wait_ns)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + stage * PA_BYTES);
                const uint32_t b_addr = smem_u32(sB + stage * PB_BYTES);
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k)
                    umma_kind_pair<KIND>(d_tmem, make_sdesc_kmajor_sw128(a_addr + k * UMMA_K),
                                         make_sdesc_kmajor_sw128(b_addr + k * UMMA_K), IDESC, (kb | k) != 0 ? 1u : 0u);
                issued = true;
                const uint32_t e = smem_u32(&bars->empty[stage]);
                umma_commit_pair(mapa_shared(e, 0));
                umma_commit_pair(mapa_shared(e, 1));
                if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) {
                const uint32_t f = smem_u32(&bars->tmem_full[acc]);
                umma_commit_pair(mapa_shared(f, 0));
                umma_commit_pair(mapa_shared(f, 1));
            }
        }
        if (!ok && issued) {
            umma_commit_pair(mapa_shared(smem_u32(&bars->drain), 0));
            mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - EPI_WARP0;
        const int row = ew * 32 + lane;
        const bool fold = p.chk.record != nullptr || p.chk.expect != nullptr;
        int iter = 0;
        for (int t = pair; t < tiles; t += pairs, ++iter) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            const uint32_t acc = iter & 1;
            const uint32_t acc_phase = (iter >> 1) & 1;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&bars->tmem_full[acc], acc_phase, abort_flag, p.status, SITE_EPI, p.wait_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const int m = mt * 2 * BM + (int)rank * BM + row;
            const bool row_ok = m < p.M;
            const float sam = (KIND == KIND_I8 && OUT != QG_OUT_S32 && row_ok) ? __ldg(p.sa + m) : 0.0f;
            uint32_t ck = 0, ofp = 0;
            const uint32_t t_row = tmem_base + ((uint32_t)(ew * 32) << 16) + acc * ACC_COLS;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait_regs(r);
                epilogue_chunk<KIND, OUT>(r, m, nt * BN + c, row_ok, sam, p, ck, fold, ofp);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars->tmem_empty[acc]), 0));
            if (p.row_cksum && row_ok) atomicAdd(p.row_cksum + m, ck);
            if (fold) check_segment(p.chk, row_ok, seg_index(m, nt, p.N), ck + ofp);
        }
    }

    // the even CTA's MMAs read this CTA's shared memory and write its TMEM:
    // neither CTA frees anything before both are done
    tc_fence_before();
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
        if (lane == 0 && *abort_flag) atomicAdd(&p.status->drained, 1u);   // gave up, drained, TMEM freed
    }
}

// ---------------------------------------------------------------------------
// Wide CTA-pair variant (M >= 256, N > 256, 2- and 4-byte kinds): a cluster of two CTAs computes
// 256x512 tiles as two 256-column halves, each half one tcgen05.mma
// .cta_group::2 (M = 256, N = 256, K = 32) per K step into its own 256 TMEM
// columns.  Per K block each CTA loads its 128 rows of A and its 128 rows of
// each half of B: 48 KB for 128 x 512 x 128 products, a quarter fewer bytes
// per product than the 256x256 pair tile (32 KB for 128 x 256 x 128).  The
// operand stream into shared memory is what bounds the 256x256 kernel: with
// B's loads left out (a timing copy, wrong results) it ran 12 % faster at the
// maximum clock and 15 % faster under the power cap, with no loads at all
// 21 %.  The accumulator now fills TMEM (512 columns), so there is no second
// buffer: the epilogue drains the two halves in parallel (warps 4-7 columns
// 0-255, warps 8-11 columns 256-511) and releases each on its own barrier,
// and the next tile's first MMA into a half waits only for that half.
// Protocol otherwise as the 256x256 pair kernel's.
constexpr int W_BN = 2 * BN;                        // 512 tile columns
constexpr int W_STAGES = 4;
constexpr int WA_BYTES = BM * BK;                   // 16 KB: this CTA's A rows
constexpr int WB_HALF = (BN / 2) * BK;              // 16 KB: its 128 rows of one half of B
constexpr int WB_BYTES = 2 * WB_HALF;
constexpr int W_STAGE_BYTES = WA_BYTES + WB_BYTES;  // 48 KB
constexpr int W_SMEM_BYTES = W_STAGES * W_STAGE_BYTES + 1024 + 256;
constexpr int W_EPI_WARPS = 8;
constexpr int W_THREADS = (EPI_WARP0 + W_EPI_WARPS) * 32;   // 384

template <int KIND, int OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W_THREADS, 1)
gemm_i8_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + W_STAGES * WA_BYTES;
    struct WBarriers {
        uint64_t full[W_STAGES];
        uint64_t empty[W_STAGES];
        uint64_t acc_full;
        uint64_t acc_empty[2];   // per 256-column half
        uint64_t drain;
        uint32_t tmem_base;
        int abort;
    };
    WBarriers* bars = reinterpret_cast<WBarriers*>(smem + W_STAGES * W_STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
    const int tiles_n = (p.N + W_BN - 1) / W_BN;
    const int tiles = tiles_m * tiles_n;
    const int nk = (p.K * elem_bytes(KIND) + BK - 1) / BK;   // 128-byte K blocks
    const int pair = blockIdx.x >> 1;
    const int pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < W_STAGES; ++s) { mbar_init(&bars->full[s], 1); mbar_init(&bars->empty[s], 1); }
        mbar_init(&bars->acc_full, 1);
        for (int h = 0; h < 2; ++h) mbar_init(&bars->acc_empty[h], 2 * (W_EPI_WARPS / 2));
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 2) {
        tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort_flag = &bars->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        uint32_t stage = 0, phase = 0;
        uint32_t armed = 0, armed_phase = 0;
        bool ok = true;
        for (int t = pair; t < tiles && ok; t += pairs) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PRODUCER, p.wait_ns)) { ok = false; break; }
                if (leader) mbar_arrive_expect_tx(&bars->full[stage], 2 * W_STAGE_BYTES);
                const uint32_t full_leader = mapa_shared(smem_u32(&bars->full[stage]), 0);
                tma_load_2d_pair(sA + stage * WA_BYTES, &tmA, full_leader, kb * BK, mt * 2 * BM + (int)rank * BM);
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    tma_load_2d_pair(sB + stage * WB_BYTES + h * WB_HALF, &tmB, full_leader, kb * BK,
                                     nt * W_BN + h * BN + (int)rank * (BN / 2));
                armed |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok && leader) {
            // copies of both CTAs complete on these barriers: let them land
            for (int s = 0; s < W_STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        constexpr uint32_t IDESC = kind_idesc(KIND, 2 * BM, BN);
        uint32_t stage = 0, phase = 0;
        bool ok = true, issued = false;
        int iter = 0;
        for (int t = pair; t < tiles && ok; t += pairs, ++iter) {
            const uint32_t acc_phase = iter & 1;
            for (int kb = 0; kb < nk && ok; ++kb) {
                if (!mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_MMA_FULL, p.wait_ns)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + stage * WA_BYTES);
                const uint32_t b_addr = smem_u32(sB + stage * WB_BYTES);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (kb == 0) {   // this half of the accumulator drained by the previous tile's epilogue
                        if (!mbar_wait(&bars->acc_empty[h], acc_phase ^ 1u, abort_flag, p.status, SITE_MMA_TMEM, p.wait_ns)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_kind_pair<KIND>(tmem_base + h * BN, make_sdesc_kmajor_sw128(a_addr + k * UMMA_K),
                                             make_sdesc_kmajor_sw128(b_addr + h * WB_HALF + k * UMMA_K), IDESC,
                                             (kb | k) != 0 ? 1u : 0u);
                    issued = true;
                }
                if (!ok) break;
                const uint32_t e = smem_u32(&bars->empty[stage]);
                umma_commit_pair(mapa_shared(e, 0));
                umma_commit_pair(mapa_shared(e, 1));
                if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) {
                const uint32_t f = smem_u32(&bars->acc_full);
                umma_commit_pair(mapa_shared(f, 0));
                umma_commit_pair(mapa_shared(f, 1));
            }
        }
        if (!ok && issued) {
            umma_commit_pair(mapa_shared(smem_u32(&bars->drain), 0));
            mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - EPI_WARP0;
        const int h = ew >> 2;                  // column half
        const int q = warp & 3;                 // TMEM lane quarter (a warp reaches lanes 32 (warp % 4) ..)
        const int row = q * 32 + lane;
        const bool fold = p.chk.record != nullptr || p.chk.expect != nullptr;
        int iter = 0;
        for (int t = pair; t < tiles; t += pairs, ++iter) {
            int mt, nt;
            tile_coords<group_m(KIND)>(t, tiles_m, tiles_n, mt, nt);
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&bars->acc_full, iter & 1, abort_flag, p.status, SITE_EPI, p.wait_ns) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const int m = mt * 2 * BM + (int)rank * BM + row;
            const bool row_ok = m < p.M;
            const int n0 = nt * W_BN + h * BN;
            const float sam = (KIND == KIND_I8 && OUT != QG_OUT_S32 && row_ok) ? __ldg(p.sa + m) : 0.0f;
            uint32_t ck = 0, ofp = 0;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + h * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait_regs(r);
                epilogue_chunk<KIND, OUT>(r, m, n0 + c, row_ok, sam, p, ck, fold, ofp);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars->acc_empty[h]), 0));
            if (p.row_cksum && row_ok) atomicAdd(p.row_cksum + m, ck);
            // this half is one 256-column fingerprint segment of the row
            if (fold) check_segment(p.chk, row_ok && n0 < p.N, seg_index(m, 2 * nt + h, p.N), ck + ofp);
        }
    }

    // the even CTA's MMAs read this CTA's shared memory and write its TMEM:
    // neither CTA frees anything before both are done
    tc_fence_before();
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
        if (lane == 0 && *abort_flag) atomicAdd(&p.status->drained, 1u);   // gave up, drained, TMEM freed
    }
}
template <int KIND, int OUT>
static int launch(const void* A, const void* B, const float* sa, const float* sb, float alpha, void* C,
                  uint32_t* cksum, int M, int N, int K, cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{},
                  uint64_t wait_ns = QG_WAIT_LIMIT_NS, int withhold_kb = -1) {
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    DeviceStatus* status = nullptr;
    if ((rc = device_status_ptr(&status))) return rc;

    // operands as byte matrices: rows of K * elem_bytes bytes
    const uint64_t kb = (uint64_t)K * elem_bytes(KIND);
    CUtensorMap tmA;
    if ((rc = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, kb, (uint64_t)M, kb, BK, BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;

    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<KIND, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        QG_CUDA(cudaFuncSetAttribute(gemm_i8_pair_kernel<KIND, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     P_SMEM_BYTES));
        QG_CUDA(cudaFuncSetAttribute(gemm_i8_wide_kernel<KIND, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     W_SMEM_BYTES));
        attr_set[dev & 63] = true;
    }
    if (cksum) QG_CUDA(cudaMemsetAsync(cksum, 0, sizeof(uint32_t) * (size_t)M, stream));

    Params p{M, N, K, sa, sb, C, cksum, status, alpha, chk, wait_ns, withhold_kb};
    if (M >= 2 * BM && info->sm_count >= 2 && withhold_kb < 0) {
        // CTA pairs: each CTA's B box is half a tile high
        CUtensorMap tmBh;
        if ((rc = make_tmap_2d(&tmBh, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, kb, (uint64_t)N, kb, BK, BN / 2,
                               CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
        // persistent pairs: only as many as can be resident at once (a pair needs
        // two free SMs of one GPC, so this can be below sm_count / 2)
        // 256x512 tiles for the 2- and 4-byte kinds wider than 256 columns
        // (8192^3, burst / ~1 s at the power cap: BF16 +4.8 / +4.7 %, FP16
        // +5.3 / +4.6 %, TF32 +7.0 / +10 %).  The 1-byte kinds keep 256x256:
        // their MMA is twice as fast per K byte, so the single accumulator
        // buffer's drain between tiles weighs twice as much (E4M3 -0.9 %), and
        // INT8's epilogue (checksum, dequant, fingerprint: ~9 instructions per
        // element, ~4.6k cycles per 128x512 drain) more still (-1.5 % at the
        // maximum clock, -9 % per clock under the power cap).
        const bool wide = elem_bytes(KIND) >= 2 && N > BN;
        static int resident[64][2] = {};
        int& res = resident[dev & 63][wide ? 1 : 0];
        if (!res) {
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(info->sm_count & ~1);
            lc.blockDim = dim3(wide ? W_THREADS : THREADS);
            lc.dynamicSmemBytes = wide ? W_SMEM_BYTES : P_SMEM_BYTES;
            int n = 0;
            if (wide) QG_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_i8_wide_kernel<KIND, OUT>, &lc));
            else QG_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_i8_pair_kernel<KIND, OUT>, &lc));
            res = n > 0 ? n : 1;
        }
        const int tiles2 = ceil_div(M, 2 * BM) * ceil_div(N, wide ? W_BN : BN);
        const int pairs = tiles2 < res ? tiles2 : res;
        if (wide) gemm_i8_wide_kernel<KIND, OUT><<<2 * pairs, W_THREADS, W_SMEM_BYTES, stream>>>(tmA, tmBh, p);
        else gemm_i8_pair_kernel<KIND, OUT><<<2 * pairs, THREADS, P_SMEM_BYTES, stream>>>(tmA, tmBh, p);
        QG_CUDA(cudaGetLastError());
        return QG_OK;
    }
    CUtensorMap tmB;
    if ((rc = make_tmap_2d(&tmB, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, kb, (uint64_t)N, kb, BK, BN,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
    const int grid = tiles < info->sm_count ? tiles : info->sm_count;
    gemm_i8_kernel<KIND, OUT><<<grid, THREADS, SMEM_BYTES, stream>>>(tmA, tmB, p);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace i8

int gemm_i8(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type, void* row_cksum,
            int M, int N, int K, cudaStream_t stream, const LaunchCheck& chk) {
    QG_CHECK_ARG(A && B && C, "qg_gemm_i8: null operand or output");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemm_i8: empty shape %dx%dx%d", M, N, K);
    QG_CHECK_ARG(K % 16 == 0, "qg_gemm_i8: K=%d must be a multiple of 16 (TMA row stride)", K);
    QG_CHECK_ARG(K <= 131072, "qg_gemm_i8: K=%d exceeds 131072 (INT32 accumulator range)", K);
    QG_CHECK_ARG(out_type == QG_OUT_S32 || (sa && sb), "qg_gemm_i8: scales required for a dequantised output");
    const float* fsa = static_cast<const float*>(sa);
    const float* fsb = static_cast<const float*>(sb);
    uint32_t* ck = static_cast<uint32_t*>(row_cksum);
    switch (out_type) {
        case QG_OUT_BF16: return i8::launch<i8::KIND_I8, QG_OUT_BF16>(A, B, fsa, fsb, 1.0f, C, ck, M, N, K, stream, chk);
        case QG_OUT_F32: return i8::launch<i8::KIND_I8, QG_OUT_F32>(A, B, fsa, fsb, 1.0f, C, ck, M, N, K, stream, chk);
        case QG_OUT_S32: return i8::launch<i8::KIND_I8, QG_OUT_S32>(A, B, fsa, fsb, 1.0f, C, ck, M, N, K, stream, chk);
        default: set_error("qg_gemm_i8: unknown out_type %d", out_type); return QG_ERR_ARG;
    }
}

uint64_t gemm_i8_check_slots(int M, int N) { return (uint64_t)M * (uint64_t)((N + i8::BN - 1) / i8::BN); }

// Fault drill: one INT8 GEMM (bf16 out) on the single-CTA kernel whose
// producers stop before K block `withhold_kb` of their first tile, with every
// bounded wait limited to `wait_ns`.  The MMA issuer's wait for the withheld
// block expires; the kernel records the site, lets its copies and MMAs in
// flight land, frees TMEM and returns.
int fault_drill_i8(const void* A, const void* B, const void* sa, const void* sb, void* C, int M, int N, int K,
                   uint64_t wait_ns, int withhold_kb, cudaStream_t stream) {
    QG_CHECK_ARG(A && B && sa && sb && C, "qg_fault_drill_i8: null operand or output");
    QG_CHECK_ARG(M > 0 && M < 2 * i8::BM && N > 0 && K > 0 && K % 16 == 0,
                 "qg_fault_drill_i8: shape %dx%dx%d (M < 256 for the single-CTA kernel, K %% 16 == 0)", M, N, K);
    QG_CHECK_ARG(withhold_kb >= 0 && withhold_kb < (K + i8::BK - 1) / i8::BK && withhold_kb < i8::STAGES,
                 "qg_fault_drill_i8: withhold_kb %d must name a K block within the first %d of the tile",
                 withhold_kb, i8::STAGES);
    QG_CHECK_ARG(wait_ns >= 100000ull && wait_ns <= QG_WAIT_LIMIT_NS,
                 "qg_fault_drill_i8: wait limit %llu ns outside [1e5, 2e9]", (unsigned long long)wait_ns);
    return i8::launch<i8::KIND_I8, QG_OUT_BF16>(A, B, static_cast<const float*>(sa), static_cast<const float*>(sb),
                                                1.0f, C, nullptr, M, N, K, stream, LaunchCheck{}, wait_ns, withhold_kb);
}

// Tensor-furnace GEMMs: C = alpha * A B^T with f32 accumulation; bf16, fp16,
// tf32 or e4m3 operands; bf16, fp16 or f32 output.
namespace {
template <int KIND>
int dense_out(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
              cudaStream_t stream, const LaunchCheck& chk) {
    switch (out_type) {
        case QG_OUT_BF16: return i8::launch<KIND, QG_OUT_BF16>(A, B, nullptr, nullptr, alpha, C, nullptr, M, N, K, stream, chk);
        case QG_OUT_F16: return i8::launch<KIND, QG_OUT_F16>(A, B, nullptr, nullptr, alpha, C, nullptr, M, N, K, stream, chk);
        default: return i8::launch<KIND, QG_OUT_F32>(A, B, nullptr, nullptr, alpha, C, nullptr, M, N, K, stream, chk);
    }
}
} // namespace

const char* dense_kind_entry(int kind) {
    switch (kind) {
        case i8::KIND_BF16: return "qg_gemm_bf16";
        case i8::KIND_F16: return "qg_gemm_f16";
        case i8::KIND_TF32: return "qg_gemm_tf32";
        case i8::KIND_E4M3: return "qg_gemm_e4m3";
        default: return "qg_gemm_dense";
    }
}

int gemm_dense(int kind, const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
               cudaStream_t stream, const LaunchCheck& chk = LaunchCheck{}) {
    const char* name = dense_kind_entry(kind);
    QG_CHECK_ARG(kind == i8::KIND_BF16 || kind == i8::KIND_F16 || kind == i8::KIND_TF32 || kind == i8::KIND_E4M3,
                 "%s: unknown operand kind %d", name, kind);
    QG_CHECK_ARG(A && B && C, "%s: null operand or output", name);
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "%s: empty shape %dx%dx%d", name, M, N, K);
    QG_CHECK_ARG(((int64_t)K * i8::elem_bytes(kind)) % 16 == 0, "%s: K=%d: rows must be a multiple of 16 bytes", name, K);
    QG_CHECK_ARG(out_type == QG_OUT_BF16 || out_type == QG_OUT_F16 || out_type == QG_OUT_F32,
                 "%s: out_type %d (bf16, f16 or f32)", name, out_type);
    switch (kind) {
        case i8::KIND_BF16: return dense_out<i8::KIND_BF16>(A, B, alpha, C, out_type, M, N, K, stream, chk);
        case i8::KIND_F16: return dense_out<i8::KIND_F16>(A, B, alpha, C, out_type, M, N, K, stream, chk);
        case i8::KIND_TF32: return dense_out<i8::KIND_TF32>(A, B, alpha, C, out_type, M, N, K, stream, chk);
        default: return dense_out<i8::KIND_E4M3>(A, B, alpha, C, out_type, M, N, K, stream, chk);
    }
}

int gemm_dense_format(int fmt, const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                      cudaStream_t stream, const LaunchCheck& chk) {
    switch (fmt) {
        case QG_FMT_BF16: return gemm_dense(i8::KIND_BF16, A, B, alpha, C, out_type, M, N, K, stream, chk);
        case QG_FMT_FP16: return gemm_dense(i8::KIND_F16, A, B, alpha, C, out_type, M, N, K, stream, chk);
        case QG_FMT_TF32: return gemm_dense(i8::KIND_TF32, A, B, alpha, C, out_type, M, N, K, stream, chk);
        case QG_FMT_E4M3: return gemm_dense(i8::KIND_E4M3, A, B, alpha, C, out_type, M, N, K, stream, chk);
        default: set_error("format %d is not a dense format", fmt); return QG_ERR_ARG;
    }
}

} // namespace qg

extern "C" int qg_gemm_i8(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type,
                          void* row_checksums, int M, int N, int K, void* stream) {
    return qg::gemm_i8(A, B, sa, sb, C, out_type, row_checksums, M, N, K, static_cast<cudaStream_t>(stream),
                       qg::LaunchCheck{});
}

extern "C" int qg_gemm_bf16(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                            void* stream) {
    return qg::gemm_dense(qg::i8::KIND_BF16, A, B, alpha, C, out_type, M, N, K, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gemm_e4m3(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                            void* stream) {
    return qg::gemm_dense(qg::i8::KIND_E4M3, A, B, alpha, C, out_type, M, N, K, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gemm_f16(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                           void* stream) {
    return qg::gemm_dense(qg::i8::KIND_F16, A, B, alpha, C, out_type, M, N, K, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gemm_tf32(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                            void* stream) {
    return qg::gemm_dense(qg::i8::KIND_TF32, A, B, alpha, C, out_type, M, N, K, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_fault_drill_i8(const void* A, const void* B, const void* sa, const void* sb, void* C, int M, int N,
                                 int K, uint64_t wait_ns, int withhold_kb, void* stream) {
    return qg::fault_drill_i8(A, B, sa, sb, C, M, N, K, wait_ns, withhold_kb, static_cast<cudaStream_t>(stream));
}
