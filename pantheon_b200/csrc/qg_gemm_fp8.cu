// qg_gemm_fp8.cu -- FP8 e4m3 GEMM with fp32 block scales (1x128 on A, 128x128
// on B) on the sm_100a tensor cores (tcgen05.mma kind::f8f6f4).
//
//   C[m,n] = out( sum_kb  P_kb[m,n] * sa[m,kb] * sb[n/128,kb] ),
//   P_kb[m,n] = sum_{k in block kb} A[m,k] * B[n,k]       (fp32, one 128-deep block)
//
// fp32 block scales that are not powers of two cannot ride in the MMA's own
// block-scale path, so each 128-deep K block is its own MMA accumulation and
// its partial is promoted on the CUDA cores: acc = fma(P_kb, sa*sb, acc).
//
// One persistent CTA per SM, 320 threads (10 warps):
//   warp 0      TMA producer: A 128x128 and B 256x128 e4m3 tiles (128-byte swizzle),
//               4-stage shared-memory ring.
//   warp 1      TMEM allocator (512 columns) and MMA issuer: per K block, 4 x
//               tcgen05.mma M=128 N=256 K=32 into one of two 256-column TMEM
//               partial buffers (the next block's MMAs run while the epilogue
//               promotes the previous partial).
//   warps 2-9   promotion + epilogue: warp w reads TMEM lane quarter w % 4,
//               columns 128 * ((w - 2) / 4) .. +127 (one B scale block), keeps
//               128 fp32 accumulators of its row in registers, and after the
//               last K block converts and stores its row segment.
// All barrier waits are bounded (qg_ptx.cuh).
#include "qg_common.cuh"
#include "qg_check.cuh"

#include <cuda_bf16.h>

namespace qg {
namespace f8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;              // e4m3 elements = bytes per K block (one swizzle row)
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int PART_COLS = BN;        // fp32 partial columns per buffer
constexpr int TMEM_COLS = 2 * PART_COLS;
constexpr int THREADS = 320;
constexpr int EPI_WARP0 = 2;
constexpr int EPI_THREADS = 256;
constexpr int GROUP_M = 16;
constexpr int COLS_PER_EPI = 128;    // columns per epilogue thread (its row)

struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t part_full[2];
    uint64_t part_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

constexpr uint32_t SITE_PRODUCER = 0x00020001u;
constexpr uint32_t SITE_MMA_FULL = 0x00020002u;
constexpr uint32_t SITE_MMA_PART = 0x00020003u;
constexpr uint32_t SITE_EPI = 0x00020004u;

struct Params {
    int M, N, K;
    const float* sa;     // [M, K/128]
    const float* sb;     // [ceil(N/128), K/128]
    void* C;
    DeviceStatus* status;
    LaunchCheck chk;     // per-launch check: one fingerprint per (row, 128-column segment)
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
    const int group = GROUP_M * tiles_n;
    const int g = t / group;
    const int first_m = g * GROUP_M;
    const int gm = min(tiles_m - first_m, GROUP_M);
    const int r = t - g * group;
    mt = first_m + r % gm;
    nt = r / gm;
}

template <int OUT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
    extern __shared__ uint8_t smem_raw[];
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
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&bars->full[s], 1); mbar_init(&bars->empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&bars->part_full[a], 1); mbar_init(&bars->part_empty[a], EPI_THREADS / 32); }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
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
        uint32_t stage = 0, phase = 0, armed = 0, armed_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, tiles_m, tiles_n, mt, nt);
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PRODUCER)) { ok = false; break; }
                mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
                tma_load_2d(sA + stage * A_BYTES, &tmA, &bars->full[stage], kb * BK, mt * BM);
                tma_load_2d(sB + stage * B_BYTES, &tmB, &bars->full[stage], kb * BK, nt * BN);
                armed |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok)
            for (int s = 0; s < STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t IDESC = make_idesc(/*f32*/ 1, /*e4m3*/ 0, /*e4m3*/ 0, BM, BN);
        uint32_t stage = 0, phase = 0;
        uint32_t pcount = 0;           // K blocks issued so far (partial ring position)
        bool ok = true, issued = false;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < nk; ++kb, ++pcount) {
                const uint32_t buf = pcount & 1u;
                const uint32_t pph = (pcount >> 1) & 1u;
                if (!mbar_wait(&bars->part_empty[buf], pph ^ 1u, abort_flag, p.status, SITE_MMA_PART)) { ok = false; break; }
                tc_fence_after();
                if (!mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_MMA_FULL)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
                const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
                const uint32_t d_tmem = tmem_base + buf * PART_COLS;
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k)
                    umma_f8(d_tmem, make_sdesc_kmajor_sw128(a_addr + k * UMMA_K),
                            make_sdesc_kmajor_sw128(b_addr + k * UMMA_K), IDESC, k != 0 ? 1u : 0u);
                issued = true;
                umma_commit(&bars->empty[stage]);
                umma_commit(&bars->part_full[buf]);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok && issued) {
            umma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ promotion + epilogue
        const int quarter = warp & 3;                    // TMEM lanes 32*quarter .. +31
        const int half = (warp - EPI_WARP0) >> 2;        // column half 0 / 1 of the tile
        const int row = quarter * 32 + lane;
        const int sb_rows = (p.N + 127) / 128;
        const bool fold = p.chk.record != nullptr || p.chk.expect != nullptr;
        uint32_t pcount = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, tiles_m, tiles_n, mt, nt);
            const int m = mt * BM + row;
            const bool row_ok = m < p.M;
            const int nb = nt * 2 + half;                // B scale block of this column half
            const bool nb_ok = nb < sb_rows;
            const float* sa_row = p.sa + (size_t)(row_ok ? m : 0) * nk;
            const float* sb_row = p.sb + (size_t)(nb_ok ? nb : 0) * nk;
            float acc[COLS_PER_EPI];
#pragma unroll
            for (int i = 0; i < COLS_PER_EPI; ++i) acc[i] = 0.0f;
            // scales of the first K block; later ones are fetched a block ahead
            float sa_next = row_ok ? __ldg(sa_row) : 0.0f;
            float sb_next = nb_ok ? __ldg(sb_row) : 0.0f;
            for (int kb = 0; kb < nk; ++kb, ++pcount) {
                const uint32_t buf = pcount & 1u;
                const uint32_t pph = (pcount >> 1) & 1u;
                const float scale = __fmul_rn(sa_next, sb_next);
                if (kb + 1 < nk) {
                    sa_next = row_ok ? __ldg(sa_row + kb + 1) : 0.0f;
                    sb_next = nb_ok ? __ldg(sb_row + kb + 1) : 0.0f;
                }
                // every lane waits (no divergent branch around the wait)
                if (!__all_sync(0xffffffffu, mbar_wait(&bars->part_full[buf], pph, abort_flag, p.status, SITE_EPI))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t t_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * PART_COLS + half * COLS_PER_EPI;
                // two 16-column loads in flight: the next chunk loads while this one is promoted
                uint32_t ra[16], rb[16];
                tmem_ld_32x32b_x16(t_addr, ra);
                tmem_ld_wait_regs(ra);
#pragma unroll
                for (int c = 0; c < COLS_PER_EPI; c += 32) {
                    tmem_ld_32x32b_x16(t_addr + c + 16, rb);
#pragma unroll
                    for (int i = 0; i < 16; i += 2)
                        fma2_scalar(acc[c + i], acc[c + i + 1], __uint_as_float(ra[i]), __uint_as_float(ra[i + 1]), scale);
                    tmem_ld_wait_regs(rb);
                    if (c + 32 < COLS_PER_EPI) tmem_ld_32x32b_x16(t_addr + c + 32, ra);
#pragma unroll
                    for (int i = 0; i < 16; i += 2)
                        fma2_scalar(acc[c + 16 + i], acc[c + 17 + i], __uint_as_float(rb[i]), __uint_as_float(rb[i + 1]), scale);
                    if (c + 32 < COLS_PER_EPI) tmem_ld_wait_regs(ra);
                }
                // release the partial buffer: one arrival per warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->part_empty[buf]);
            }
            if (!ok) break;
            // store this row's 128-column segment, folding the stored words into
            // its fingerprint in a golden or checked launch (qg_check.cuh)
            const int n0 = nt * BN + half * COLS_PER_EPI;
            const bool seg_ok = row_ok && n0 < p.N;
            uint32_t ofp = 0;
            if (seg_ok) {
                const bool full_seg = (n0 + COLS_PER_EPI <= p.N);
                if (OUT == QG_OUT_F32) {
                    float* dst = static_cast<float*>(p.C) + (size_t)m * p.N + n0;
                    if (full_seg && (p.N % 4) == 0) {
#pragma unroll
                        for (int i = 0; i < COLS_PER_EPI; i += 4)
                            *reinterpret_cast<float4*>(dst + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < COLS_PER_EPI; ++i)
                            if (n0 + i < p.N) dst[i] = acc[i];
                    }
                    if (fold) {
#pragma unroll
                        for (int i = 0; i < COLS_PER_EPI; ++i)
                            if (full_seg || n0 + i < p.N)
                                ofp = ofp * kCheckMul + __float_as_uint(acc[i]);
                    }
                } else {
                    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.C) + (size_t)m * p.N + n0;
                    if (full_seg && (p.N % 8) == 0) {
#pragma unroll
                        for (int i = 0; i < COLS_PER_EPI; i += 8) {
                            uint32_t w[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                __nv_bfloat162 h = __floats2bfloat162_rn(acc[i + 2 * j], acc[i + 2 * j + 1]);
                                w[j] = *reinterpret_cast<uint32_t*>(&h);
                                if (fold) ofp = ofp * kCheckMul + w[j];
                            }
                            *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < COLS_PER_EPI; ++i)
                            if (n0 + i < p.N) {
                                const __nv_bfloat16 h = __float2bfloat16_rn(acc[i]);
                                dst[i] = h;
                                if (fold)
                                    ofp = ofp * kCheckMul + (uint32_t)__bfloat16_as_ushort(h);
                            }
                    }
                }
            }
            if (fold)
                check_segment(p.chk, seg_ok, (uint64_t)m * (uint64_t)((p.N + COLS_PER_EPI - 1) / COLS_PER_EPI) +
                                                 (uint64_t)(nt * 2 + half), ofp);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int OUT>
static int launch(const void* A, const void* B, const float* sa, const float* sb, void* C, int M, int N, int K,
                  cudaStream_t stream, const LaunchCheck& chk) {
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    DeviceStatus* status = nullptr;
    if ((rc = device_status_ptr(&status))) return rc;
    CUtensorMap tmA, tmB;
    if ((rc = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)M, (uint64_t)K, BK, BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tmap_2d(&tmB, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)N, (uint64_t)K, BK, BN,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(gemm_fp8_kernel<QG_OUT_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        QG_CUDA(cudaFuncSetAttribute(gemm_fp8_kernel<QG_OUT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr_set[dev & 63] = true;
    }
    Params p{M, N, K, sa, sb, C, status, chk};
    const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
    const int grid = tiles < info->sm_count ? tiles : info->sm_count;
    gemm_fp8_kernel<OUT><<<grid, THREADS, SMEM_BYTES, stream>>>(tmA, tmB, p);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace f8

uint64_t gemm_fp8_check_slots(int M, int N) { return (uint64_t)M * (uint64_t)((N + f8::COLS_PER_EPI - 1) / f8::COLS_PER_EPI); }

int gemm_fp8(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type, int M, int N, int K,
             cudaStream_t stream, const LaunchCheck& chk) {
    QG_CHECK_ARG(A && B && sa && sb && C, "qg_gemm_fp8_b128: null operand");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemm_fp8_b128: empty shape %dx%dx%d", M, N, K);
    QG_CHECK_ARG(K % 128 == 0, "qg_gemm_fp8_b128: K=%d must be a multiple of 128 (scale block)", K);
    const float* fsa = static_cast<const float*>(sa);
    const float* fsb = static_cast<const float*>(sb);
    switch (out_type) {
        case QG_OUT_BF16: return f8::launch<QG_OUT_BF16>(A, B, fsa, fsb, C, M, N, K, stream, chk);
        case QG_OUT_F32: return f8::launch<QG_OUT_F32>(A, B, fsa, fsb, C, M, N, K, stream, chk);
        default: set_error("qg_gemm_fp8_b128: bad out_type %d", out_type); return QG_ERR_ARG;
    }
}

} // namespace qg

extern "C" int qg_gemm_fp8_b128(const void* A, const void* B, const void* sa, const void* sb, void* C, int out_type,
                                int M, int N, int K, void* stream) {
    return qg::gemm_fp8(A, B, sa, sb, C, out_type, M, N, K, static_cast<cudaStream_t>(stream), qg::LaunchCheck{});
}
