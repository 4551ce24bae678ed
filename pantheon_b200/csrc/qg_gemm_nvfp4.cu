// qg_gemm_nvfp4.cu -- NVFP4 GEMM on the sm_100a tensor cores:
// tcgen05.mma kind::mxf4nvf4 with ue4m3 block scales per 16 elements along K.
//
//   C[m,n] = out( (GA * GB) * sum_k (qa[m,k] * sfa[m,k/16]) * (qb[n,k] * sfb[n,k/16]) )
//
// A, B: e2m1 codes packed two per byte along K (low nibble = even k), [M, K/2]
// and [N, K/2]; sfa, sfb: ue4m3 bytes in the scale-factor atom layout the MMA
// reads (one 512-byte atom per 128 rows x 64 K: row r's four scales at
// (r%32)*16 + ((r/32)%4)*4 + 0..3; atoms ordered [row block][K/64]); GA, GB:
// per-tensor fp32 scales applied in the epilogue.
//
// One persistent CTA per SM, 448 threads:
//   warp 0      producer: per 256-element K block, TMA loads of the A (128 rows)
//               and B (256 rows) code tiles (128-byte swizzle) and bulk copies
//               of the matching scale atoms (2 KB + 4 KB), 4-stage ring.
//   warps 2, 3, 12, 13   scale writers, one per TMEM lane quarter: each lane
//               reads its 16 bytes of every atom of the stage from shared
//               memory and writes them to TMEM with tcgen05.st, giving the
//               layout tcgen05.cp 32x128b.warpx4 would (each atom broadcast to
//               the four lane quarters, 4 columns per MMA).  tcgen05.cp runs
//               in the tensor pipe in order with the MMAs (12 copies per K
//               block cost ~40 % of the MMA time when measured); tcgen05.st
//               does not occupy that pipe.
//   warp 1      TMEM allocator and MMA issuer: 4 x tcgen05.mma M=128 N=256
//               K=64 per K block into a 256-column accumulator, once the
//               stage's operands have landed and its scales are in TMEM.
//               Each ring stage has its own 48-column scale region in TMEM,
//               free again exactly when the stage's shared memory is (the
//               producer refills a stage only after the commit of the MMAs
//               that read it, and the writers wait for that refill).
//   warps 4-11  epilogue: TMEM lane quarter warp % 4, column half (warp-4)/4;
//               scale by GA*GB, round, store.
// All barrier waits are bounded (qg_ptx.cuh).
#include "qg_common.cuh"
#include "qg_check.cuh"

#include <cuda_bf16.h>

namespace qg {
namespace f4 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 256;                       // fp4 elements per K block = 128 bytes per row
constexpr int BK_BYTES = BK / 2;
constexpr int UMMA_K = 64;                    // elements per tcgen05.mma kind::mxf4nvf4
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK_BYTES;        // 16 KB
constexpr int B_BYTES = BN * BK_BYTES;        // 32 KB
constexpr int SFA_BYTES = (BM / 128) * (BK / 64) * 512;   // 2 KB
constexpr int SFB_BYTES = (BN / 128) * (BK / 64) * 512;   // 4 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int ACC_COLS = BN;
constexpr int SFA_COLS = (BK / UMMA_K) * 4;                  // 16: 4 MMAs x 4 columns
constexpr int SFB_COLS = (BK / UMMA_K) * (BN / 128) * 4;     // 32
constexpr int SF_STAGE_COLS = SFA_COLS + SFB_COLS;           // 48 per ring stage
constexpr int TMEM_COLS = 512;                // 256 accumulator + 4 x 48 scale columns, rounded up
static_assert(ACC_COLS + STAGES * SF_STAGE_COLS <= TMEM_COLS, "TMEM budget");
constexpr int THREADS = 448;
constexpr int EPI_WARP0 = 4;
constexpr int EPI_WARP_END = 12;
constexpr int SF_WRITERS = 4;                 // warps 2, 3, 12, 13: lane quarters 2, 3, 0, 1
constexpr int EPI_THREADS = 256;
// Tile rasterisation: consecutive tiles walk group_m row-tiles (sharing B tiles
// in L2) before moving to the next columns; B is re-read once per group, A's
// rows of a group must stay in L2 meanwhile.  The group is sized so its rows
// of A total about 32 MB: at 16384^3 (8 KB rows) that is 32 row-tiles, and
// DRAM reads per launch measured 1.36 GB at 16, 0.80 GB at 32, 4.25 GB at 64
// (thrashing), with 1890 / 1852 / 2110 us.
constexpr uint64_t GROUP_A_BYTES = 32ull << 20;
static int group_rows(int K) {
    const uint64_t per_tile = (uint64_t)BM * (uint64_t)K / 2;     // A bytes of one row-tile
    const uint64_t g = GROUP_A_BYTES / (per_tile ? per_tile : 1);
    return (int)(g < 1 ? 1 : (g > 64 ? 64 : g));
}

struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t sf_ready[STAGES];
    uint64_t tmem_full;
    uint64_t tmem_empty;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

constexpr uint32_t SITE_PRODUCER = 0x00030001u;
constexpr uint32_t SITE_MMA_FULL = 0x00030002u;
constexpr uint32_t SITE_MMA_TMEM = 0x00030003u;
constexpr uint32_t SITE_EPI = 0x00030004u;
constexpr uint32_t SITE_SF = 0x00030005u;
constexpr uint32_t SITE_MMA_SF = 0x00030006u;

struct Params {
    int M, N, K;
    const uint8_t* sfa;
    const uint8_t* sfb;
    float gab;            // GA * GB
    void* C;
    DeviceStatus* status;
    int group_m;          // row-tiles per rasterisation group
    LaunchCheck chk;      // per-launch check: one fingerprint per (row, 128-column segment)
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& mt, int& nt) {
    const int group = group_m * tiles_n;
    const int g = t / group;
    const int first_m = g * group_m;
    const int gm = min(tiles_m - first_m, group_m);
    const int r = t - g * group;
    mt = first_m + r % gm;
    nt = r / gm;
}

template <int OUT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sA = smem;
    uint8_t* sB = sA + STAGES * A_BYTES;
    uint8_t* sSFA = sB + STAGES * B_BYTES;
    uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
    Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tiles_m = (p.M + BM - 1) / BM;
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int nk = p.K / BK;
    const int kchunks = p.K / 64;                 // scale atoms per 128-row block
    const int n_row_blocks = (p.N + 127) / 128;   // 128-row blocks of B's scales

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
            mbar_init(&bars->sf_ready[s], SF_WRITERS);
        }
        mbar_init(&bars->tmem_full, 1);
        mbar_init(&bars->tmem_empty, EPI_THREADS / 32);
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
            tile_coords(t, tiles_m, tiles_n, p.group_m, mt, nt);
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, p.status, SITE_PRODUCER)) { ok = false; break; }
                mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
                tma_load_2d(sA + stage * A_BYTES, &tmA, &bars->full[stage], kb * BK_BYTES, mt * BM);
                tma_load_2d(sB + stage * B_BYTES, &tmB, &bars->full[stage], kb * BK_BYTES, nt * BN);
                // scale atoms of this K block: 4 consecutive atoms per 128-row block
                bulk_load(sSFA + stage * SFA_BYTES, p.sfa + ((size_t)mt * kchunks + kb * 4) * 512, SFA_BYTES / (BM / 128),
                          &bars->full[stage]);
                // (a 128-row block past the end of B exists only in a ragged last
                // tile; its columns are never stored, so block 0 stands in for it)
#pragma unroll
                for (int h = 0; h < BN / 128; ++h) {
                    const int blk = nt * (BN / 128) + h < n_row_blocks ? nt * (BN / 128) + h : 0;
                    bulk_load(sSFB + stage * SFB_BYTES + h * (SFB_BYTES / (BN / 128)),
                              p.sfb + ((size_t)blk * kchunks + kb * 4) * 512, SFB_BYTES / (BN / 128),
                              &bars->full[stage]);
                }
                armed |= 1u << stage;
                armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (!ok)
            for (int s = 0; s < STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ scale copies + MMA issuer
        constexpr uint32_t IDESC = make_idesc_bs(/*e2m1*/ 1, /*e2m1*/ 1, /*ue4m3*/ 0, BM, BN);
        uint32_t stage = 0, phase = 0;
        bool ok = true, issued = false;
        int iter = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++iter) {
            if (!mbar_wait(&bars->tmem_empty, (iter & 1) ^ 1u, abort_flag, p.status, SITE_MMA_TMEM)) { ok = false; break; }
            tc_fence_after();
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_MMA_FULL)) { ok = false; break; }
                if (!mbar_wait(&bars->sf_ready[stage], phase, abort_flag, p.status, SITE_MMA_SF)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sfa_col = tmem_base + ACC_COLS + stage * SF_STAGE_COLS;
                const uint32_t sfb_col = sfa_col + SFA_COLS;
                const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
                const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k)
                    umma_nvf4(tmem_base, make_sdesc_kmajor_sw128(a_addr + k * (UMMA_K / 2)),
                              make_sdesc_kmajor_sw128(b_addr + k * (UMMA_K / 2)), IDESC,
                              sfa_col + 4 * k, sfb_col + (BN / 128) * 4 * k,
                              (kb | k) != 0 ? 1u : 0u);
                issued = true;
                umma_commit(&bars->empty[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) umma_commit(&bars->tmem_full);
        }
        if (!ok && issued) {
            umma_commit(&bars->drain);
            mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
        }
    } else if (warp == 2 || warp == 3 || warp >= EPI_WARP_END) {
        // ------------------------------------------------------------ scale writers
        const int quarter = warp & 3;
        const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16) + ACC_COLS;
        uint32_t stage = 0, phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < nk; ++kb) {
                // every lane waits: a lane-0 poll with a shuffle after it cost the FP8
                // GEMM's per-K-block waits ~15 %
                if (!__all_sync(0xffffffffu, mbar_wait(&bars->full[stage], phase, abort_flag, p.status, SITE_SF))) {
                    ok = false;
                    break;
                }
                // lane i takes bytes [16 i, 16 i + 16) of each atom: TMEM columns
                // 4k..4k+3 (A) and 16 + 8k + 4h .. +3 (B) of this stage's region
                const uint4* sfa = reinterpret_cast<const uint4*>(sSFA + stage * SFA_BYTES) + lane;
                const uint4* sfb = reinterpret_cast<const uint4*>(sSFB + stage * SFB_BYTES) + lane;
                uint32_t va[16], vb0[16], vb1[16];
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k) {
                    const uint4 a = sfa[k * 32];
                    va[4 * k] = a.x; va[4 * k + 1] = a.y; va[4 * k + 2] = a.z; va[4 * k + 3] = a.w;
                }
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k) {
#pragma unroll
                    for (int h = 0; h < BN / 128; ++h) {
                        const uint4 b = sfb[h * (SFB_BYTES / (BN / 128) / 16) + k * 32];
                        uint32_t* d = (2 * k + h) < 4 ? &vb0[4 * (2 * k + h)] : &vb1[4 * (2 * k + h - 4)];
                        d[0] = b.x; d[1] = b.y; d[2] = b.z; d[3] = b.w;
                    }
                }
                const uint32_t col = t_lane + stage * SF_STAGE_COLS;
                tmem_st_32x32b_x16(col, va);
                tmem_st_32x32b_x16(col + SFA_COLS, vb0);
                tmem_st_32x32b_x16(col + SFA_COLS + 16, vb1);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->sf_ready[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const int half = (warp - EPI_WARP0) >> 2;
        const int row = quarter * 32 + lane;
        const bool fold = p.chk.record != nullptr || p.chk.expect != nullptr;
        int iter = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++iter) {
            int mt, nt;
            tile_coords(t, tiles_m, tiles_n, p.group_m, mt, nt);
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&bars->tmem_full, iter & 1, abort_flag, p.status, SITE_EPI) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const int m = mt * BM + row;
            const bool row_ok = m < p.M;
            const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * (BN / 2);
            uint32_t ofp = 0;   // fingerprint of the words stored for this row segment (qg_check.cuh)
#pragma unroll 1
            for (int c = 0; c < BN / 2; c += 32) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(t_row + c, r);
                tmem_ld_wait_regs(r);
                if (c + 32 == BN / 2) {
                    // the tile's last accumulator columns are in registers: the MMA of
                    // the next tile may overwrite TMEM while this chunk is stored
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->tmem_empty);
                }
                const int n0 = nt * BN + half * (BN / 2) + c;
                if (!row_ok || n0 >= p.N) continue;
                const bool full_chunk = (n0 + 32 <= p.N);
                float f[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) f[i] = __fmul_rn(__uint_as_float(r[i]), p.gab);
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
                            if (full_chunk || n0 + i < p.N)
                                ofp = ofp * kCheckMul + __float_as_uint(f[i]);
                    }
                } else {
                    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.C) + (size_t)m * p.N + n0;
                    if (full_chunk && (p.N % 8) == 0) {
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            uint32_t w[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                __nv_bfloat162 h = __floats2bfloat162_rn(f[i + 2 * j], f[i + 2 * j + 1]);
                                w[j] = *reinterpret_cast<uint32_t*>(&h);
                                if (fold) ofp = ofp * kCheckMul + w[j];
                            }
                            *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (n0 + i < p.N) {
                                const __nv_bfloat16 h = __float2bfloat16_rn(f[i]);
                                dst[i] = h;
                                if (fold)
                                    ofp = ofp * kCheckMul + (uint32_t)__bfloat16_as_ushort(h);
                            }
                    }
                }
            }
            if (fold) {
                const int seg = nt * 2 + half;
                check_segment(p.chk, row_ok && seg * (BN / 2) < p.N,
                              (uint64_t)m * (uint64_t)((p.N + BN / 2 - 1) / (BN / 2)) + (uint64_t)seg, ofp);
            }
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
static int launch(const void* A, const void* SFA, const void* B, const void* SFB, float gab, void* C, int M, int N,
                  int K, cudaStream_t stream, const LaunchCheck& chk) {
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    DeviceStatus* status = nullptr;
    if ((rc = device_status_ptr(&status))) return rc;
    CUtensorMap tmA, tmB;
    if ((rc = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K / 2, (uint64_t)M, (uint64_t)K / 2,
                           BK_BYTES, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tmap_2d(&tmB, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                           BK_BYTES, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(gemm_nvfp4_kernel<QG_OUT_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        QG_CUDA(cudaFuncSetAttribute(gemm_nvfp4_kernel<QG_OUT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr_set[dev & 63] = true;
    }
    Params p{M, N, K, static_cast<const uint8_t*>(SFA), static_cast<const uint8_t*>(SFB), gab, C, status, group_rows(K),
             chk};
    const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
    const int grid = tiles < info->sm_count ? tiles : info->sm_count;
    gemm_nvfp4_kernel<OUT><<<grid, THREADS, SMEM_BYTES, stream>>>(tmA, tmB, p);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace f4

uint64_t nvfp4_sf_bytes(int R, int K) { return (uint64_t)((R + 127) / 128) * (uint64_t)(K / 64) * 512; }

uint64_t gemm_nvfp4_check_slots(int M, int N) { return (uint64_t)M * (uint64_t)((N + f4::BN / 2 - 1) / (f4::BN / 2)); }

int gemm_nvfp4(const void* A, const void* SFA, const void* B, const void* SFB, float ga, float gb, void* C,
               int out_type, int M, int N, int K, cudaStream_t stream, const LaunchCheck& chk) {
    QG_CHECK_ARG(A && SFA && B && SFB && C, "qg_gemm_nvfp4: null operand");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemm_nvfp4: empty shape %dx%dx%d", M, N, K);
    QG_CHECK_ARG(K % 256 == 0, "qg_gemm_nvfp4: K=%d must be a multiple of 256", K);
    QG_CHECK_ARG(((uintptr_t)SFA & 15) == 0 && ((uintptr_t)SFB & 15) == 0, "qg_gemm_nvfp4: scale tensors must be 16-byte aligned");
    const float gab = ga * gb;
    switch (out_type) {
        case QG_OUT_BF16: return f4::launch<QG_OUT_BF16>(A, SFA, B, SFB, gab, C, M, N, K, stream, chk);
        case QG_OUT_F32: return f4::launch<QG_OUT_F32>(A, SFA, B, SFB, gab, C, M, N, K, stream, chk);
        default: set_error("qg_gemm_nvfp4: bad out_type %d", out_type); return QG_ERR_ARG;
    }
}

} // namespace qg

extern "C" int qg_gemm_nvfp4(const void* A, const void* SFA, const void* B, const void* SFB, float ga, float gb,
                             void* C, int out_type, int M, int N, int K, void* stream) {
    return qg::gemm_nvfp4(A, SFA, B, SFB, ga, gb, C, out_type, M, N, K, static_cast<cudaStream_t>(stream),
                          qg::LaunchCheck{});
}

extern "C" int qg_nvfp4_sf_bytes(int rows, int K, uint64_t* bytes) {
    QG_CHECK_ARG(bytes && rows > 0 && K > 0 && K % 64 == 0, "qg_nvfp4_sf_bytes: bad argument");
    *bytes = qg::nvfp4_sf_bytes(rows, K);
    return QG_OK;
}
