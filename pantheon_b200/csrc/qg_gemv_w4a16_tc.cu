// qg_gemv_w4a16_tc.cu -- W4A16 group-128 skinny GEMM for 3..16 activation rows
// on the sm_100a tensor cores (tcgen05.mma kind::i8, A operand in TMEM).
//
//   Y[m, n] = sum_k X[m, k] * (q[k, n] - Z[k/128, n]) * S[k/128, n],  q = u - 8
//
// Same operands as the CUDA-core GEMV (qg_gemv_w4a16.cu): X bf16 [M, K];
// W uint32 [K/8, N] (nibble j of word (k8, n) is u(8*k8 + j, n)); S, Z fp16
// [K/128, N]; Y bf16 or fp32 [M, N].
//
// At 8-16 rows a CUDA-core GEMV needs M FMAs per weight (3.8 GFMA per call at
// M = 16, >= 100 us on the FP32 pipes against ~19 us of HBM time), so the
// products go to the tensor cores with the weights as the MMA's M side:
// D[n, r] = sum_k Wt[n, k] * B[r, k], M = 128 weight columns, N = 32 rows.
//
// Integer arithmetic, exact up to the fold (the CUDA-core path's numerics):
// * weights: the signed byte 16 q (the nibble in a byte's high half with its
//   top bit flipped), two LOP3s per four weights;
// * activations: per (row, group) the bf16 values become 14-bit fixed point
//   x = xi * 2^e (the group's absmax below 2^14, xi clamped to 2^14 - 1),
//   split into digits xi = 128 h + l, h = xi >> 7 in [-128, 127], l in
//   [0, 127] (both int8); B rows 0-15 hold h, rows 16-31 l;
// * per group the MMA gives D_h = sum 16 q h and D_l = sum 16 q l in int32, so
//   sum_k q xi = 8 D_h + D_l / 16 exactly, and the fold is
//   y += s * 2^e * (sum q xi - z * sum xi).
// Measured against the bf16 formulation of the same kernel, 8-bit operands
// halve the MMA count (K = 32 per instruction; the M=128 N<=32 MMAs cost a
// fixed ~45 cycles each) and the TMEM store traffic.
//
// Unit of work = one 128-column tile x UG = 2 groups of 128 K (16 KB of W).
// The units, tile-major, are cut into one contiguous range per CTA (one CTA
// per SM, one wave); a tile whose units span several CTAs is reduced through
// a workspace with a ticket per (tile, lane quarter): the last CTA to finish
// sums the pieces in order, so the result is bit-for-bit reproducible.
//
// Per CTA, 832 threads (26 warps):
//   warp 0      producer: per unit, TMA loads of the W tile (32 packed rows x
//               128 columns, no swizzle) and the raw X slab (M rows x 256 bf16)
//               into a 6-stage ring (96 KB of W in flight per SM).
//   warps 2-5   activation staging: quantise the X slab as above into one
//               32-row x 128-byte, 128-byte-swizzled K-major tile per group (in
//               the MMA's K order, below), plus each (row, group)'s 2^e and
//               sum xi.  Rows M..15 (and 16+M..31) are zeroed once.
//   warps 10-25 dequant, two teams of 8 taking alternate units (one team's
//               barrier round trips overlap the other's): each warp owns a TMEM
//               lane quarter and 8 of the 16 packed rows of a group; lane n
//               turns each word into two TMEM columns of four 16q bytes, written
//               with tcgen05.st as the MMA's A operand.
//   warp 1      TMEM allocator and MMA issuer: per group 4 x tcgen05.mma M=128
//               N=32 K=32 into a 32-column int32 accumulator.
//   warps 6-9   fold, one per lane quarter: per unit, read both groups'
//               accumulators and fold all 16 rows; scales and zero points
//               arrive by cp.async SZ_AHEAD units ahead (a load consumed in its
//               own iteration put an HBM round trip on every unit).
// K order inside each packed word kw: TMEM column 2kw holds k = 8kw + 0, 2, 4,
// 6 and column 2kw+1 holds k = 8kw + 1, 3, 5, 7, so the activation tile stores
// each run of eight as (x0, x2, x4, x6, x1, x3, x5, x7); both operands use the
// same permutation, which leaves the sum over k unchanged.  Groups past K (odd
// K/128) load as zeros and carry zero scales, so they add nothing.
// All barrier waits are bounded (qg_ptx.cuh).
#include "qg_common.cuh"
#include "qg_gemv.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qg {
namespace w4tc {

constexpr int TILE_N = 128;                   // weight columns per tile = MMA M
constexpr int GROUP = 128;                    // K per group (one scale / zero point)
constexpr int UG = 2;                         // groups per unit
constexpr int MROWS = 16;                     // activation rows, padded
constexpr int MMA_N = 2 * MROWS;              // h rows, then l rows
constexpr int UMMA_K = 32;                    // int8 elements per MMA
constexpr int STAGES = 6;
constexpr int W_ROWS = UG * GROUP / 8;                    // 32 packed rows
constexpr int W_BYTES = TILE_N * W_ROWS * 4;              // 16 KB
constexpr int XRAW_ROW = UG * GROUP * 2;                  // 512 B per activation row
constexpr int XRAW_BYTES = MROWS * XRAW_ROW;              // 8 KB (rows >= M not loaded)
constexpr int XT_GROUP = MMA_N * GROUP;                   // 4 KB int8 tile per group
constexpr int XT_OFF = W_BYTES + XRAW_BYTES;
constexpr int STAGE_BYTES = XT_OFF + UG * XT_GROUP;       // 32 KB
static_assert(XT_OFF % 1024 == 0 && STAGE_BYTES % 1024 == 0, "swizzled tiles need 1 KB alignment");
constexpr int TEAMS = 2;                      // dequant teams, alternate units
constexpr int NA = 4;                         // A operand buffers in TMEM
constexpr int A_COLS = UG * GROUP / 4;        // 64 columns per unit: 2 x 128 bytes per lane
constexpr int ND = 4;                         // accumulator buffers in TMEM
constexpr int D_COLS = UG * MMA_N;            // 64 columns per unit
constexpr int D_COL0 = NA * A_COLS;
constexpr int TMEM_COLS = 512;
static_assert(D_COL0 + ND * D_COLS <= TMEM_COLS, "TMEM budget");
static_assert(NA % TEAMS == 0, "each team cycles through its own A buffers");
constexpr int XS_RING = 16;                   // row sums / scales by unit (>= STAGES + ND)
constexpr int SZ_AHEAD = 4;                   // units between an S/Z fetch and its fold
constexpr int SZ_RING = 8;                    // >= SZ_AHEAD + 1
static_assert(XS_RING >= STAGES + ND && SZ_RING >= SZ_AHEAD + 1, "ring depths");
constexpr int XW0 = 2, XWARPS = 4;            // activation staging warps
constexpr int FW0 = 6, FWARPS = 4;            // fold warps
constexpr int DW0 = 10, DWARPS = 8;           // dequant warps per team
constexpr int THREADS = (DW0 + TEAMS * DWARPS) * 32;      // 832
// A warp reaches TMEM lanes 32 * (warp % 4) .. +31 only: the four fold warps and
// each half-team of four dequant warps are consecutive, so they cover all four.
constexpr int SLICES = FWARPS;                // reduction slices of a tile = lane quarters
constexpr int EMPTY_ARRIVALS = DWARPS + XWARPS + 1;       // one team, staging warps, MMA commit

constexpr uint32_t SITE_PRODUCER = 0x00040001u;
constexpr uint32_t SITE_MMA = 0x00040002u;
constexpr uint32_t SITE_X = 0x00040003u;
constexpr uint32_t SITE_DEQ = 0x00040004u;
constexpr uint32_t SITE_FOLD = 0x00040005u;

struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t x_full[STAGES];
    uint64_t a_full[NA];
    uint64_t a_empty[NA];
    uint64_t d_full[ND];
    uint64_t d_empty[ND];
    uint64_t xs_full[XS_RING];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

// per (unit slot, group, row): the row's 2^e and sum of xi
constexpr int XSUM_BYTES = XS_RING * UG * MROWS * 4 * 2;              // 4 KB
constexpr int SZ_BYTES = FWARPS * SZ_RING * UG * 64 * 2;              // 8 KB: 32 scales + 32 zeros
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + XSUM_BYTES + SZ_BYTES + (int)sizeof(Barriers) + 1024;

struct Params {
    const __half* S;
    const __half* Z;
    void* Y;
    float* ws;               // [tiles][maxp][SLICES][16 rows][32 lanes] fp32 partials
    unsigned int* tickets;   // [tiles][SLICES], zero between calls
    int M, N, K;
    int G;                   // groups = K / 128
    int upt;                 // units per tile = ceil(G / UG)
    long long units;         // tiles * upt
    int maxp;                // most CTAs sharing one tile
    int out_type;
    DeviceStatus* status;
};

// The CTA whose unit range [c*U/C, (c+1)*U/C) holds unit u.
__host__ __device__ __forceinline__ int owner(long long u, long long units, int ctas) {
    return (int)(((u + 1) * ctas - 1) / units);
}

// (tile, unit-in-tile) of a unit, walked forward without dividing (a 64-bit
// division per unit was a quarter of a unit's time in the consumer warps).
struct UnitPos {
    int t, j;
    __device__ __forceinline__ void next(int upt) {
        if (++j == upt) { j = 0; ++t; }
    }
};

// Every lane of the warp waits (each lane then reads shared memory the
// barrier's phase published); true only if all lanes saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, DeviceStatus* status,
                                          uint32_t site) {
    const bool ok = mbar_wait(bar, parity, abort, status, site);
    return __all_sync(0xffffffffu, ok);
}

// Byte offset of (row, 16-byte chunk) in a 32-row x 128-byte K-major tile with
// the 128-byte swizzle (chunk index XOR row % 8 inside each 8-row atom).
__device__ __forceinline__ int xt_offset(int row, int chunk) {
    return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}

__global__ void __launch_bounds__(THREADS, 1)
gemv_w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* stages = smem;
    float* xscale = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);     // [XS_RING][UG][16]
    float* xsum = xscale + XS_RING * UG * MROWS;                              // [XS_RING][UG][16]
    uint16_t* szring = reinterpret_cast<uint16_t*>(smem + STAGES * STAGE_BYTES + XSUM_BYTES);
    Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES + XSUM_BYTES + SZ_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ctas = gridDim.x;
    const long long u0 = (long long)blockIdx.x * p.units / ctas;
    const long long u1 = (long long)(blockIdx.x + 1) * p.units / ctas;
    const int nu = (int)(u1 - u0);
    const UnitPos start{(int)(u0 / p.upt), (int)(u0 % p.upt)};

    // launched with programmatic stream serialization: no global access (and
    // no TMEM) until the previous grid on the stream is complete
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], EMPTY_ARRIVALS);
            mbar_init(&bars->x_full[s], XWARPS);
        }
        for (int b = 0; b < NA; ++b) { mbar_init(&bars->a_full[b], DWARPS); mbar_init(&bars->a_empty[b], 1); }
        for (int b = 0; b < ND; ++b) { mbar_init(&bars->d_full[b], 1); mbar_init(&bars->d_empty[b], FWARPS); }
        for (int b = 0; b < XS_RING; ++b) mbar_init(&bars->xs_full[b], XWARPS);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
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

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t armed = 0, armed_phase = 0;
            const uint32_t tx = W_BYTES + (uint32_t)p.M * XRAW_ROW;
            UnitPos pos = start;
            for (int i = 0; i < nu; ++i, pos.next(p.upt)) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!mbar_wait(&bars->empty[s], ph ^ 1u, abort_flag, p.status, SITE_PRODUCER)) break;
                uint8_t* st = stages + s * STAGE_BYTES;
                mbar_arrive_expect_tx(&bars->full[s], tx);
                tma_load_2d(st, &tmW, &bars->full[s], pos.t * TILE_N, pos.j * W_ROWS);
                tma_load_2d(st + W_BYTES, &tmX, &bars->full[s], pos.j * UG * GROUP, 0);
                armed |= 1u << s;
                armed_phase = (armed_phase & ~(1u << s)) | (ph << s);
            }
            // every load of this CTA is issued: the next call may launch
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
            // no copy may still be landing when the CTA exits
            for (int s = 0; s < STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = make_idesc(/*s32*/ 2, /*s8*/ 1, /*s8*/ 1, TILE_N, MMA_N);
            bool ok = true, issued = false;
            for (int i = 0; i < nu && ok; ++i) {
                const int s = i % STAGES, ab = i % NA, db = i % ND;
                if (!mbar_wait(&bars->x_full[s], (uint32_t)(i / STAGES) & 1u, abort_flag, p.status, SITE_MMA) ||
                    !mbar_wait(&bars->a_full[ab], (uint32_t)(i / NA) & 1u, abort_flag, p.status, SITE_MMA) ||
                    !mbar_wait(&bars->d_empty[db], ((uint32_t)(i / ND) & 1u) ^ 1u, abort_flag, p.status, SITE_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t xt = smem_u32(stages + s * STAGE_BYTES + XT_OFF);
#pragma unroll
                for (int k = 0; k < GROUP / UMMA_K; ++k)
#pragma unroll
                    for (int g = 0; g < UG; ++g)
                        umma_i8_tmem_a(tmem_base + D_COL0 + db * D_COLS + g * MMA_N,
                                       tmem_base + ab * A_COLS + g * (GROUP / 4) + k * (UMMA_K / 4),
                                       make_sdesc_kmajor_sw128(xt + g * XT_GROUP + k * UMMA_K), IDESC, k > 0 ? 1u : 0u);
                issued = true;
                umma_commit(&bars->d_full[db]);
                umma_commit(&bars->a_empty[ab]);
                umma_commit(&bars->empty[s]);
            }
            if (!ok && issued) {
                umma_commit(&bars->drain);
                mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
            }
        }
    } else if (warp < FW0) {
        // ------------------------------------------------------------ activation staging
        const int xi = threadIdx.x - XW0 * 32;      // 0..127
        const int m = xi >> 3;                      // row 0..15
        const int g = (xi >> 2) & 1;                // group of the unit
        const int qk = xi & 3;                      // 32-element quarter of the group: chunks 2qk, 2qk+1
        // rows M..15 (h) and 16+M..31 (l) of every stage's tiles stay zero for the whole kernel
        if (m >= p.M)
            for (int s = 0; s < STAGES; ++s) {
                uint8_t* xt = stages + s * STAGE_BYTES + XT_OFF + g * XT_GROUP;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    *reinterpret_cast<uint4*>(xt + xt_offset(m, 2 * qk + c)) = make_uint4(0u, 0u, 0u, 0u);
                    *reinterpret_cast<uint4*>(xt + xt_offset(MROWS + m, 2 * qk + c)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
        for (int i = 0; i < nu; ++i) {
            const int s = i % STAGES, slot = i % XS_RING;
            if (!warp_wait(&bars->full[s], (uint32_t)(i / STAGES) & 1u, abort_flag, p.status, SITE_X)) break;
            // every lane runs the shuffles below (rows >= M as zeros), so the
            // full-warp masks hold whatever M is
            const bool live = m < p.M;
            uint4 v[4];
            {
                const uint4* xraw =
                    reinterpret_cast<const uint4*>(stages + s * STAGE_BYTES + W_BYTES + m * XRAW_ROW + g * (GROUP * 2)) + qk * 4;
#pragma unroll
                for (int r = 0; r < 4; ++r) v[r] = live ? xraw[r] : make_uint4(0u, 0u, 0u, 0u);
            }
            // group absmax over the 4 threads of this (row, group)
            uint32_t amax = 0;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t w4[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) amax = max(amax, max(w4[e] & 0x7FFFu, (w4[e] >> 16) & 0x7FFFu));
            }
            amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            // xi = round(x * 2^(13 - E)), E = the absmax's exponent: |xi| <= 2^14.  A
            // group whose absmax is below 2^-113 (or zero) is taken as zero.
            const int ebits = (int)(amax >> 7);
            const bool usable = ebits >= 14;
            const float mul = usable ? __uint_as_float((uint32_t)(127 + 13 + 127 - ebits) << 23) : 0.0f;
            const float scale = usable ? __uint_as_float((uint32_t)(ebits - 13) << 23) : 0.0f;
            int isum = 0;
            uint8_t* xt = stages + s * STAGE_BYTES + XT_OFF + g * XT_GROUP;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const uint4 vv = v[2 * c + rr];
                    const uint32_t w4[4] = {vv.x, vv.y, vv.z, vv.w};
                    int xiv[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // exact scaling by a power of two, then round half to even via the 1.5 * 2^23 shifter
                        const float lo = __uint_as_float(w4[e] << 16) * mul;
                        const float hi = __uint_as_float(w4[e] & 0xFFFF0000u) * mul;
                        xiv[2 * e] = min(__float_as_int(lo + 12582912.0f) - 0x4B400000, 16383);
                        xiv[2 * e + 1] = min(__float_as_int(hi + 12582912.0f) - 0x4B400000, 16383);
                    }
                    uint32_t hb[8], lb[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        isum += xiv[e];
                        hb[e] = (uint32_t)(xiv[e] >> 7) & 0xFFu;   // arithmetic shift: floor
                        lb[e] = (uint32_t)xiv[e] & 0x7Fu;
                    }
                    // K order (x0, x2, x4, x6, x1, x3, x5, x7)
                    hw[2 * rr] = hb[0] | (hb[2] << 8) | (hb[4] << 16) | (hb[6] << 24);
                    hw[2 * rr + 1] = hb[1] | (hb[3] << 8) | (hb[5] << 16) | (hb[7] << 24);
                    lw[2 * rr] = lb[0] | (lb[2] << 8) | (lb[4] << 16) | (lb[6] << 24);
                    lw[2 * rr + 1] = lb[1] | (lb[3] << 8) | (lb[5] << 16) | (lb[7] << 24);
                }
                if (live) {
                    *reinterpret_cast<uint4*>(xt + xt_offset(m, 2 * qk + c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(xt + xt_offset(MROWS + m, 2 * qk + c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
            }
            isum += __shfl_xor_sync(0xffffffffu, isum, 1);
            isum += __shfl_xor_sync(0xffffffffu, isum, 2);
            if (qk == 0) {
                xscale[(slot * UG + g) * MROWS + m] = scale;
                xsum[(slot * UG + g) * MROWS + m] = (float)isum;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // tiles visible to the MMA
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars->x_full[s]);
                mbar_arrive(&bars->xs_full[slot]);
                mbar_arrive(&bars->empty[s]);
            }
        }
    } else if (warp < DW0) {
        // ------------------------------------------------------------ fold
        const int q = warp & 3;                     // TMEM lane quarter
        const int n_local = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        float y[MROWS];
#pragma unroll
        for (int m = 0; m < MROWS; ++m) y[m] = 0.0f;

        auto publish = [&](int t) {
            const int n = t * TILE_N + n_local;
            const long long gu = (long long)t * p.upt;
            const int first = owner(gu, p.units, ctas);
            const int np = owner(gu + p.upt - 1, p.units, ctas) - first + 1;
            auto store = [&](const float* v) {
                if (n >= p.N) return;
#pragma unroll
                for (int m = 0; m < MROWS; ++m) {
                    if (m >= p.M) break;
                    if (p.out_type == QG_OUT_F32) static_cast<float*>(p.Y)[(size_t)m * p.N + n] = v[m];
                    else static_cast<__nv_bfloat16*>(p.Y)[(size_t)m * p.N + n] = __float2bfloat16_rn(v[m]);
                }
            };
            if (np == 1) {
                store(y);
            } else {
                const int piece = (int)blockIdx.x - first;
                float* dst = p.ws + (((size_t)t * p.maxp + piece) * SLICES + q) * (MROWS * 32);
#pragma unroll
                for (int m = 0; m < MROWS; ++m) dst[m * 32 + lane] = y[m];
                __threadfence();
                __syncwarp();
                unsigned int tk = 0;
                if (lane == 0) tk = atomicAdd(p.tickets + (size_t)t * SLICES + q, 1u);
                tk = __shfl_sync(0xffffffffu, tk, 0);
                if (tk == (unsigned int)np - 1) {
                    __threadfence();
                    float acc[MROWS];
#pragma unroll
                    for (int m = 0; m < MROWS; ++m) acc[m] = 0.0f;
                    for (int pc = 0; pc < np; ++pc) {
                        const float* src = p.ws + (((size_t)t * p.maxp + pc) * SLICES + q) * (MROWS * 32);
#pragma unroll
                        for (int m = 0; m < MROWS; ++m) acc[m] += __ldcg(src + m * 32 + lane);
                    }
                    store(acc);
                    if (lane == 0) p.tickets[(size_t)t * SLICES + q] = 0;   // ready for the next call
                }
            }
#pragma unroll
            for (int m = 0; m < MROWS; ++m) y[m] = 0.0f;
        };

        // S/Z ring of this warp: [SZ_RING][UG][S: 32 | Z: 32] fp16, filled in unit order
        uint16_t* my_sz = szring + q * SZ_RING * UG * 64;
        UnitPos zpos = start;
        auto fetch_sz = [&](int i) {   // lanes 0-15: scale pairs, 16-31: zero pairs
            if (i < nu) {
                const int w = lane & 15;
                const int n = zpos.t * TILE_N + q * 32 + 2 * w;
#pragma unroll
                for (int g = 0; g < UG; ++g) {
                    const int grp = zpos.j * UG + g;
                    const bool in = n < p.N && grp < p.G;
                    const __half* src = (lane < 16 ? p.S : p.Z) + (in ? (size_t)grp * p.N + n : 0);
                    cp_async_4(my_sz + ((i % SZ_RING) * UG + g) * 64 + (lane >> 4) * 32 + 2 * w, src, in ? 4u : 0u);
                }
                zpos.next(p.upt);
            }
            cp_async_commit();   // one group per unit, empty past the end
        };
        for (int i = 0; i < SZ_AHEAD; ++i) fetch_sz(i);

        UnitPos fpos = start;
        for (int i = 0; i < nu; ++i) {
            fetch_sz(i + SZ_AHEAD);
            const int db = i % ND, slot = i % XS_RING;
            if (!warp_wait(&bars->d_full[db], (uint32_t)(i / ND) & 1u, abort_flag, p.status, SITE_FOLD) ||
                !warp_wait(&bars->xs_full[slot], (uint32_t)(i / XS_RING) & 1u, abort_flag, p.status, SITE_FOLD))
                break;
            tc_fence_after();
            cp_async_wait<SZ_AHEAD>();
            __syncwarp();
#pragma unroll
            for (int g = 0; g < UG; ++g) {
                uint32_t r[32];   // D_h (columns 0-15) and D_l (16-31) of the group
                tmem_ld_32x32b_x32(t_lane + D_COL0 + db * D_COLS + g * MMA_N, r);
                tmem_ld_wait_regs(r);
                const uint16_t* sz = my_sz + ((i % SZ_RING) * UG + g) * 64;
                const float sc = __half2float(__ushort_as_half(sz[lane]));
                const float z = __half2float(__ushort_as_half(sz[32 + lane]));
                const float4* xs4 = reinterpret_cast<const float4*>(xsum + (slot * UG + g) * MROWS);
                const float4* xe4 = reinterpret_cast<const float4*>(xscale + (slot * UG + g) * MROWS);
#pragma unroll
                for (int m4 = 0; m4 < MROWS / 4; ++m4) {
                    const float4 xs = xs4[m4], xe = xe4[m4];
                    const float xsv[4] = {xs.x, xs.y, xs.z, xs.w}, xev[4] = {xe.x, xe.y, xe.z, xe.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int m = 4 * m4 + e;
                        const int sqx = 8 * (int)r[m] + ((int)r[MROWS + m] >> 4);   // sum_k q xi, exact
                        y[m] = fmaf(sc * xev[e], fmaf(-z, xsv[e], (float)sqx), y[m]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->d_empty[db]);
            if (fpos.j == p.upt - 1 || i == nu - 1) publish(fpos.t);
            fpos.next(p.upt);
        }
        cp_async_wait<0>();
    } else {
        // ------------------------------------------------------------ dequant (two teams)
        const int team = (warp - DW0) / DWARPS;
        const int q = warp & 3;                     // TMEM lane quarter = columns 32q .. 32q+31
        const int h = ((warp - DW0) % DWARPS) >> 2; // packed rows 8h .. 8h+7 of each group
        const int n_local = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int i = team; i < nu; i += TEAMS) {
            const int s = i % STAGES, ab = i % NA;
            if (!warp_wait(&bars->full[s], (uint32_t)(i / STAGES) & 1u, abort_flag, p.status, SITE_DEQ) ||
                !warp_wait(&bars->a_empty[ab], ((uint32_t)(i / NA) & 1u) ^ 1u, abort_flag, p.status, SITE_DEQ))
                break;
            tc_fence_after();
#pragma unroll
            for (int g = 0; g < UG; ++g) {
                const uint32_t* wsm =
                    reinterpret_cast<const uint32_t*>(stages + s * STAGE_BYTES) + (g * 16 + 8 * h) * TILE_N + n_local;
                uint32_t a[16];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t w = wsm[j * TILE_N];
                    a[2 * j] = ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;   // 16 q of k = 8kw + 0, 2, 4, 6
                    a[2 * j + 1] = (w & 0xF0F0F0F0u) ^ 0x80808080u;      // 16 q of k = 8kw + 1, 3, 5, 7
                }
                tmem_st_32x32b_x16(t_lane + ab * A_COLS + g * (GROUP / 4) + 16 * h, a);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars->a_full[ab]);
                mbar_arrive(&bars->empty[s]);
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

struct Shape {
    int tiles, G, upt, ctas, maxp;
    long long units;
};

static Shape shape_of(int N, int K) {
    Shape s;
    s.tiles = (N + TILE_N - 1) / TILE_N;
    s.G = K / GROUP;
    s.upt = (s.G + UG - 1) / UG;
    s.units = (long long)s.tiles * s.upt;
    s.ctas = s.units < kGemvSms ? (int)s.units : kGemvSms;
    s.maxp = 1;
    for (int t = 0; t < s.tiles; ++t) {
        const long long gu = (long long)t * s.upt;
        const int np = owner(gu + s.upt - 1, s.units, s.ctas) - owner(gu, s.units, s.ctas) + 1;
        if (np > s.maxp) s.maxp = np;
    }
    return s;
}

} // namespace w4tc

uint64_t gemv_w4a16_tc_partial_bytes(int N, int K) {
    const w4tc::Shape s = w4tc::shape_of(N, K);
    return (uint64_t)s.tiles * s.maxp * w4tc::SLICES * w4tc::MROWS * 32 * 4;
}

uint64_t gemv_w4a16_tc_ticket_count(int N) { return (uint64_t)((N + w4tc::TILE_N - 1) / w4tc::TILE_N) * w4tc::SLICES; }

int gemv_w4a16_tc(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                  int K, float* partials, unsigned int* tickets, cudaStream_t stream) {
    QG_CHECK_ARG(mrows >= 1 && mrows <= w4tc::MROWS, "gemv_w4a16_tc: %d rows (1..16)", mrows);
    DeviceStatus* status = nullptr;
    int rc = device_status_ptr(&status);
    if (rc) return rc;
    CUtensorMap tmW, tmX;
    if ((rc = make_tmap_2d(&tmW, W, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)N, (uint64_t)K / 8, (uint64_t)N * 4,
                           w4tc::TILE_N, w4tc::W_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if ((rc = make_tmap_2d(&tmX, X, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)K, (uint64_t)mrows, (uint64_t)K * 2,
                           w4tc::UG * w4tc::GROUP, (uint32_t)mrows, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(w4tc::gemv_w4a16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     w4tc::SMEM_BYTES));
        attr_set[dev & 63] = true;
    }
    const w4tc::Shape s = w4tc::shape_of(N, K);
    w4tc::Params p;
    p.S = static_cast<const __half*>(S);
    p.Z = static_cast<const __half*>(Z);
    p.Y = Y;
    p.ws = partials;
    p.tickets = tickets;
    p.M = mrows;
    p.N = N;
    p.K = K;
    p.G = s.G;
    p.upt = s.upt;
    p.units = s.units;
    p.maxp = s.maxp;
    p.out_type = out_type;
    p.status = status;
    QG_CUDA(launch_pdl(w4tc::gemv_w4a16_tc_kernel, dim3(s.ctas), dim3(w4tc::THREADS), (size_t)w4tc::SMEM_BYTES, stream,
                       tmW, tmX, p));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace qg
