// qg_gemv_w4a16_tc.cu -- W4A16 group-128 skinny GEMM for up to 16 activation
// rows on the sm_100a tensor cores (tcgen05.mma kind::i8, A operand in TMEM);
// the GEMV entry routes 13..16 rows here (2..12 rows run faster on
// register-fed warp MMAs, qg_gemv_w4a16_mma.cu).
//
//   Y[m, n] = sum_k X[m, k] * (q[k, n] - Z[k/128, n]) * S[k/128, n],  q = u - 8
//
// Same operands as the CUDA-core GEMV (qg_gemv_w4a16.cu): X bf16 [M, K];
// W uint32 [K/8, N] (nibble j of word (k8, n) is u(8*k8 + j, n)); S, Z fp16
// [K/128, N]; Y bf16 or fp32 [M, N].
//
// At 13-16 rows a CUDA-core GEMV needs M FMAs per weight (3.8 GFMA per call at
// M = 16, >= 100 us on the FP32 pipes against ~19 us of HBM time), and warp
// MMAs need twice the MMA count of 8 rows (two activation digits x 16 rows =
// 8 m16n8k32 per 32 x 32 weight tile; a 16-row warp-MMA build tied this
// kernel), so the products go to tcgen05 with the weights as the MMA's M side:
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
// Two launches per call (both with programmatic stream serialization):
//   xprep_kernel  quantises X once per call, one CTA per pair of groups: per
//                 (row, group) the 14-bit digits above, written straight into
//                 the MMA's 32-row x 128-byte, 128-byte-swizzled K-major tile
//                 per group (in the MMA's K order, below; rows M..15 and
//                 16+M..31 zero), plus the row's 2^e and sum of xi.  Every unit
//                 of the main kernel used to redo this for its own slab of X
//                 (the largest CUDA-core cost of a unit).
//   gemv kernel   per CTA, 736 threads (23 warps):
//   warp 0      W producer: per unit, a TMA load of the W tile (32 packed rows
//               x 128 columns, no swizzle) into a 4-stage ring (64 KB of W
//               in flight per SM); a stage is free again as soon as the dequant
//               team has turned it into TMEM columns, so the HBM stream does not
//               wait for the MMA or the fold.
//   warp 2      X producer: per unit, the unit's two prepared X tiles (8 KB,
//               hot in L2) copied with per-lane 16-byte cp.async into a
//               10-stage ring freed by the unit's MMA commit, and published
//               X_LAG units later.  Not a TMA copy: the SM's TMA engine serves
//               its copies in order, and an X tile queued behind 128 KB of
//               weight loads arrived ~7 us after issue, which with the ring
//               refilled only after each MMA held the kernel to one unit per
//               ~1500 cycles.
//   warps 7-22  dequant, four teams of 4 taking units in turn (one team's
//               barrier round trips overlap the others'): each warp owns a TMEM
//               lane quarter; lane n turns each word of its column into two
//               TMEM columns of four 16q bytes, written with tcgen05.st as the
//               MMA's A operand.
//   warp 1      TMEM allocator and MMA issuer: per group 4 x tcgen05.mma M=128
//               N=32 K=32 into a 32-column int32 accumulator.
//   warps 3-6   fold, one per lane quarter: per unit, read both groups'
//               accumulators and fold all 16 rows; scales, zero points and the
//               rows' 2^e and sums arrive by cp.async SZ_AHEAD units ahead (a
//               load consumed in its own iteration put an HBM round trip on
//               every unit).
// K order inside each packed word kw: TMEM column 2kw holds k = 8kw + 0, 2, 4,
// 6 and column 2kw+1 holds k = 8kw + 1, 3, 5, 7, so the activation tile stores
// each run of eight as (x0, x2, x4, x6, x1, x3, x5, x7); both operands use the
// same permutation, which leaves the sum over k unchanged.  Groups past K (odd
// K/128) load as zeros and carry zero scales, so they add nothing.
// All barrier waits are bounded (qg_ptx.cuh).
#include "qg_common.cuh"
#include "qg_check.cuh"
#include "qg_gemv.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qg {
namespace w4tc {

constexpr int TILE_N = 128;                   // weight columns per tile = MMA M
constexpr int GROUP = 128;                    // K per group (one scale / zero point)
constexpr int UG = 2;                         // groups per unit
constexpr int MAX_MROWS = 16;                 // activation rows per launch, at most
constexpr int UMMA_K = 32;                    // int8 elements per MMA
constexpr int W_ROWS = UG * GROUP / 8;                    // 32 packed rows
constexpr int W_BYTES = TILE_N * W_ROWS * 4;              // 16 KB
// Ring depths measured (M=16, 4 rotating weight sets): W 4 / 6 / 8 stages with
// X 10 took 48.0 / 48.8 / 49.6 us; under this saturated stream every load,
// L2 hits included, takes ~7 us, so fewer weight bytes in flight shorten the
// queues the X tiles wait in without costing weight bandwidth.
constexpr int W_STAGES = 4;                               // W ring: 64 KB
constexpr int X_STAGES = 10;                              // prepared-X ring: 80 KB at 16 rows
constexpr int X_LAG = 4;                                  // units between an X copy and its publication
static_assert(X_LAG < X_STAGES, "X ring depth");
constexpr int X_RING_OFF = W_STAGES * W_BYTES;
// Four teams of four dequant warps, one unit each in turn (two teams of
// eight took 1-2 % longer at 12 and 16 rows).
constexpr int TEAMS = 4;                      // dequant teams, alternate units
constexpr int NA = 4;                         // A operand buffers in TMEM
constexpr int A_COLS = UG * GROUP / 4;        // 64 columns per unit: 2 x 128 bytes per lane
constexpr int ND = 4;                         // accumulator buffers in TMEM
constexpr int D_COL0 = NA * A_COLS;
// One MMA commit per unit, to mma_done[unit % DONE_RING]: the fold (its
// accumulators), the dequant team (its A buffer, NA units later) and the X
// producer (its X stage, X_STAGES units later) all wait on that one barrier.
// Three commits per unit (one per consumer) slowed the issuing thread by ~20
// cycles per MMA.  The ring is deeper than the MMA can run ahead of any
// waiter (X_STAGES - 1 units), so no waiter sees a barrier two phases on.
constexpr int DONE_RING = 16;
static_assert(DONE_RING > X_STAGES && DONE_RING > NA && DONE_RING > ND, "mma_done ring depth");
constexpr int TMEM_COLS = 512;
static_assert(NA % TEAMS == 0, "each team cycles through its own A buffers");
// Likewise each W stage must belong to one team: with an odd stage count the
// other team would wait on a stage's w_full for a unit two loads ahead, and a
// parity wait that far ahead passes at once (a timing copy with 3 stages read
// W before it landed and failed to launch cleanly).
static_assert(W_STAGES % TEAMS == 0, "each team cycles through its own W stages");
constexpr int SZ_AHEAD = 4;                   // units between an S/Z fetch and its fold
constexpr int SZ_RING = 8;                    // >= SZ_AHEAD + 1
static_assert(SZ_RING >= SZ_AHEAD + 1, "ring depth");
constexpr int XPW = 2;                        // X producer warp
constexpr int FW0 = 3, FWARPS = 4;            // fold warps
constexpr int DW0 = 7, DWARPS = 4;            // dequant warps per team
constexpr int THREADS = (DW0 + TEAMS * DWARPS) * 32;      // 736
static_assert(FW0 + FWARPS == DW0, "the fold warps are the ones between the MMA warp and the dequant teams");
// A warp reaches TMEM lanes 32 * (warp % 4) .. +31 only: the four fold warps and
// each team of four dequant warps are consecutive, so they cover all four.
constexpr int SLICES = FWARPS;                // reduction slices of a tile = lane quarters
constexpr int W_EMPTY_ARRIVALS = DWARPS;      // the dequant team of the unit
constexpr int XPREP_THREADS = 128;            // prepass CTA: 16 rows x 2 groups x 4 quarters
constexpr int SZ_BYTES = FWARPS * SZ_RING * UG * 64 * 2;              // 8 KB: 32 scales + 32 zeros

// Everything that depends on the activation rows a launch carries: MR = 8 for
// 1..8 rows, 16 for 9..16.  At 8 rows the X tiles and the fold's work are half
// the 16-row ones: at M = 8 the kernel took 41.2 us against 47.6 us with
// 16-row tiles (bit-identical results).
template <int MR>
struct Tile {
    static constexpr int MROWS = MR;                      // activation rows, padded
    static constexpr int MMA_N = 2 * MR;                  // h rows, then l rows
    static constexpr int XT_GROUP = MMA_N * GROUP;        // int8 tile per group (2 / 4 KB)
    static constexpr int XT_BYTES = UG * XT_GROUP;        // a unit's two X tiles
    // prepared X per group in the workspace: the tile, then (after all tiles)
    // MR scales 2^e and MR sums of xi per group
    static constexpr int XS_GROUP = 2 * MR;               // floats per group
    static constexpr int D_COLS = UG * MMA_N;             // accumulator columns per unit
    static constexpr int RINGS_BYTES = X_RING_OFF + X_STAGES * XT_BYTES;
    static constexpr int XS_BYTES = FWARPS * SZ_RING * UG * XS_GROUP * 4;   // rows' 2^e and sums
    static_assert(MR == 8 || MR == 16, "8 or 16 activation rows per tile");
    static_assert(XS_GROUP <= 32, "the fold warps fetch a group's 2^e and sums with one 4-byte copy per lane");
    static_assert(X_RING_OFF % 1024 == 0 && XT_GROUP % 1024 == 0, "swizzled tiles need 1 KB alignment");
    static_assert(D_COL0 + ND * D_COLS <= TMEM_COLS, "TMEM budget");
};

constexpr uint32_t SITE_PRODUCER = 0x00040001u;
constexpr uint32_t SITE_MMA = 0x00040002u;
constexpr uint32_t SITE_DEQ = 0x00040004u;
constexpr uint32_t SITE_FOLD = 0x00040005u;

struct Barriers {
    uint64_t w_full[W_STAGES];
    uint64_t w_empty[W_STAGES];
    uint64_t x_full[X_STAGES];
    uint64_t a_full[NA];
    uint64_t d_empty[ND];
    uint64_t mma_done[DONE_RING];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

template <int MR>
constexpr int smem_bytes() {
    return Tile<MR>::RINGS_BYTES + SZ_BYTES + Tile<MR>::XS_BYTES + (int)sizeof(Barriers) + 1024;
}
static_assert(smem_bytes<16>() <= 232448 && smem_bytes<8>() <= 232448, "shared memory budget (227 KB per CTA)");

struct Params {
    const uint8_t* xprep;    // [G2][XT_GROUP] prepared X tiles, then [G2][2][MR] fp32 (2^e, sum xi)
    const __half* S;
    const __half* Z;
    void* Y;
    float* ws;               // [tiles][maxp][SLICES][MR rows][32 lanes] fp32 partials
    unsigned int* tickets;   // [tiles][SLICES], zero between calls
    int M, N, K;
    int G;                   // groups = K / 128
    int upt;                 // units per tile = ceil(G / UG); G2 = UG * upt prepared groups
    long long units;         // tiles * upt
    int maxp;                // most CTAs sharing one tile
    int out_type;
    DeviceStatus* status;
    uint32_t* fp_record;                 // golden launch: per-column fingerprints of Y, or null
    const uint32_t* fp_expect;           // checked launch: the recorded fingerprints, or null
    unsigned long long* check_count;     // checked launch: columns whose fingerprint differs
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

// Two fp32 lanes per instruction, each rounded exactly as its scalar form:
// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1), and (d0, d1) = (a0, a1) * (b0, b1).
__device__ __forceinline__ void fma_x2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                       float c1) {
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 c, a, b, c;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void mul_x2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 a, a, b;\n\t"
        "mov.b64 {%0, %1}, a;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Byte offset of (row, 16-byte chunk) in a 32-row x 128-byte K-major tile with
// the 128-byte swizzle (chunk index XOR row % 8 inside each 8-row atom).
__device__ __forceinline__ int xt_offset(int row, int chunk) {
    return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}

template <int MR>
__global__ void __launch_bounds__(THREADS, 1)
gemv_w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmW, Params p) {
    using T = Tile<MR>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t* wring = smem;
    uint8_t* xring = smem + X_RING_OFF;
    uint16_t* szring = reinterpret_cast<uint16_t*>(smem + T::RINGS_BYTES);
    float* xsring = reinterpret_cast<float*>(smem + T::RINGS_BYTES + SZ_BYTES);
    Barriers* bars = reinterpret_cast<Barriers*>(smem + T::RINGS_BYTES + SZ_BYTES + T::XS_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ctas = gridDim.x;
    const long long u0 = (long long)blockIdx.x * p.units / ctas;
    const long long u1 = (long long)(blockIdx.x + 1) * p.units / ctas;
    const int nu = (int)(u1 - u0);
    const UnitPos start{(int)(u0 / p.upt), (int)(u0 % p.upt)};

    // Launched with programmatic stream serialization after xprep_kernel, whose
    // CTAs trigger this launch only once their own griddepcontrol.wait has
    // returned: when any CTA of this grid runs, every kernel before the pre-pass
    // is complete, so W, S, Z, Y, the workspace and TMEM may be touched at once.
    // Only the pre-pass's output (the prepared X) waits for griddepcontrol.wait
    // (the X producer before its first tile, the fold warps before their first
    // scale fetch).

    if (threadIdx.x == 0) {
        for (int s = 0; s < W_STAGES; ++s) { mbar_init(&bars->w_full[s], 1); mbar_init(&bars->w_empty[s], W_EMPTY_ARRIVALS); }
        for (int s = 0; s < X_STAGES; ++s) mbar_init(&bars->x_full[s], 1);
        for (int b = 0; b < NA; ++b) mbar_init(&bars->a_full[b], DWARPS);
        for (int b = 0; b < ND; ++b) mbar_init(&bars->d_empty[b], FWARPS);
        for (int b = 0; b < DONE_RING; ++b) mbar_init(&bars->mma_done[b], 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmW);
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
        // ------------------------------------------------------------ W producer
        if (lane == 0) {
            uint32_t armed = 0, armed_phase = 0;
            UnitPos pos = start;
            for (int i = 0; i < nu; ++i, pos.next(p.upt)) {
                const int s = i % W_STAGES;
                const uint32_t ph = (uint32_t)(i / W_STAGES) & 1u;
                if (!mbar_wait(&bars->w_empty[s], ph ^ 1u, abort_flag, p.status, SITE_PRODUCER)) break;
                mbar_arrive_expect_tx(&bars->w_full[s], W_BYTES);
                tma_load_2d(wring + s * W_BYTES, &tmW, &bars->w_full[s], pos.t * TILE_N, pos.j * W_ROWS);
                armed |= 1u << s;
                armed_phase = (armed_phase & ~(1u << s)) | (ph << s);
            }
            // every weight load of this CTA is issued: the next call may launch
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
            // no copy may still be landing when the CTA exits
            for (int s = 0; s < W_STAGES; ++s)
                if (armed & (1u << s)) mbar_wait(&bars->w_full[s], (armed_phase >> s) & 1u, nullptr, nullptr, 0);
        }
    } else if (warp == XPW) {
        // ------------------------------------------------------------ X producer (whole warp)
        asm volatile("griddepcontrol.wait;" ::: "memory");   // the pre-pass's tiles
        auto publish_x = [&](int u) {   // unit u's copies have landed (cp.async.wait_group done)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the MMA
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->x_full[u % X_STAGES]);
        };
        UnitPos pos = start;
        int i = 0;
        for (; i < nu; ++i, pos.next(p.upt)) {
            const int s = i % X_STAGES;
            if (i >= X_STAGES) {   // the MMA of the stage's previous unit is complete
                const int j = i - X_STAGES;
                if (!warp_wait(&bars->mma_done[j % DONE_RING], (uint32_t)(j / DONE_RING) & 1u, abort_flag, p.status,
                               SITE_PRODUCER))
                    break;
            }
            const uint8_t* src = p.xprep + (size_t)pos.j * T::XT_BYTES;
            uint8_t* dst = xring + s * T::XT_BYTES;
#pragma unroll
            for (int c = 0; c < T::XT_BYTES / (32 * 16); ++c) cp_async_16(dst + (c * 32 + lane) * 16, src + (c * 32 + lane) * 16);
            cp_async_commit();
            if (i >= X_LAG) {
                cp_async_wait<X_LAG>();
                publish_x(i - X_LAG);
            }
        }
        cp_async_wait<0>();   // nothing may still be landing when the CTA exits
        for (int u = (i > X_LAG ? i - X_LAG : 0); u < i; ++u) publish_x(u);
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = make_idesc(/*s32*/ 2, /*s8*/ 1, /*s8*/ 1, TILE_N, T::MMA_N);
            bool ok = true, issued = false;
            // Ring positions and operand addresses advance by additions only: forming
            // each MMA's descriptors from the unit index (i % X_STAGES, ...) cost the
            // issuing thread ~35 cycles per MMA, about as much as the MMA itself
            // (M=128, N<=64: ~46 cycles).  The descriptor's address field is bits
            // 0-13 (address >> 4), which the shared-memory offsets stay inside.
            const uint64_t x_desc0 = make_sdesc_kmajor_sw128(smem_u32(xring));
            uint64_t x_desc = x_desc0;
            uint32_t a_tm = tmem_base, d_tm = tmem_base + D_COL0;
            int s = 0, ab = 0, db = 0, r = 0;
            uint32_t x_ph = 0, a_ph = 0, d_ph = 1;
            for (int i = 0; i < nu && ok; ++i) {
                if (!mbar_wait(&bars->x_full[s], x_ph, abort_flag, p.status, SITE_MMA) ||
                    !mbar_wait(&bars->a_full[ab], a_ph, abort_flag, p.status, SITE_MMA) ||
                    !mbar_wait(&bars->d_empty[db], d_ph, abort_flag, p.status, SITE_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < GROUP / UMMA_K; ++k)
#pragma unroll
                    for (int g = 0; g < UG; ++g)
                        umma_i8_tmem_a(d_tm + g * T::MMA_N, a_tm + g * (GROUP / 4) + k * (UMMA_K / 4),
                                       x_desc + (uint64_t)((g * T::XT_GROUP + k * UMMA_K) >> 4), IDESC, k > 0 ? 1u : 0u);
                issued = true;
                umma_commit(&bars->mma_done[r]);
                if (++r == DONE_RING) r = 0;
                if (++s == X_STAGES) { s = 0; x_desc = x_desc0; x_ph ^= 1u; } else { x_desc += T::XT_BYTES >> 4; }
                if (++ab == NA) { ab = 0; a_tm = tmem_base; a_ph ^= 1u; } else { a_tm += A_COLS; }
                if (++db == ND) { db = 0; d_tm = tmem_base + D_COL0; d_ph ^= 1u; } else { d_tm += T::D_COLS; }
            }
            if (!ok && issued) {
                umma_commit(&bars->drain);
                mbar_wait(&bars->drain, 0, nullptr, nullptr, 0);
            }
        }
    } else if (warp < DW0) {
        // ------------------------------------------------------------ fold
        asm volatile("griddepcontrol.wait;" ::: "memory");   // the prepared X's scales
        const int q = warp & 3;                     // TMEM lane quarter
        const int n_local = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        float y[T::MROWS];
#pragma unroll
        for (int m = 0; m < T::MROWS; ++m) y[m] = 0.0f;
        uint32_t exp_fp = 0;   // checked launch: the recorded fingerprint of this lane's column

        auto publish = [&](int t) {
            const int n = t * TILE_N + n_local;
            const long long gu = (long long)t * p.upt;
            const int first = owner(gu, p.units, ctas);
            const int np = owner(gu + p.upt - 1, p.units, ctas) - first + 1;
            // every lane of the warp calls store (n past N stores nothing); in a
            // golden or checked launch the stored words of column n are folded
            // into its fingerprint, recorded or compared with `exp_fp`
            auto store = [&](const float* v) {
                uint32_t fp = 0;
                if (n < p.N) {
#pragma unroll
                    for (int m = 0; m < T::MROWS; ++m) {
                        if (m >= p.M) break;
                        const size_t i = (size_t)m * p.N + n;
                        if (p.out_type == QG_OUT_F32) {
                            static_cast<float*>(p.Y)[i] = v[m];
                            fp = fp * kCheckMul + __float_as_uint(v[m]);
                        } else {
                            const __nv_bfloat16 h = __float2bfloat16_rn(v[m]);
                            static_cast<__nv_bfloat16*>(p.Y)[i] = h;
                            fp = fp * kCheckMul + (uint32_t)__bfloat16_as_ushort(h);
                        }
                    }
                }
                if (p.fp_record) {
                    if (n < p.N) p.fp_record[n] = fp;
                } else if (p.fp_expect) {
                    check_count_warp(p.check_count, (n < p.N && fp != exp_fp) ? 1u : 0u);
                }
            };
            if (np == 1) {
                store(y);
            } else {
                const int piece = (int)blockIdx.x - first;
                float* dst = p.ws + (((size_t)t * p.maxp + piece) * SLICES + q) * (T::MROWS * 32);
#pragma unroll
                for (int m = 0; m < T::MROWS; ++m) dst[m * 32 + lane] = y[m];
                __threadfence();
                __syncwarp();
                unsigned int tk = 0;
                if (lane == 0) tk = atomicAdd(p.tickets + (size_t)t * SLICES + q, 1u);
                tk = __shfl_sync(0xffffffffu, tk, 0);
                if (tk == (unsigned int)np - 1) {
                    __threadfence();
                    float acc[T::MROWS];
#pragma unroll
                    for (int m = 0; m < T::MROWS; ++m) acc[m] = 0.0f;
                    for (int pc = 0; pc < np; ++pc) {
                        const float* src = p.ws + (((size_t)t * p.maxp + pc) * SLICES + q) * (T::MROWS * 32);
#pragma unroll
                        for (int m = 0; m < T::MROWS; ++m) acc[m] += __ldcg(src + m * 32 + lane);
                    }
                    store(acc);
                    if (lane == 0) p.tickets[(size_t)t * SLICES + q] = 0;   // ready for the next call
                }
            }
#pragma unroll
            for (int m = 0; m < T::MROWS; ++m) y[m] = 0.0f;
        };

        // S/Z ring of this warp: [SZ_RING][UG][S: 32 | Z: 32] fp16, filled in unit order,
        // and the rows' 2^e and sums: [SZ_RING][UG][2^e: 16 | sum: 16] fp32
        uint16_t* my_sz = szring + q * SZ_RING * UG * 64;
        float* my_xs = xsring + q * SZ_RING * UG * T::XS_GROUP;
        const float* xs_src = reinterpret_cast<const float*>(p.xprep + (size_t)p.upt * UG * T::XT_GROUP);
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
                    if (lane < T::XS_GROUP)   // one float per lane: 2^e of each row, then the sums
                        cp_async_4(my_xs + ((i % SZ_RING) * UG + g) * T::XS_GROUP + lane,
                                   xs_src + (size_t)(zpos.j * UG + g) * T::XS_GROUP + lane, 4u);
                }
                zpos.next(p.upt);
            }
            cp_async_commit();   // one group per unit, empty past the end
        };
        for (int i = 0; i < SZ_AHEAD; ++i) fetch_sz(i);

        UnitPos fpos = start;
        for (int i = 0; i < nu; ++i) {
            if (p.fp_expect && (i == 0 || fpos.j == 0)) {
                // a tile starts: load its column's expected fingerprint now, so the
                // compare at the tile's end does not wait for memory
                const int n = fpos.t * TILE_N + n_local;
                exp_fp = n < p.N ? __ldcg(p.fp_expect + n) : 0u;
            }
            fetch_sz(i + SZ_AHEAD);
            const int db = i % ND;
            if (!warp_wait(&bars->mma_done[i % DONE_RING], (uint32_t)(i / DONE_RING) & 1u, abort_flag, p.status, SITE_FOLD))
                break;
            tc_fence_after();
            cp_async_wait<SZ_AHEAD>();
            __syncwarp();
#pragma unroll
            for (int g = 0; g < UG; ++g) {
                uint32_t r[T::MMA_N];   // D_h (columns 0..MR-1) and D_l (MR..2MR-1) of the group
                if constexpr (MR == 16) tmem_ld_32x32b_x32(t_lane + D_COL0 + db * T::D_COLS + g * T::MMA_N, r);
                else tmem_ld_32x32b_x16(t_lane + D_COL0 + db * T::D_COLS + g * T::MMA_N, r);
                tmem_ld_wait_regs(r);
                const uint16_t* sz = my_sz + ((i % SZ_RING) * UG + g) * 64;
                const float sc = __half2float(__ushort_as_half(sz[lane]));
                const float z = __half2float(__ushort_as_half(sz[32 + lane]));
                const float* xsg = my_xs + ((i % SZ_RING) * UG + g) * T::XS_GROUP;
                const float4* xe4 = reinterpret_cast<const float4*>(xsg);
                const float4* xs4 = reinterpret_cast<const float4*>(xsg + T::MROWS);
#pragma unroll
                for (int m4 = 0; m4 < T::MROWS / 4; ++m4) {
                    const float4 xs = xs4[m4], xe = xe4[m4];
                    const float xsv[4] = {xs.x, xs.y, xs.z, xs.w}, xev[4] = {xe.x, xe.y, xe.z, xe.w};
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {   // rows m, m + 1 as fp32 pairs
                        const int m = 4 * m4 + e;
                        // sum_k q xi, exact (an I2F-free conversion through the 1.5 * 2^23
                        // bit trick, exact for these |D| < 2^21, measured slower)
                        const float f0 = (float)(8 * (int)r[m] + ((int)r[T::MROWS + m] >> 4));
                        const float f1 = (float)(8 * (int)r[m + 1] + ((int)r[T::MROWS + m + 1] >> 4));
                        // y += (sc * 2^e) * (sum q xi - z * sum xi), rounded as the scalar
                        // fmaf(sc * xe, fmaf(-z, xs, f), y)
                        float t0, t1, p0, p1;
                        fma_x2(t0, t1, -z, -z, xsv[e], xsv[e + 1], f0, f1);
                        mul_x2(p0, p1, sc, sc, xev[e], xev[e + 1]);
                        fma_x2(y[m], y[m + 1], p0, p1, t0, t1, y[m], y[m + 1]);
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
        // ------------------------------------------------------------ dequant (four teams)
        const int team = (warp - DW0) / DWARPS;
        const int q = warp & 3;                     // TMEM lane quarter = columns 32q .. 32q+31
        const int n_local = q * 32 + lane;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
        for (int i = team; i < nu; i += TEAMS) {
            const int s = i % W_STAGES, ab = i % NA;
            if (!warp_wait(&bars->w_full[s], (uint32_t)(i / W_STAGES) & 1u, abort_flag, p.status, SITE_DEQ)) break;
            if (i >= NA) {   // the MMA that read this A buffer (unit i - NA) is complete
                const int j = i - NA;
                if (!warp_wait(&bars->mma_done[j % DONE_RING], (uint32_t)(j / DONE_RING) & 1u, abort_flag, p.status,
                               SITE_DEQ))
                    break;
            }
            tc_fence_after();
#pragma unroll
            for (int gh = 0; gh < 2 * UG; ++gh) {   // group g, packed rows 8h .. 8h+7 of it
                const int g = gh >> 1, h = gh & 1;
                const uint32_t* wsm =
                    reinterpret_cast<const uint32_t*>(wring + s * W_BYTES) + (g * 16 + 8 * h) * TILE_N + n_local;
                uint32_t a[16];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t w = wsm[j * TILE_N];
                    a[2 * j] = ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;   // 16 q of k = 8kw + 0, 2, 4, 6
                    a[2 * j + 1] = (w & 0xF0F0F0F0u) ^ 0x80808080u;      // 16 q of k = 8kw + 1, 3, 5, 7
                }
                tmem_st_32x32b_x16(t_lane + ab * A_COLS + g * (GROUP / 4) + 16 * h, a);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->w_empty[s]);   // W is in registers / TMEM now
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->a_full[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// X for one call, prepared once: CTA j quantises groups 2j and 2j + 1 (thread
// xi: row m = xi / 8, group g = (xi / 4) % 2, 32-element quarter qk = xi % 4)
// into the MMA's swizzled tiles and the rows' 2^e and sums.  Rows >= M and
// groups past K come out as zero tiles with zero scales.
template <int MR>
__global__ void __launch_bounds__(XPREP_THREADS)
xprep_kernel(const __nv_bfloat16* __restrict__ X, int M, int K, int G, uint8_t* __restrict__ xprep, int G2,
             int early_x) {
    using T = Tile<MR>;
    // Programmatic stream serialization: X may come from the previous kernel,
    // and the previous GEMV may still be reading the prepared-X area.  So the
    // kernel waits for it before reading X -- or, when the caller declares
    // that the previous kernel does not write X (early_x), quantises X into
    // registers first and waits only before its stores.
    auto wait_previous = []() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    };
    if (!early_x) wait_previous();
    const int xi = threadIdx.x;
    const int m = xi >> 3;                      // row 0..15
    const int g = (xi >> 2) & 1;                // group of the pair
    const int qk = xi & 3;                      // 32-element quarter of the group: chunks 2qk, 2qk+1
    const int grp = blockIdx.x * UG + g;
    const bool live = m < M && grp < G;
    uint4 v[4];
    {
        const uint4* xg = reinterpret_cast<const uint4*>(X + (size_t)(live ? m : 0) * K + (size_t)(live ? grp : 0) * GROUP) + qk * 4;
#pragma unroll
        for (int r = 0; r < 4; ++r) v[r] = live ? __ldg(xg + r) : make_uint4(0u, 0u, 0u, 0u);
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
    uint8_t* xt = xprep + (size_t)grp * T::XT_GROUP;
    uint32_t hw[2][4], lw[2][4];   // per 16-byte chunk c: h and l digit words
#pragma unroll
    for (int c = 0; c < 2; ++c) {
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
            hw[c][2 * rr] = hb[0] | (hb[2] << 8) | (hb[4] << 16) | (hb[6] << 24);
            hw[c][2 * rr + 1] = hb[1] | (hb[3] << 8) | (hb[5] << 16) | (hb[7] << 24);
            lw[c][2 * rr] = lb[0] | (lb[2] << 8) | (lb[4] << 16) | (lb[6] << 24);
            lw[c][2 * rr + 1] = lb[1] | (lb[3] << 8) | (lb[5] << 16) | (lb[7] << 24);
        }
    }
    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
    isum += __shfl_xor_sync(0xffffffffu, isum, 2);
    if (early_x) wait_previous();
    if (m < T::MROWS) {   // an 8-row tile has no rows 8-15 (their threads only join the shuffles)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            *reinterpret_cast<uint4*>(xt + xt_offset(m, 2 * qk + c)) = make_uint4(hw[c][0], hw[c][1], hw[c][2], hw[c][3]);
            *reinterpret_cast<uint4*>(xt + xt_offset(T::MROWS + m, 2 * qk + c)) =
                make_uint4(lw[c][0], lw[c][1], lw[c][2], lw[c][3]);
        }
    }
    if (qk == 0 && m < T::MROWS) {
        float* xs = reinterpret_cast<float*>(xprep + (size_t)G2 * T::XT_GROUP) + (size_t)grp * T::XS_GROUP;
        xs[m] = scale;
        xs[T::MROWS + m] = (float)isum;
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
    return (uint64_t)s.tiles * s.maxp * w4tc::SLICES * w4tc::MAX_MROWS * 32 * 4;   // enough for either tile
}

uint64_t gemv_w4a16_tc_ticket_count(int N) { return (uint64_t)((N + w4tc::TILE_N - 1) / w4tc::TILE_N) * w4tc::SLICES; }

uint64_t gemv_w4a16_tc_xprep_bytes(int K) {
    const int G2 = (K / w4tc::GROUP + w4tc::UG - 1) / w4tc::UG * w4tc::UG;
    return (uint64_t)G2 * (w4tc::Tile<16>::XT_GROUP + w4tc::Tile<16>::XS_GROUP * 4);   // enough for either tile
}

int gemv_w4a16_tc(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                  int K, float* partials, unsigned int* tickets, void* xprep, cudaStream_t stream, uint32_t* fp_record,
                  const uint32_t* fp_expect, unsigned long long* check_count, unsigned int flags) {
    QG_CHECK_ARG(mrows >= 1 && mrows <= w4tc::MAX_MROWS, "gemv_w4a16_tc: %d rows (1..16)", mrows);
    DeviceStatus* status = nullptr;
    int rc = device_status_ptr(&status);
    if (rc) return rc;
    QG_CHECK_ARG(((uintptr_t)xprep & 15) == 0, "gemv_w4a16_tc: prepared-X area must be 16-byte aligned");
    CUtensorMap tmW;
    if ((rc = make_tmap_2d(&tmW, W, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)N, (uint64_t)K / 8, (uint64_t)N * 4,
                           w4tc::TILE_N, w4tc::W_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(w4tc::gemv_w4a16_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     w4tc::smem_bytes<8>()));
        QG_CUDA(cudaFuncSetAttribute(w4tc::gemv_w4a16_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     w4tc::smem_bytes<16>()));
        attr_set[dev & 63] = true;
    }
    const w4tc::Shape s = w4tc::shape_of(N, K);
    w4tc::Params p;
    p.xprep = static_cast<const uint8_t*>(xprep);
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
    p.fp_record = fp_record;
    p.fp_expect = fp_expect;
    p.check_count = check_count;
    // 8-row tiles for up to 8 rows: half the X traffic and fold work of 16-row ones
    const __nv_bfloat16* Xb = static_cast<const __nv_bfloat16*>(X);
    uint8_t* xp = static_cast<uint8_t*>(xprep);
    if (mrows <= 8) {
        QG_CUDA(launch_pdl(w4tc::xprep_kernel<8>, dim3(s.upt), dim3(w4tc::XPREP_THREADS), 0, stream, Xb, mrows, K, s.G, xp,
                           s.upt * w4tc::UG, (flags & QG_GEMV_ACTIVATIONS_CONST) ? 1 : 0));
        QG_CUDA(launch_pdl(w4tc::gemv_w4a16_tc_kernel<8>, dim3(s.ctas), dim3(w4tc::THREADS),
                           (size_t)w4tc::smem_bytes<8>(), stream, tmW, p));
    } else {
        QG_CUDA(launch_pdl(w4tc::xprep_kernel<16>, dim3(s.upt), dim3(w4tc::XPREP_THREADS), 0, stream, Xb, mrows, K, s.G, xp,
                           s.upt * w4tc::UG, (flags & QG_GEMV_ACTIVATIONS_CONST) ? 1 : 0));
        QG_CUDA(launch_pdl(w4tc::gemv_w4a16_tc_kernel<16>, dim3(s.ctas), dim3(w4tc::THREADS),
                           (size_t)w4tc::smem_bytes<16>(), stream, tmW, p));
    }
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace qg
