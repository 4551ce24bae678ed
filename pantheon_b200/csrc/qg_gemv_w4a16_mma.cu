// qg_gemv_w4a16_mma.cu -- W4A16 group-128 skinny GEMM for 2..12 activation
// rows on register-fed warp MMAs (mma.sync m16n8k32, u8 x s8 -> s32).
//
//   Y[m, n] = sum_k X[m, k] * (q[k, n] - Z[k/128, n]) * S[k/128, n],  q = u - 8
//
// Same operands as the other GEMV kernels: X bf16 [M, K]; W uint32 [K/8, N]
// (nibble j of word (k8, n) is u(8*k8 + j, n)); S, Z fp16 [K/128, N]; Y bf16
// or fp32 [M, N].
//
// Why warp MMAs.  At 2..12 rows the call is a 117 MB weight stream (configs[3]:
// K = 8192, N = 28672) with M multiply-adds per weight: the FP32 pipes cannot
// keep up, so the products go to tensor cores, but only ~100 TOPS of them.
// The warp-level MMA takes both operands from registers, so each weight goes
// global -> shared -> register -> MMA in the thread that copied it, with no
// TMEM round trip, no single issuing thread and no barrier between producer
// and consumer roles (the tcgen05 kernel, qg_gemv_w4a16_tc.cu, spends most of
// its time in those hand-offs).  Measured on this part the warp MMA sustains
// 0.5 m16n8k32 per clock per SM (~1.1 POPS int8).  Each 4 rows add 2 MMAs
// per lane quad and K step (below); past 12 rows the tcgen05 kernel takes
// over (per call at configs[3]: 12 rows 33.0 us here against 43.2 there; a
// 16-row build of this kernel, four fragments, 43.4 against 43.4, and with a
// 4-deep ring, whose activations no longer fit one wave, 57.3).
//
// Integer arithmetic, exact up to the fold -- the same per-group numbers as
// the tcgen05 kernel:
// * weights: the unsigned nibble u itself is the MMA's u8 A element, one LOP3
//   (low nibbles) or shift + LOP3 (high nibbles) per four weights;
// * activations: per (row, group) 14-bit fixed point x = xi * 2^e (the group's
//   absmax below 2^14, xi clamped to 2^14 - 1), split into s8 digits
//   xi = 128 h + l, h in [-128, 127], l in [0, 127], quantised by each CTA for
//   its own groups straight into the MMA's B-fragment register order in
//   shared memory;
// * per group the MMAs give C_h = sum u h and C_l = sum u l - 8 sum xi (the
//   l accumulator starts at -8 sum xi), so sum_k q xi = 128 C_h + C_l exactly
//   (|.| <= 2^24), and the fold is y += (s * 2^e) * (sum q xi - z * sum xi),
//   rounded as fmaf(s * 2^e, fmaf(-z, sum xi, sum q xi), y).
//
// MMA mapping (PTX fragment layouts of m16n8k32): A = 16 weight columns x 32 K,
// B = 32 K x 8 "digit rows", D = 16 x 8 int32.  Lane (g, t) = (lane / 4,
// lane % 4) copies one 16-byte word quad per K step: packed row 4s + t of the
// step, columns 4g .. 4g+3 of its warp's 32.  Columns 4g, 4g+1 are A rows g,
// g+8 of the first MMA and 4g+2, 4g+3 those of the second.  A row's registers
// hold K = 4t..4t+3 and 16+4t..16+4t+3 of the step; the kernel lets them be the
// word's low nibbles (k = 8t + 0, 2, 4, 6) and high nibbles (k = 8t + 1, 3, 5,
// 7), and the activation digits are written in that same K order, which
// leaves every dot product unchanged.  Digit row 2r of B fragment b is the h
// digit of activation row 4b + r and digit row 2r + 1 its l digit, so the
// accumulator pair (c0, c1) of lane (g, t) is (C_h, C_l) of activation row
// 4b + t and one weight column: the fold needs no data exchange between lanes.
// NB = 1, 2 or 3 B fragments serve up to 4, 8 or 12 rows: 2 NB MMAs per
// lane quad and K step.
//
// Work split.  A super-tile is 512 columns (16 warps x 32); an iteration is one
// (super-tile, group) pair, and the iterations, super-tile-major, are cut into
// one contiguous range per CTA (one CTA per SM, one wave when the activations
// of a range fit in shared memory, else as many waves as make them fit).  All
// warps of a CTA walk the same iterations, each on its own 32 columns, so the
// CTA quantises the activations of its groups once, at start, and every warp
// reads them from shared memory.  Each warp streams its weights, scales and
// zero points through its own cp.async ring, RING groups deep, with no
// synchronisation with other warps.  A super-tile whose iterations span
// several CTAs is reduced through the workspace with a ticket per
// (super-tile, warp): the last CTA to finish sums the pieces in order, so the
// result is bit-for-bit reproducible.
//
// One launch per call.  The kernel has no spin-waits: cp.async groups and
// __syncthreads are its only waits.
#include "qg_common.cuh"
#include "qg_check.cuh"
#include "qg_gemv.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qg {
namespace w4mma {

constexpr int GROUP = 128;                    // K per group (one scale / zero point)
constexpr int STEPS = GROUP / 32;             // MMA K steps per group
constexpr int WARPS = 16;                     // per CTA, one CTA per SM
constexpr int THREADS = WARPS * 32;
constexpr int WCOLS = 32;                     // weight columns per warp
constexpr int ST_COLS = WARPS * WCOLS;        // columns per super-tile
constexpr int STEP_BYTES = 512;               // a warp's W of one K step: 4 packed rows x 128 B
constexpr int W_SLOT = STEPS * STEP_BYTES;    // ... of one group
constexpr int SZ_SLOT = 128;                  // 8 column quads x (4 scales, 4 zero points) fp16
constexpr int SLOT = W_SLOT + SZ_SLOT;
constexpr int SMEM_BUDGET = 227 * 1024;

template <int NB>
struct Cfg {
    static_assert(NB >= 1 && NB <= 3, "1 to 3 B fragments");
    static constexpr int MR = 4 * NB;                        // activation rows, padded
    static constexpr int XF_STEP = NB * 256;                 // B fragments of one K step
    static constexpr int XS_OFF = STEPS * XF_STEP;           // then per (t, b): {2^e, sum xi, 8 sum xi, 0}
    static constexpr int XG = XS_OFF + 4 * NB * 16;          // prepared bytes per group
    // Weight ring depth per warp (groups copied ahead of the one computed).
    // Measured at configs[3]: 3 instead of 5 at one fragment cost 2 %, 5 or 3
    // instead of 4 at two fragments 2 % and 0.4 % (5: fewer registers for the
    // rest); at three fragments 3 measured 1 % faster than 4 and leaves room
    // to stage the activations of a CTA's whole range (one wave).
    static constexpr int RING = NB == 1 ? 5 : (NB == 2 ? 4 : 3);
    static constexpr int RING_BYTES = WARPS * RING * SLOT;
    static constexpr int XMAX = (SMEM_BUDGET - RING_BYTES) / XG;   // groups of activations a CTA can stage
    static_assert(XG % 16 == 0 && RING_BYTES % 16 == 0, "16-byte copies");
    static_assert(XMAX >= 8, "shared-memory budget");
};

// Byte offset of lane `lane`'s 8 bytes of B fragment b inside one K step.
// Fragments go in pairs: a lane reads both of a pair with one 16-byte load,
// and 32 lanes x 16 bytes are contiguous (no bank conflicts); an odd last
// fragment follows as 32 lanes x 8 bytes.
template <int NB>
__host__ __device__ __forceinline__ int frag_offset(int b, int lane) {
    return (NB & 1) && b == NB - 1 ? (NB - 1) * 256 + lane * 8 : (b >> 1) * 512 + lane * 16 + (b & 1) * 8;
}

struct Params {
    const __nv_bfloat16* X;
    const uint32_t* W;
    const __half* S;
    const __half* Z;
    void* Y;
    float* ws;               // [nst][maxp][WARPS][32 lanes][4 NB] fp32 partials
    unsigned int* tickets;   // [nst][WARPS], zero between calls
    const void* golden;      // checked launch: the golden Y (same layout), or null
    unsigned long long* check_count;
    int M, N, K, G, nst;
    long long iters;         // nst * G
    int ctas, maxp, out_type;
    int early_w;             // QG_GEMV_WEIGHTS_CONST: first weight loads before the dependency wait
    int early_x;             // QG_GEMV_ACTIVATIONS_CONST: activations quantised before the dependency wait
};

// The CTA whose iteration range [c*I/C, (c+1)*I/C) holds iteration i.
__host__ __device__ __forceinline__ int owner(long long i, long long iters, int ctas) {
    return (int)(((i + 1) * ctas - 1) / iters);
}

// 16-byte global -> shared copy; src_bytes 0 writes zeros (src is then not read).
__device__ __forceinline__ void cp_async_16z(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = a b + (0, c_odd, 0, c_odd): the first K step of a group, whose h
// accumulators (c0, c2) start at zero and l accumulators (c1, c3) at c_odd.
__device__ __forceinline__ void mma_u8s8_init(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c_odd) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%10, %11, %10, %11};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(c_odd));
}

// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1) and (d0, d1) = (a0, a1) * (b0, b1),
// two fp32 lanes per instruction, each rounded as its scalar form.
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

// The activations of `xcount` groups (group q is `xall ? q : (grp0 + q) % G`)
// quantised into the CTA's shared memory in B-fragment order.  Task (q, row m,
// step s) quantises 32 activations; the four steps of a row are adjacent
// lanes (absmax and sum by shuffles).  Rows >= M come out as zero digits with
// zero scales.  Every round's loads are issued before any is used.
template <int NB>
__device__ __forceinline__ void prep_x(const Params& p, uint8_t* xsm, int xcount, bool xall, int grp0) {
    using C = Cfg<NB>;
    constexpr int TPG = C::MR * STEPS;                       // tasks per group
    constexpr int ROUNDS = (C::XMAX * TPG + THREADS - 1) / THREADS;
    const int ntask = xcount * TPG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint4 v[ROUNDS][4];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        const int tau = r * THREADS + threadIdx.x;
        const int q = tau / TPG, m = (tau % TPG) / STEPS, s = tau % STEPS;
        int grp = q;
        if (!xall) { grp = grp0 + q; if (grp >= p.G) grp -= p.G; }
        const bool live = tau < ntask && m < p.M;
        const uint4* src = reinterpret_cast<const uint4*>(p.X + (live ? (size_t)m * p.K + (size_t)grp * GROUP + s * 32 : 0));
#pragma unroll
        for (int i = 0; i < 4; ++i) v[r][i] = live ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        if (r * THREADS + warp * 32 >= ntask) break;   // warp-uniform: no task of this warp is left
        const int tau = r * THREADS + threadIdx.x;
        const bool active = tau < ntask;               // whole lane quads are active or not
        const int q = tau / TPG, m = (tau % TPG) / STEPS, s = tau % STEPS;
        // group absmax: |x| bits of both halves of each word at once (packed 16-bit max)
        uint32_t am2 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w4[4] = {v[r][i].x, v[r][i].y, v[r][i].z, v[r][i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) am2 = __vmaxu2(am2, w4[e] & 0x7FFF7FFFu);
        }
        uint32_t amax = max(am2 & 0xFFFFu, am2 >> 16);
        amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        // xi = round(x * 2^(13 - E)), E = the absmax's exponent: |xi| <= 2^14.  A
        // group whose absmax is below 2^-113 (or zero) is taken as zero.
        const int ebits = (int)(amax >> 7);
        const bool usable = ebits >= 14;
        const float mul = usable ? __uint_as_float((uint32_t)(127 + 13 + 127 - ebits) << 23) : 0.0f;
        const float scale = usable ? __uint_as_float((uint32_t)(ebits - 13) << 23) : 0.0f;
        // Rounding through the 1.5 * 2^23 shifter: x * mul is exact (a power of
        // two), so fmaf(x, mul, 1.5 * 2^23) rounds it half to even and leaves
        // bits = 0x4B400000 + xi, with 0x4B400000 a multiple of 2^22: bits 0-6
        // are l and bits 7-14 are h = xi >> 7 (two's complement), and the
        // clamp of xi to 2^14 - 1 is an integer min on the bits.
        constexpr float kShift = 12582912.0f;
        constexpr int kBase = 0x4B400000;
        int bsum = 0;   // sum of the bits words: isum = bsum - 32 kBase (mod 2^32, exact)
        uint8_t* xstep = xsm + (size_t)q * C::XG + s * C::XF_STEP;
        const int b = m >> 2, nh = 2 * (m & 3);   // B fragment; digit rows nh (h) and nh + 1 (l)
#pragma unroll
        for (int i = 0; i < 4; ++i) {   // k = 8i .. 8i+7 of the step: lane (digit row, t = i)
            const uint32_t w4[4] = {v[r][i].x, v[r][i].y, v[r][i].z, v[r][i].w};
            uint32_t bits[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                bits[2 * e] = (uint32_t)min(__float_as_int(fmaf(__uint_as_float(w4[e] << 16), mul, kShift)), kBase + 16383);
                bits[2 * e + 1] =
                    (uint32_t)min(__float_as_int(fmaf(__uint_as_float(w4[e] & 0xFFFF0000u), mul, kShift)), kBase + 16383);
                bsum += (int)(bits[2 * e] + bits[2 * e + 1]);
            }
            // the low bytes of four words, in order, as one word
            auto pack4 = [](uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
                return __byte_perm(__byte_perm(a0, a1, 0x0040), __byte_perm(a2, a3, 0x0040), 0x5410);
            };
            // register 0: k = 8i + 0, 2, 4, 6; register 1: k = 8i + 1, 3, 5, 7
            if (active) {
                *reinterpret_cast<uint2*>(xstep + frag_offset<NB>(b, 4 * nh + i)) =
                    make_uint2(pack4(bits[0] >> 7, bits[2] >> 7, bits[4] >> 7, bits[6] >> 7),
                               pack4(bits[1] >> 7, bits[3] >> 7, bits[5] >> 7, bits[7] >> 7));
                *reinterpret_cast<uint2*>(xstep + frag_offset<NB>(b, 4 * (nh + 1) + i)) =
                    make_uint2(pack4(bits[0], bits[2], bits[4], bits[6]) & 0x7F7F7F7Fu,
                               pack4(bits[1], bits[3], bits[5], bits[7]) & 0x7F7F7F7Fu);
            }
        }
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
        const int isum = (int)((uint32_t)bsum - (uint32_t)(GROUP * kBase));
        if (active && s == 0)
            *(reinterpret_cast<int4*>(xsm + (size_t)q * C::XG + C::XS_OFF) + ((m & 3) * NB + b)) =
                make_int4(__float_as_int(scale), __float_as_int((float)isum), 8 * isum, 0);
    }
}

template <int NB>
__global__ void __launch_bounds__(THREADS, 1)
gemv_w4a16_mma_kernel(Params p) {
    using C = Cfg<NB>;
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem + warp * (C::RING * SLOT);
    uint8_t* xsm = smem + C::RING_BYTES;
    const long long i0 = (long long)blockIdx.x * p.iters / p.ctas;
    const long long i1 = (long long)(blockIdx.x + 1) * p.iters / p.ctas;
    const int nit = (int)(i1 - i0);
    const int st0 = (int)(i0 / p.G), grp0 = (int)(i0 % p.G);
    const bool xall = nit >= p.G;   // the range covers every group: stage them by group index
    const int wcol = warp * WCOLS + 4 * g;   // this lane's first column inside a super-tile
    // Where the lane's 16 bytes of a K step sit in shared memory: packed row t
    // keeps its own 128-byte line (each copy of a warp's 128-byte global
    // segment stays inside one line; spreading a segment over four lines
    // measured 40 % slower), and its 16-byte chunks are XOR-swizzled, g ^ 2t,
    // so the eight lanes of a quarter-warp read eight different bank groups.
    const int woff = t * 128 + ((g ^ (2 * t)) << 4);
    const size_t N = (size_t)p.N;

    // Weights, scales and zero points of the next iteration to copy (super-tile
    // ast, group agrp) into ring slot islot: each lane copies its own word quad
    // of every K step (and reads back only those), and one quarter of its
    // column quad's scales / zero points.  Positions, slots and source
    // addresses advance by additions (a division or modulo per iteration
    // measured 1.3 % slower at 8 rows).
    int ast = st0, agrp = grp0, islot = 0;
    const uint32_t* wsrc = nullptr;
    const __half* zsrc = nullptr;
    bool ain = false;   // this lane's column quad lies inside N (N % 4 == 0: wholly in or out)
    auto aim = [&]() {
        const int col = ast * ST_COLS + wcol;
        ain = col < p.N;
        wsrc = p.W + (size_t)(agrp * (GROUP / 8) + t) * N + (ain ? col : 0);
        zsrc = ((t >> 1) ? p.Z : p.S) + (ain ? (size_t)agrp * N + col + 2 * (t & 1) : 0);
    };
    aim();
    auto issue = [&]() {
        uint8_t* dst = ring + islot * SLOT;
#pragma unroll
        for (int s = 0; s < STEPS; ++s)
            cp_async_16z(dst + s * STEP_BYTES + woff, wsrc + (size_t)(4 * s) * N, ain ? 16u : 0u);
        cp_async_4(dst + W_SLOT + g * 16 + t * 4, zsrc, ain ? 4u : 0u);
        if (++islot == C::RING) islot = 0;
        if (++agrp == p.G) {
            agrp = 0;
            ++ast;
            aim();
        } else if (ain) {
            wsrc += (size_t)(GROUP / 8) * N;
            zsrc += N;
        }
    };

    // Prologue: the first RING - 1 groups, and the activations.  Launched with
    // programmatic stream serialization, this CTA may be resident before the
    // previous kernel on the stream has finished, so nothing global is read or
    // written before griddepcontrol.wait -- except what the caller declares
    // that kernel does not write: the first weight copies (W, S, Z constant)
    // and the quantisation of X into shared memory (X constant), which then
    // overlap the previous call's tail (1.2-1.9 us per call at 2-8 rows for the
    // activations).  Y, the partial sums and the tickets are touched only after
    // the wait.
    auto prologue = [&]() {
#pragma unroll
        for (int j = 0; j < C::RING - 1; ++j) {
            if (j < nit) issue();
            cp_async_commit();
        }
    };
    if (p.early_w) prologue();
    if (p.early_x) prep_x<NB>(p, xsm, xall ? p.G : nit, xall, grp0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!p.early_w) prologue();
    if (!p.early_x) prep_x<NB>(p, xsm, xall ? p.G : nit, xall, grp0);
    // every CTA of this grid has started: the next kernel may launch (it waits
    // for this grid to complete before touching anything this one reads or
    // writes, and its CTAs take SMs only as these exit)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __syncthreads();

    float y[4][NB];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int b = 0; b < NB; ++b) y[c][b] = 0.0f;
    uint32_t bad = 0;   // checked launch: output words of this lane that differ from the golden run

    // Write one super-tile's results of this lane: columns col .. col+3 of
    // activation rows 4b + t.  In a checked launch each stored word is
    // compared with the golden output.
    auto store = [&](int col, const float (&v)[4][NB]) {
        if (col >= p.N) return;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const int m = 4 * b + t;
            if (m >= p.M) continue;
            const size_t i = (size_t)m * N + col;
            if (p.out_type == QG_OUT_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(p.Y) + i) = make_float4(v[0][b], v[1][b], v[2][b], v[3][b]);
                if (p.golden) {
                    const uint4 gw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const float*>(p.golden) + i));
                    bad += (gw.x != __float_as_uint(v[0][b])) + (gw.y != __float_as_uint(v[1][b])) +
                           (gw.z != __float_as_uint(v[2][b])) + (gw.w != __float_as_uint(v[3][b]));
                }
            } else {
                __nv_bfloat162 lo = __floats2bfloat162_rn(v[0][b], v[1][b]);
                __nv_bfloat162 hi = __floats2bfloat162_rn(v[2][b], v[3][b]);
                const uint2 w = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.Y) + i) = w;
                if (p.golden) {
                    const uint2 gw = __ldcg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.golden) + i));
                    bad += (gw.x != w.x) + (gw.y != w.y);
                }
            }
        }
    };

    // The end of this CTA's part of super-tile st: store, or leave a partial
    // and let the last of the super-tile's CTAs (ticket) sum the parts in order.
    auto publish = [&](int st) {
        const int col = st * ST_COLS + wcol;
        const long long gi = (long long)st * p.G;
        const int first = owner(gi, p.iters, p.ctas);
        const int np = owner(gi + p.G - 1, p.iters, p.ctas) - first + 1;
        if (np == 1) {
            store(col, y);
        } else {
            const int piece = (int)blockIdx.x - first;
            float4* dst = reinterpret_cast<float4*>(p.ws) + ((((size_t)st * p.maxp + piece) * WARPS + warp) * 32 + lane) * NB;
#pragma unroll
            for (int b = 0; b < NB; ++b) dst[b] = make_float4(y[0][b], y[1][b], y[2][b], y[3][b]);
            __threadfence();
            __syncwarp();
            unsigned int tk = 0;
            if (lane == 0) tk = atomicAdd(p.tickets + (size_t)st * WARPS + warp, 1u);
            tk = __shfl_sync(0xffffffffu, tk, 0);
            if (tk == (unsigned int)np - 1) {
                __threadfence();
                float acc[4][NB];
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int b = 0; b < NB; ++b) acc[c][b] = 0.0f;
                for (int pc = 0; pc < np; ++pc) {
                    const float4* src =
                        reinterpret_cast<const float4*>(p.ws) + ((((size_t)st * p.maxp + pc) * WARPS + warp) * 32 + lane) * NB;
#pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        const float4 v = __ldcg(src + b);
                        acc[0][b] += v.x; acc[1][b] += v.y; acc[2][b] += v.z; acc[3][b] += v.w;
                    }
                }
                store(col, acc);
                if (lane == 0) p.tickets[(size_t)st * WARPS + warp] = 0;   // ready for the next call
            }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int b = 0; b < NB; ++b) y[c][b] = 0.0f;
    };

    int st = st0, grp = grp0;
    int cslot = 0;                                                   // ring slot of iteration j
    const uint8_t* xg = xsm + (size_t)(xall ? grp0 : 0) * C::XG;     // its staged activations
    // One pass of the outer loop per super-tile this CTA touches: its groups
    // grp .. grp + seg - 1 in the inner loop, then the super-tile's publish
    // (checking for the super-tile's end in every iteration, and iterating
    // without the unrolling by two, measured 1-3 % slower).
    for (int j = 0; j < nit;) {
        const int seg = min(p.G - grp, nit - j);
#pragma unroll 2
        for (const int jend = j + seg; j < jend; ++j) {
            // refill the slot iteration j - 1 used: every lane's reads of it
            // (its own weights; the scales and zero points of its column quad,
            // copied by four lanes) are complete past this barrier
            __syncwarp();
            if (j + C::RING - 1 < nit) issue();
            cp_async_commit();
            cp_async_wait<C::RING - 1>();   // this lane's copies of iteration j have landed
            __syncwarp();                   // ... and the other lanes' (scales, zero points)
            const uint8_t* wsl = ring + cslot * SLOT;

            // activation rows 4b + t of this group: 2^e, sum xi, 8 sum xi
            float xe[NB], xsum[NB];
            int nsum8[NB];   // the l accumulators' start value, -8 sum xi
            int acc[2][NB][4];
    #pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int4 v = *reinterpret_cast<const int4*>(xg + C::XS_OFF + (t * NB + b) * 16);
                xe[b] = __int_as_float(v.x);
                xsum[b] = __int_as_float(v.y);
                nsum8[b] = -v.z;
            }
    #pragma unroll
            for (int s = 0; s < STEPS; ++s) {
                const uint4 w = *reinterpret_cast<const uint4*>(wsl + s * STEP_BYTES + woff);
                const uint32_t a0[4] = {w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, (w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu};
                const uint32_t a1[4] = {w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu};
                const uint8_t* xf = xg + s * C::XF_STEP;
                uint32_t bf[NB][2];
    #pragma unroll
                for (int b = 0; b + 1 < NB; b += 2) {
                    const uint4 v = *reinterpret_cast<const uint4*>(xf + frag_offset<NB>(b, lane));
                    bf[b][0] = v.x; bf[b][1] = v.y;
                    bf[b + 1][0] = v.z; bf[b + 1][1] = v.w;
                }
                if constexpr (NB & 1) {
                    const uint2 v = *reinterpret_cast<const uint2*>(xf + frag_offset<NB>(NB - 1, lane));
                    bf[NB - 1][0] = v.x; bf[NB - 1][1] = v.y;
                }
    #pragma unroll
                for (int b = 0; b < NB; ++b) {
                    if (s == 0) {   // the group's first step starts the accumulators at (0, -8 sum xi)
                        mma_u8s8_init(acc[0][b], a0, bf[b][0], bf[b][1], nsum8[b]);
                        mma_u8s8_init(acc[1][b], a1, bf[b][0], bf[b][1], nsum8[b]);
                    } else {
                        mma_u8s8(acc[0][b], a0, bf[b][0], bf[b][1]);
                        mma_u8s8(acc[1][b], a1, bf[b][0], bf[b][1]);
                    }
                }
            }

            // fold: columns 4g + 2a (c0, c1) and 4g + 2a + 1 (c2, c3) of row 4b + t
            {
                const uint4 szv = *reinterpret_cast<const uint4*>(wsl + W_SLOT + g * 16);
                const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&szv.x));
                const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&szv.y));
                const float2 z01 = __half22float2(*reinterpret_cast<const __half2*>(&szv.z));
                const float2 z23 = __half22float2(*reinterpret_cast<const __half2*>(&szv.w));
                const float sc[4] = {s01.x, s01.y, s23.x, s23.y};
                const float nz[4] = {-z01.x, -z01.y, -z23.x, -z23.y};
    #pragma unroll
                for (int a = 0; a < 2; ++a)
    #pragma unroll
                    for (int b = 0; b < NB; ++b) {
                        const float f0 = (float)(128 * acc[a][b][0] + acc[a][b][1]);   // sum q xi, exact
                        const float f1 = (float)(128 * acc[a][b][2] + acc[a][b][3]);
                        float t0, t1, p0, p1;
                        fma_x2(t0, t1, nz[2 * a], nz[2 * a + 1], xsum[b], xsum[b], f0, f1);
                        mul_x2(p0, p1, sc[2 * a], sc[2 * a + 1], xe[b], xe[b]);
                        fma_x2(y[2 * a][b], y[2 * a + 1][b], p0, p1, t0, t1, y[2 * a][b], y[2 * a + 1][b]);
                    }
            }
            if (++cslot == C::RING) cslot = 0;
            xg += C::XG;
        }
        publish(st);
        grp = 0;
        ++st;
        if (xall) xg = xsm;
    }
    cp_async_wait<0>();   // nothing may still be landing when the CTA exits
    if (p.golden) check_count_warp(p.check_count, bad);
}

struct Shape {
    int nst, G, ctas, maxp, xcount;
    long long iters;
    size_t smem;
};

template <int NB>
static Shape shape_of(int N, int K) {
    using C = Cfg<NB>;
    Shape s;
    s.nst = (N + ST_COLS - 1) / ST_COLS;
    s.G = K / GROUP;
    s.iters = (long long)s.nst * s.G;
    // one wave of kGemvSms CTAs unless a CTA's range would hold more groups of
    // activations than shared memory can stage
    const long long per_wave = (long long)kGemvSms * C::XMAX;
    const long long waves = (s.iters + per_wave - 1) / per_wave;
    const long long ctas = waves * kGemvSms;
    s.ctas = (int)(ctas < s.iters ? ctas : s.iters);
    const long long longest = (s.iters + s.ctas - 1) / s.ctas;
    s.xcount = (int)(longest < s.G ? longest : s.G);
    s.smem = (size_t)C::RING_BYTES + (size_t)s.xcount * C::XG;
    s.maxp = 1;
    for (int st = 0; st < s.nst; ++st) {
        const long long gi = (long long)st * s.G;
        const int np = owner(gi + s.G - 1, s.iters, s.ctas) - owner(gi, s.iters, s.ctas) + 1;
        if (np > s.maxp) s.maxp = np;
    }
    return s;
}

static int nb_for(int mrows) { return (mrows + 3) / 4; }   // B fragments for 1..12 rows

template <int NB>
static int launch(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                  int K, float* partials, unsigned int* tickets, unsigned int flags, cudaStream_t stream,
                  const void* golden, unsigned long long* check_count) {
    const Shape s = shape_of<NB>(N, K);
    static bool attr_set[64] = {};
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    if (!attr_set[dev & 63]) {
        QG_CUDA(cudaFuncSetAttribute(gemv_w4a16_mma_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     SMEM_BUDGET));
        attr_set[dev & 63] = true;
    }
    Params p;
    p.X = static_cast<const __nv_bfloat16*>(X);
    p.W = static_cast<const uint32_t*>(W);
    p.S = static_cast<const __half*>(S);
    p.Z = static_cast<const __half*>(Z);
    p.Y = Y;
    p.ws = partials;
    p.tickets = tickets;
    p.golden = golden;
    p.check_count = check_count;
    p.M = mrows;
    p.N = N;
    p.K = K;
    p.G = s.G;
    p.nst = s.nst;
    p.iters = s.iters;
    p.ctas = s.ctas;
    p.maxp = s.maxp;
    p.out_type = out_type;
    p.early_w = (flags & QG_GEMV_WEIGHTS_CONST) ? 1 : 0;
    p.early_x = (flags & QG_GEMV_ACTIVATIONS_CONST) ? 1 : 0;
    QG_CUDA(launch_pdl(gemv_w4a16_mma_kernel<NB>, dim3(s.ctas), dim3(THREADS), s.smem, stream, p));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace w4mma

uint64_t gemv_w4a16_mma_partial_bytes(int mrows, int N, int K) {
    using namespace w4mma;
    const int nb = nb_for(mrows);
    const int maxp = nb == 1 ? shape_of<1>(N, K).maxp : nb == 2 ? shape_of<2>(N, K).maxp : shape_of<3>(N, K).maxp;
    const uint64_t nst = (uint64_t)((N + ST_COLS - 1) / ST_COLS);
    return maxp == 1 ? 0 : nst * maxp * WARPS * 32 * 4 * nb * 4;
}

uint64_t gemv_w4a16_mma_ticket_count(int N) { return (uint64_t)((N + w4mma::ST_COLS - 1) / w4mma::ST_COLS) * w4mma::WARPS; }

int gemv_w4a16_mma(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                   int K, float* partials, unsigned int* tickets, unsigned int flags, cudaStream_t stream,
                   const void* golden, unsigned long long* check_count) {
    QG_CHECK_ARG(mrows >= 1 && mrows <= 12, "gemv_w4a16_mma: %d rows (1..12)", mrows);
    QG_CHECK_ARG(((uintptr_t)partials & 15) == 0, "gemv_w4a16_mma: the partial sums must be 16-byte aligned");
    switch (w4mma::nb_for(mrows)) {
        case 1: return w4mma::launch<1>(X, W, S, Z, Y, out_type, mrows, N, K, partials, tickets, flags, stream, golden, check_count);
        case 2: return w4mma::launch<2>(X, W, S, Z, Y, out_type, mrows, N, K, partials, tickets, flags, stream, golden, check_count);
        default: return w4mma::launch<3>(X, W, S, Z, Y, out_type, mrows, N, K, partials, tickets, flags, stream, golden, check_count);
    }
}

} // namespace qg
