// qg_gemv_w4a16.cu -- weight-only W4A16 group-128 decode GEMV: the C entry
// points, and the CUDA-core kernel for the single-row decode step
// (bandwidth-bound).  2-12 rows run on warp MMAs (qg_gemv_w4a16_mma.cu), 13-16
// on tcgen05 (qg_gemv_w4a16_tc.cu); larger M is processed 16 rows at a time.
//
//   Y[m, n] = sum_k X[m, k] * (q[k, n] - Z[k/128, n]) * S[k/128, n],  q = u - 8
//
// X bf16 [M, K]; W uint32 [K/8, N] (nibble j of word (k8, n) is u(8*k8 + j, n));
// S, Z fp16 [K/128, N]; Y bf16 or fp32 [M, N].
//
// The weights are read once per call, so the kernel is a stream over W: each
// thread owns CPT adjacent columns and issues non-allocating 64/128-bit loads
// of W (CPT columns x 8 k per load), coalesced across the warp, software-
// pipelined so the loads of the next batch are in flight while the current
// batch is unpacked.  Per group of 128 the group's dot product is folded with
// its scale and zero point:  sum_k x (u - 8 - z) s = s * (sum_k x u - (8 + z) sum_k x).
//
// The inner product sum_k x u is integer: the word's nibbles become bytes with
// one shift and two masks (u0 u2 u4 u6 | u1 u3 u5 u7), the activations of each
// (row, group) are staged as int16 fixed point with a shared power-of-two scale
// (the group's absmax maps below 2^14), and dp2a forms two 16x8-bit products
// per instruction into an exact int32 group accumulator.  The only rounding is
// the activation's, at most 2^-15 of the group absmax per element.
// The sum of the activations of each group is exact fp32 from bf16.
//
// Work split: the K/8 packed rows of a column block are cut into `splits`
// contiguous ranges of (almost) equal length, so the grid is one wave of
// equally sized CTAs; a range may begin or end inside a group, and each group
// segment is folded with its own scale and zero point.  Each CTA writes its
// fp32 partial to the workspace; the last CTA of a column block (atomic
// ticket) sums the partials in split order and writes Y, so the result is
// bit-for-bit reproducible run to run.
//
// The path it sits on in the reference: llm_decode (kernels/llm_decode/
// llm_decode.cpp:28-46, a KV gather + FMA chain with no weights) is the decode
// workload; this kernel is the weight-only quantized projection it is named for.
#include "qg_common.cuh"
#include "qg_check.cuh"
#include "qg_gemv.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

namespace qg {
namespace w4 {

constexpr int THREADS = 128;
constexpr int GROUP = 128;
constexpr int CHUNKS_PER_GROUP = GROUP / 8;
constexpr int MAX_M = 16;    // rows per launch (either kernel)
constexpr int kSplitSms = kGemvSms;
constexpr int CPT = 4;       // columns per thread: one 128-bit load = 4 columns x 8 k

// Per row-count template (1 or 2): resident CTAs per SM (register budget) and
// loads per pipeline half.
__host__ __device__ constexpr int blocks_per_sm(int mt) { return mt == 1 ? 7 : 5; }
__host__ __device__ constexpr int load_depth(int) { return 4; }
__host__ __device__ constexpr int cols_per_cta(int) { return THREADS * CPT; }

struct Params {
    const __nv_bfloat16* X;
    const uint32_t* W;
    const __half* S;
    const __half* Z;
    void* Y;
    float* ws;               // [splits][MT][N] fp32 partials
    unsigned int* tickets;   // [column blocks], zero between calls
    int M, N, K;
    int splits;
    int out_type;
    int early_w;             // QG_GEMV_WEIGHTS_CONST: first weight loads before the dependency wait
    int early_x;             // QG_GEMV_ACTIVATIONS_CONST: with early_w, the whole prologue before the wait
    const void* golden;      // per-launch check: the golden Y (same layout), or null
    unsigned long long* check_count;   // differing output words found
};

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int c) { return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w; }

__device__ __forceinline__ float pow2(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

template <int MT>
__global__ void __launch_bounds__(THREADS, blocks_per_sm(MT))
gemv_w4a16_kernel(Params p) {
    static_assert(MT == 1 || MT == 2, "the kernel is written for 1-2 rows (the GEMV entry uses it for 1)");
    constexpr int DEPTH = load_depth(MT);
    constexpr int CPC = cols_per_cta(MT);
    using VT = uint4;

    const int nchunks = p.K / 8;
    const int c0 = (int)(((long long)blockIdx.y * nchunks) / p.splits);
    const int c1 = (int)(((long long)(blockIdx.y + 1) * nchunks) / p.splits);
    const int len = c1 - c0;
    const int g_first = c0 / CHUNKS_PER_GROUP;
    const int n_groups = (c1 - 1) / CHUNKS_PER_GROUP - g_first + 1;
    const int col0 = blockIdx.x * CPC;

    // Shared memory for this CTA's k range (g = group index within the range):
    //   gsum  fp32  [groups][MT]     sum of the activations of the group segment
    //   gpow  fp32  [groups][MT]     2^e of the segment's fixed point
    //   sz    half2 [groups][CPC]    (scale, zero) of each column
    //   xdat  int32 [len][MT][4]     int16 pairs (x0,x2) (x4,x6) (x1,x3) (x5,x7)
    extern __shared__ __align__(16) uint8_t smem[];
    const int gmax = (len + CHUNKS_PER_GROUP - 1) / CHUNKS_PER_GROUP + 1;
    float* gsum = reinterpret_cast<float*>(smem);
    float* gpow = gsum + gmax * MT;
    __half2* sz = reinterpret_cast<__half2*>(gpow + gmax * MT);
    // 16-byte aligned for the int4 / float4 accesses (the tables above end on a
    // 4-byte boundary; the size computation reserves the padding).
    uint8_t* xdat = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sz + (size_t)gmax * CPC) + 15) &
                                               ~static_cast<uintptr_t>(15));
    int4* xi = reinterpret_cast<int4*>(xdat);

    // The first two batches of weights are requested before anything else, so
    // they stream in while the prologue below stages activations and scales.
    const int n0 = col0 + threadIdx.x * CPT;
    const bool active = n0 < p.N;   // N % 4 == 0, so a thread's columns are wholly in or out
    const size_t row_stride = (size_t)p.N / CPT;                         // VT per packed row
    const VT* wp = reinterpret_cast<const VT*>(p.W) + (size_t)c0 * row_stride + (active ? n0 / CPT : 0);
    VT wa[DEPTH], wb[DEPTH];
    auto load_batch = [&](VT (&dst)[DEPTH], int base) {
#pragma unroll
        for (int d = 0; d < DEPTH; ++d)
            if (base + d < len) dst[d] = ld_stream(wp + (size_t)(base + d) * row_stride);
    };
    // Launched with programmatic stream serialization: this CTA may be resident
    // before the previous kernel on the stream has finished, so nothing global
    // is read or written until that grid is complete (a no-op otherwise) --
    // except what the caller declares the previous kernel does not write: with
    // the weights constant (no W, S, Z) the first weight batches, and with the
    // activations constant as well (no X) the whole prologue below, which
    // reads only W, S, Z and X and writes only shared memory; all of it then
    // overlaps the previous call's tail.
    if (p.early_w && active) {
        load_batch(wa, 0);
        if (DEPTH < len) load_batch(wb, DEPTH);
    }
    // The next call on the stream may launch once every CTA of this one has
    // passed the wait (so all of them are resident: none can be starved of an
    // SM by the next grid); its CTAs take SMs as these exit, and wait for this
    // grid before touching anything it writes.
    const bool early_prologue = p.early_w && p.early_x;
    auto wait_previous = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (!p.early_w && active) {
            load_batch(wa, 0);
            if (DEPTH < len) load_batch(wb, DEPTH);
        }
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    };
    if (!early_prologue) wait_previous();

    // Scales and zero points of this CTA's groups, staged once with 64-bit
    // loads (rows of S and Z are 8-byte aligned because N % 4 == 0): the group
    // folds never wait on a global load mid-stream.
    for (int t = threadIdx.x; t < n_groups * (CPC / 4); t += THREADS) {
        const int g = t / (CPC / 4), c4 = (t - g * (CPC / 4)) * 4;
        const int n = col0 + c4;
        uint2 s4 = make_uint2(0, 0), z4 = make_uint2(0, 0);
        if (n < p.N) {
            s4 = __ldg(reinterpret_cast<const uint2*>(p.S + (size_t)(g_first + g) * p.N + n));
            z4 = __ldg(reinterpret_cast<const uint2*>(p.Z + (size_t)(g_first + g) * p.N + n));
        }
        const __half* sh = reinterpret_cast<const __half*>(&s4);
        const __half* zh = reinterpret_cast<const __half*>(&z4);
#pragma unroll
        for (int j = 0; j < 4; ++j) sz[g * CPC + c4 + j] = __halves2half2(sh[j], zh[j]);
    }
    // Per (group segment, row): exact fp32 sum and absmax of the activations (one warp each).
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int t = warp; t < n_groups * MT; t += THREADS / 32) {
            const int g = t / MT, m = t - g * MT;
            const int ca = max(c0, (g_first + g) * CHUNKS_PER_GROUP);
            const int cb = min(c1, (g_first + g + 1) * CHUNKS_PER_GROUP);
            float s = 0.0f, a = 0.0f;
            if (m < p.M && lane < cb - ca) {   // one packed row (8 activations) per lane, <= 16 rows
                const uint4 raw = *reinterpret_cast<const uint4*>(p.X + (size_t)m * p.K + (size_t)(ca + lane) * 8);
                const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float v0 = __uint_as_float(r4[i] << 16), v1 = __uint_as_float(r4[i] & 0xFFFF0000u);
                    s += v0 + v1;
                    a = fmaxf(a, fmaxf(fabsf(v0), fabsf(v1)));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                s += __shfl_xor_sync(0xffffffffu, s, o);
                a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            }
            if (lane == 0) {
                gsum[g * MT + m] = s;
                // fixed point: the absmax of the segment maps below 2^14 (fits int16 with margin)
                int e = 0;
                if (a > 0.0f) {
                    const int E = (int)((__float_as_uint(a) >> 23) & 0xFF) - 127;
                    e = 13 - E;
                    e = e > 126 ? 126 : (e < -126 ? -126 : e);
                }
                gpow[g * MT + m] = pow2(e);
            }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < len * MT; t += THREADS) {
        const int ch = t / MT, m = t - ch * MT;
        float v[8];
        if (m < p.M) {
            const uint4 raw = *reinterpret_cast<const uint4*>(p.X + (size_t)m * p.K + (size_t)(c0 + ch) * 8);
            const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(r4[i] << 16);
                v[2 * i + 1] = __uint_as_float(r4[i] & 0xFFFF0000u);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        const float sc = gpow[((c0 + ch) / CHUNKS_PER_GROUP - g_first) * MT + m];
        int q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __float2int_rn(v[i] * sc);
        auto pk = [](int lo, int hi) { return (int)(((uint32_t)lo & 0xFFFFu) | ((uint32_t)hi << 16)); };
        xi[(size_t)ch * MT + m] = make_int4(pk(q[0], q[2]), pk(q[4], q[6]), pk(q[1], q[3]), pk(q[5], q[7]));
    }
    __syncthreads();

    if (early_prologue) wait_previous();   // Y and the workspace are written only past this point

    float y[MT][CPT];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < CPT; ++c) y[m][c] = 0.0f;

    if (active) {
        int iacc[CPT][MT];
#pragma unroll
        for (int c = 0; c < CPT; ++c)
#pragma unroll
            for (int m = 0; m < MT; ++m) iacc[c][m] = 0;

        // End of a group segment at packed row i: fold with its scale and zero point.
        auto fold = [&](int i) {
            const int g = (c0 + i) / CHUNKS_PER_GROUP - g_first;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const float2 f = __half22float2(sz[g * CPC + threadIdx.x * CPT + c]);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float corr = -(8.0f + f.y) * gsum[g * MT + m];
                    const float t = fmaf((float)iacc[c][m], 1.0f / gpow[g * MT + m], corr);
                    iacc[c][m] = 0;
                    y[m][c] = fmaf(f.x, t, y[m][c]);
                }
            }
        };

        // One packed row of the CTA's range.
        auto chunk = [&](int i, const VT& wvd) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int4 xw = xi[(size_t)i * MT + m];
#pragma unroll
                for (int c = 0; c < CPT; ++c) {
                    const uint32_t w = word_of(wvd, c);
                    const int b0 = (int)(w & 0x0F0F0F0Fu);          // u0 u2 u4 u6
                    const int b1 = (int)((w >> 4) & 0x0F0F0F0Fu);   // u1 u3 u5 u7
                    int a = iacc[c][m];
                    a = __dp2a_lo(xw.x, b0, a);
                    a = __dp2a_hi(xw.y, b0, a);
                    a = __dp2a_lo(xw.z, b1, a);
                    a = __dp2a_hi(xw.w, b1, a);
                    iacc[c][m] = a;
                }
            }
            if (((c0 + i + 1) % CHUNKS_PER_GROUP) == 0 || i + 1 == len) fold(i);
        };

        // Software pipeline: the loads of batch b + 1 are in flight while batch
        // b is unpacked, so each warp keeps DRAM requests outstanding through
        // its compute phase (ping-pong register buffers, no copies).
        // (batches 0 and 1 were requested before the prologue)
        auto run_batch = [&](const VT (&src)[DEPTH], int base) {
#pragma unroll
            for (int d = 0; d < DEPTH; ++d)
                if (base + d < len) chunk(base + d, src[d]);
        };
        for (int base = 0; base < len; base += 2 * DEPTH) {
            if (base > 0 && base + DEPTH < len) load_batch(wb, base + DEPTH);
            run_batch(wa, base);
            if (base + DEPTH >= len) break;
            if (base + 2 * DEPTH < len) load_batch(wa, base + 2 * DEPTH);
            run_batch(wb, base + DEPTH);
        }
    }

    // ---- publish: directly when K is not split, else partial + ticket.  In a
    // checked launch the writer compares each stored word with the golden output
    // (qg_check.cuh) and `bad` counts the differing words of this thread.
    uint32_t bad = 0;
    auto store_row = [&](int m, const float* v) {
        if (p.out_type == QG_OUT_F32) {
            float* dst = static_cast<float*>(p.Y) + (size_t)m * p.N + n0;
            *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            if (p.golden) {
                const uint4 g = __ldcg(reinterpret_cast<const uint4*>(static_cast<const float*>(p.golden) + (size_t)m * p.N + n0));
                bad += (g.x != __float_as_uint(v[0])) + (g.y != __float_as_uint(v[1])) + (g.z != __float_as_uint(v[2])) +
                       (g.w != __float_as_uint(v[3]));
            }
        } else {
            __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.Y) + (size_t)m * p.N + n0;
            __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
            __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
            const uint32_t wa0 = *reinterpret_cast<uint32_t*>(&a), wb0 = *reinterpret_cast<uint32_t*>(&b);
            *reinterpret_cast<uint2*>(dst) = make_uint2(wa0, wb0);
            if (p.golden) {
                const uint2 g = __ldcg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.golden) + (size_t)m * p.N + n0));
                bad += (g.x != wa0) + (g.y != wb0);
            }
        }
    };
    if (p.splits == 1) {
        if (active)
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < p.M) store_row(m, y[m]);
        if (p.golden) check_count_warp(p.check_count, bad);
        return;
    }
    if (active) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float* dst = p.ws + ((size_t)blockIdx.y * MT + m) * p.N + n0;
            *reinterpret_cast<float4*>(dst) = make_float4(y[m][0], y[m][1], y[m][2], y[m][3]);
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned int ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(p.tickets + blockIdx.x, 1u);
    __syncthreads();
    if (ticket != (unsigned int)p.splits - 1) return;
    __threadfence();
    if (active) {
        for (int m = 0; m < MT && m < p.M; ++m) {
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int sp = 0; sp < p.splits; ++sp) {
                const float* src = p.ws + ((size_t)sp * MT + m) * p.N + n0;
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
                s[0] += v.x; s[1] += v.y; s[2] += v.z; s[3] += v.w;
            }
            store_row(m, s);
        }
    }
    if (p.golden) check_count_warp(p.check_count, bad);
    if (threadIdx.x == 0) p.tickets[blockIdx.x] = 0;   // ready for the next call
}

static int col_blocks_for(int mt, int N) { return (N + cols_per_cta(mt) - 1) / cols_per_cta(mt); }

// Shared-memory bytes for a K range of `len` packed rows (see the kernel's layout).
static size_t smem_bytes_len(int mt, int len) {
    const size_t gmax = (size_t)(len + CHUNKS_PER_GROUP - 1) / CHUNKS_PER_GROUP + 1;
    const size_t per_chunk = (size_t)mt * 16;
    return gmax * mt * 8 + gmax * cols_per_cta(mt) * 4 + (size_t)len * per_chunk + 16;
}
constexpr size_t kSmemBudget = 180 * 1024;

// Equal contiguous K ranges per column block, as many as fill one wave of the
// resident CTAs (at least two packed rows each), and never fewer than keep the
// staged activations within the shared-memory budget.
static int choose_splits(int mt, int N, int K) {
    const int nchunks = K / 8;
    const int slots = kSplitSms * blocks_per_sm(mt);
    int splits = slots / col_blocks_for(mt, N);
    const int max_splits = nchunks / 2;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    while (splits < max_splits && smem_bytes_len(mt, (nchunks + splits - 1) / splits) > kSmemBudget) ++splits;
    return splits;
}

static size_t smem_bytes(int mt, int K, int splits) { return smem_bytes_len(mt, (K / 8 + splits - 1) / splits); }

} // namespace w4

// Row chunks of up to 16 rows, each on the kernel that is fastest for its
// row count (configs[3] shape, per call): 1 row on the CUDA cores (this file;
// the decode step), 2-12 on register-fed warp MMAs (qg_gemv_w4a16_mma.cu:
// 25.1 us at 2 rows against 33.9 us here, where the dp2a work doubles; 33.0
// us at 12 rows against 43.2 on tcgen05), 13-16 on the tcgen05 tensor cores
// (qg_gemv_w4a16_tc.cu).  At 16 rows the warp MMAs need 8 m16n8k32 per
// 32 x 32 weight tile (two activation digits x 16 rows) at 0.5 per clock per
// SM, ~3/4 of the weight stream's time in the MMA pipe alone, and a 16-row
// build of that kernel only tied the tcgen05 one (43.4 us each).
constexpr int kMmaMinRows = 2;
constexpr int kTcMinRows = 13;

enum class Path { kCudaCore, kMma, kTc };
static Path path_for(int mrows) {
    return mrows >= kTcMinRows ? Path::kTc : (mrows >= kMmaMinRows ? Path::kMma : Path::kCudaCore);
}

static uint64_t ticket_bytes(int N) {
    uint64_t most = (uint64_t)((N + 255) / 256);
    const uint64_t counts[2] = {gemv_w4a16_mma_ticket_count(N), gemv_w4a16_tc_ticket_count(N)};
    for (uint64_t c : counts) most = c > most ? c : most;
    return most * 4;
}

// Workspace: fp32 partials for the largest row chunk, the tcgen05 path's
// prepared X (when any chunk takes it), then the tickets (shared by all
// kernels: each leaves them zero).
static uint64_t xprep_bytes(int M, int K) {
    for (int m0 = 0; m0 < M; m0 += w4::MAX_M)
        if (path_for(M - m0 < w4::MAX_M ? M - m0 : w4::MAX_M) == Path::kTc)
            return (gemv_w4a16_tc_xprep_bytes(K) + 255) & ~255ull;
    return 0;
}

uint64_t gemv_w4a16_workspace_bytes(int M, int N, int K, int /*sm_count*/) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    uint64_t partials = 0;
    for (int m0 = 0; m0 < M; m0 += w4::MAX_M) {
        const int mrows = M - m0 < w4::MAX_M ? M - m0 : w4::MAX_M;
        uint64_t ws;
        switch (path_for(mrows)) {
            case Path::kTc: ws = gemv_w4a16_tc_partial_bytes(N, K); break;
            case Path::kMma: ws = gemv_w4a16_mma_partial_bytes(mrows, N, K); break;
            default: ws = (uint64_t)w4::choose_splits(1, N, K) * N * 4;
        }
        if (ws > partials) partials = ws;
    }
    return ((partials + 255) & ~255ull) + xprep_bytes(M, K) + ticket_bytes(N);
}

int gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int M, int N, int K,
               void* workspace, uint64_t workspace_bytes, cudaStream_t stream, unsigned int flags,
               const LaunchCheck& chk, unsigned int* tickets) {
    QG_CHECK_ARG(X && W && S && Z && Y, "qg_gemv_w4a16: null operand");
    QG_CHECK_ARG((flags & ~(unsigned int)(QG_GEMV_WEIGHTS_CONST | QG_GEMV_ACTIVATIONS_CONST)) == 0,
                 "qg_gemv_w4a16: unknown flags 0x%x", flags);
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemv_w4a16: empty shape %dx%dx%d", M, N, K);
    QG_CHECK_ARG(K % w4::GROUP == 0, "qg_gemv_w4a16: K=%d must be a multiple of 128 (group size)", K);
    QG_CHECK_ARG(N % 4 == 0, "qg_gemv_w4a16: N=%d must be a multiple of 4", N);
    QG_CHECK_ARG(out_type == QG_OUT_BF16 || out_type == QG_OUT_F32, "qg_gemv_w4a16: bad out_type %d", out_type);
    QG_CHECK_ARG(((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)S & 7) == 0 &&
                 ((uintptr_t)Z & 7) == 0 && ((uintptr_t)Y & 15) == 0,
                 "qg_gemv_w4a16: X, W, Y must be 16-byte and S, Z 8-byte aligned");
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    const uint64_t need = gemv_w4a16_workspace_bytes(M, N, K, info->sm_count) - (tickets ? ticket_bytes(N) : 0);
    QG_CHECK_ARG(workspace && workspace_bytes >= need,
                 "qg_gemv_w4a16: workspace of %llu bytes needed (got %llu)", (unsigned long long)need,
                 (unsigned long long)workspace_bytes);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const uint64_t tickets_off = need - (tickets ? 0 : ticket_bytes(N));
    const uint64_t xprep_off = tickets_off - xprep_bytes(M, K);
    unsigned int* const tk = tickets ? tickets : reinterpret_cast<unsigned int*>(ws + tickets_off);
    for (int m0 = 0; m0 < M; m0 += w4::MAX_M) {
        const int mrows = (M - m0) < w4::MAX_M ? (M - m0) : w4::MAX_M;
        const size_t y_off = (size_t)m0 * N * (out_type == QG_OUT_F32 ? 4 : 2);
        const void* golden = chk.golden ? static_cast<const uint8_t*>(chk.golden) + y_off : nullptr;
        const Path path = path_for(mrows);
        if (path == Path::kTc) {
            const size_t fp_off = (size_t)(m0 / w4::MAX_M) * N;   // per-column fingerprints of this row chunk
            rc = gemv_w4a16_tc(static_cast<const __nv_bfloat16*>(X) + (size_t)m0 * K, W, S, Z,
                               static_cast<uint8_t*>(Y) + y_off, out_type, mrows, N, K, reinterpret_cast<float*>(ws),
                               tk, ws + xprep_off, stream,
                               chk.record ? chk.record + fp_off : nullptr, chk.expect ? chk.expect + fp_off : nullptr,
                               chk.count, flags);
            if (rc) return rc;
            continue;
        }
        if (path == Path::kMma) {
            rc = gemv_w4a16_mma(static_cast<const __nv_bfloat16*>(X) + (size_t)m0 * K, W, S, Z,
                                static_cast<uint8_t*>(Y) + y_off, out_type, mrows, N, K, reinterpret_cast<float*>(ws),
                                tk, flags, stream, golden, chk.count);
            if (rc) return rc;
            continue;
        }
        const int mt = 1;   // this kernel serves the single-row chunks
        const int splits = w4::choose_splits(mt, N, K);
        w4::Params p;
        p.X = static_cast<const __nv_bfloat16*>(X) + (size_t)m0 * K;
        p.W = static_cast<const uint32_t*>(W);
        p.S = static_cast<const __half*>(S);
        p.Z = static_cast<const __half*>(Z);
        p.Y = static_cast<uint8_t*>(Y) + (size_t)m0 * N * (out_type == QG_OUT_F32 ? 4 : 2);
        p.ws = reinterpret_cast<float*>(ws);
        p.tickets = tk;
        p.M = mrows;
        p.N = N;
        p.K = K;
        p.splits = splits;
        p.out_type = out_type;
        p.early_w = (flags & QG_GEMV_WEIGHTS_CONST) ? 1 : 0;
        p.early_x = (flags & QG_GEMV_ACTIVATIONS_CONST) ? 1 : 0;
        p.golden = golden;
        p.check_count = chk.count;
        const size_t smem = w4::smem_bytes(mt, K, splits);
        QG_CHECK_ARG(smem <= 200 * 1024, "qg_gemv_w4a16: K slice too large for shared memory");
        dim3 grid(w4::col_blocks_for(mt, N), splits);
        if (smem > 48 * 1024)
            QG_CUDA(cudaFuncSetAttribute(w4::gemv_w4a16_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        QG_CUDA(launch_pdl(w4::gemv_w4a16_kernel<1>, grid, dim3(w4::THREADS), smem, stream, p));
        QG_CUDA(cudaGetLastError());
    }
    return QG_OK;
}

} // namespace qg

extern "C" int qg_gemv_w4a16_workspace_bytes(int M, int N, int K, uint64_t* bytes) {
    QG_CHECK_ARG(bytes, "qg_gemv_w4a16_workspace_bytes: null argument");
    *bytes = qg::gemv_w4a16_workspace_bytes(M, N, K, 0);
    return QG_OK;
}

extern "C" int qg_gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int M,
                             int N, int K, void* workspace, uint64_t workspace_bytes, void* stream) {
    return qg::gemv_w4a16(X, W, S, Z, Y, out_type, M, N, K, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream), 0u, qg::LaunchCheck{}, nullptr);
}

extern "C" int qg_gemv_w4a16_ex(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type,
                                int M, int N, int K, void* workspace, uint64_t workspace_bytes, unsigned int flags,
                                void* stream) {
    return qg::gemv_w4a16(X, W, S, Z, Y, out_type, M, N, K, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream), flags, qg::LaunchCheck{}, nullptr);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the W4A16 GEMV.
//
// qg_gemv_w4a16 needs a caller-provided device workspace for its split-K
// partial sums and tickets.  Some callers cannot allocate one at the point of
// the call: a process that has already claimed its device-memory budget up
// front (the stress harness sizes its working set to --mem percent of free
// memory, and a host framework's caching allocator may hold the rest, so a
// fresh cudaMalloc can fail), or a caller on a latency-critical decode path
// where an allocation, which can synchronize the device, is not acceptable.
// qg_gemv_w4a16_noalloc serves them from a fixed scratch array compiled into
// this library instead, and calls no allocating routine.
//
// The array lives in every GPU that loads the library, for the life of the
// process: kNoAllocScratchBytes of device memory per GPU.
constexpr uint64_t kNoAllocScratchBytes = 16ull << 20;   // 16 MiB
// Its first part holds the split-K tickets of every call, whatever the shape
// (N/8 bytes at most: N up to 2^21 columns); the rest the partial sums and
// prepared activations.  Every call leaves its tickets zero, so after one
// clearing at the first call on a device no call needs a memset: a memset
// between two calls would also keep the second from overlapping the first
// (programmatic dependent launch), ~4 us per call.
constexpr uint64_t kNoAllocTicketBytes = 256ull << 10;   // 256 KiB

static __device__ __align__(256) uint8_t g_gemv_noalloc_scratch[kNoAllocScratchBytes];

namespace qg {
namespace w4 {

constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of this device's scratch array.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device, with that device current, and cached; the first lookup also clears
// the ticket region on `stream` (ordered before the call that follows).
static int noalloc_scratch(void** out, cudaStream_t stream) {
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    QG_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "qg_gemv_w4a16_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_error("qg_gemv_w4a16_noalloc: cudaGetSymbolAddress failed: %s (%d)", cudaGetErrorString(e), (int)e);
            return QG_ERR_CUDA;
        }
        QG_CUDA(cudaMemsetAsync(p, 0, (size_t)kNoAllocTicketBytes, stream));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return QG_OK;
}

} // namespace w4
} // namespace qg

extern "C" int qg_gemv_w4a16_noalloc(const void* X, const void* W, const void* S, const void* Z, void* Y,
                                     int out_type, int M, int N, int K, void* stream) {
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemv_w4a16_noalloc: empty shape %dx%dx%d", M, N, K);
    const uint64_t tickets = qg::ticket_bytes(N);
    const uint64_t rest = qg::gemv_w4a16_workspace_bytes(M, N, K, 0) - tickets;
    QG_CHECK_ARG(tickets <= kNoAllocTicketBytes && rest <= kNoAllocScratchBytes - kNoAllocTicketBytes,
                 "qg_gemv_w4a16_noalloc: shape %dx%dx%d needs %llu bytes of scratch and %llu of tickets, above the "
                 "built-in maximum of %llu and %llu bytes; use qg_gemv_w4a16 with a caller-provided workspace",
                 M, N, K, (unsigned long long)rest, (unsigned long long)tickets,
                 (unsigned long long)(kNoAllocScratchBytes - kNoAllocTicketBytes), (unsigned long long)kNoAllocTicketBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* scratch = nullptr;
    int rc = qg::w4::noalloc_scratch(&scratch, s);
    if (rc) return rc;
    // The array keeps whatever the previous call (of any shape) left in it.
    // Every split-K partial and every prepared activation tile is written by
    // this call before this call reads it, and the tickets (in their own
    // region) are zero: the previous call left them so.
    uint8_t* base = static_cast<uint8_t*>(scratch);
    return qg::gemv_w4a16(X, W, S, Z, Y, out_type, M, N, K, base + kNoAllocTicketBytes,
                          kNoAllocScratchBytes - kNoAllocTicketBytes, s, 0u, qg::LaunchCheck{},
                          reinterpret_cast<unsigned int*>(base));
}
