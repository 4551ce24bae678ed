// qg_gemv_w4a16.cu -- weight-only W4A16 group-128 decode GEMV / skinny GEMM
// on the CUDA cores (no tensor cores), bandwidth-bound at M = 1.
//
//   Y[m, n] = sum_k X[m, k] * (q[k, n] - Z[k/128, n]) * S[k/128, n],  q = u - 8
//
// X bf16 [M, K]; W uint32 [K/8, N] (nibble j of word (k8, n) is u(8*k8 + j, n));
// S, Z fp16 [K/128, N]; Y bf16 or fp32 [M, N].
//
// The weights are read once per call, so the kernel is a stream over W: each
// thread owns 4 adjacent columns and issues 128-bit non-allocating loads of
// W (4 columns x 8 k per load), 8 loads deep, coalesced across the warp.  The
// int4 -> bf16 unpack is done in registers: one LOP3 turns two nibbles into a
// bf16 pair 128 + u (exact), and fma.rn.f32.bf16 multiplies it by the bf16
// activation exactly and accumulates in fp32.  Per group of 128 the offset and
// zero point come out algebraically:
//     sum_k x (u - 8 - z) s = s * (sum_k x (128 + u) - (136 + z) * sum_k x),
// with sum_k x computed once per CTA and group.  K is split over CTAs for
// parallelism; each CTA writes its fp32 partial to a workspace and the last
// CTA of a column block (atomic ticket) sums the partials in split order and
// writes Y, so the result is bit-for-bit reproducible run to run.
//
// The path it sits on in the reference: llm_decode (kernels/llm_decode/
// llm_decode.cpp:28-46, a KV gather + FMA chain with no weights) is the decode
// workload; this kernel is the weight-only quantized projection it is named for.
#include "qg_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

namespace qg {
namespace w4 {

constexpr int THREADS = 128;
constexpr int COLS_PER_THREAD = 4;
constexpr int COLS_PER_CTA = THREADS * COLS_PER_THREAD;   // 512
constexpr int GROUP = 128;
constexpr int CHUNKS_PER_GROUP = GROUP / 8;               // 16 uint4 loads per group per thread
constexpr int MAX_M = 16;

struct Params {
    const __nv_bfloat16* X;
    const uint4* W;          // viewed as uint4 = 4 columns of one k8 row
    const __half* S;
    const __half* Z;
    void* Y;
    float* ws;               // [splits][Mpad][N] fp32 partials
    unsigned int* tickets;   // [col_blocks], zero between calls
    int M, N, K;
    int splits;              // K is cut into `splits` ranges of k_per_split
    int k_per_split;         // multiple of GROUP
    int out_type;
};

__device__ __forceinline__ float fma_bf16(uint16_t a, uint16_t b, float c) {
    float d;
    asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// acc[m][c] += sum over the 8 k of one packed word w (column c) of x[m][k] * (128 + u_k).
template <int MT>
__device__ __forceinline__ void accumulate_word(uint32_t w, const uint16_t (*xs)[8], float (&acc)[MT]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // nibbles j (k = j) and j + 4 (k = j + 4) -> bf16 pair (128 + u_j, 128 + u_{j+4})
        const uint32_t pair = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
        const uint16_t lo = (uint16_t)(pair & 0xFFFFu);
        const uint16_t hi = (uint16_t)(pair >> 16);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            acc[m] = fma_bf16(xs[m][j], lo, acc[m]);
            acc[m] = fma_bf16(xs[m][j + 4], hi, acc[m]);
        }
    }
}

template <int MT>
__global__ void __launch_bounds__(THREADS)
gemv_w4a16_kernel(Params p) {
    // X slice of this CTA's k range (bf16 bits) and its per-group sums.
    extern __shared__ uint16_t smem16[];
    const int k0 = blockIdx.y * p.k_per_split;
    const int klen = min(p.k_per_split, p.K - k0);
    const int ngroups = klen / GROUP;
    uint16_t* xs = smem16;                                               // [MT][k_per_split]
    float* xsum = reinterpret_cast<float*>(smem16 + MT * p.k_per_split); // [MT][groups]

    // Stage X (rows >= M read as zero) and the group sums.
    for (int i = threadIdx.x; i < MT * klen / 8; i += THREADS) {
        const int m = i / (klen / 8);
        const int c = i - m * (klen / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < p.M) v = *reinterpret_cast<const uint4*>(p.X + (size_t)m * p.K + k0 + c * 8);
        *reinterpret_cast<uint4*>(xs + m * p.k_per_split + c * 8) = v;
    }
    __syncthreads();
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int t = warp; t < MT * ngroups; t += THREADS / 32) {
            const int m = t / ngroups, g = t - m * ngroups;
            float s = 0.0f;
            for (int k = lane; k < GROUP; k += 32)
                s += __uint_as_float((uint32_t)xs[m * p.k_per_split + g * GROUP + k] << 16);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) xsum[m * ngroups + g] = s;
        }
    }
    __syncthreads();

    const int n0 = blockIdx.x * COLS_PER_CTA + threadIdx.x * COLS_PER_THREAD;
    const bool active = n0 < p.N;   // N % 4 == 0, so a thread is wholly in or out
    float y[MT][COLS_PER_THREAD];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < COLS_PER_THREAD; ++c) y[m][c] = 0.0f;

    if (active) {
        const size_t row_stride = (size_t)p.N / 4;                   // uint4 per k8 row
        const uint4* wp = p.W + (size_t)(k0 / 8) * row_stride + n0 / 4;
        for (int g = 0; g < ngroups; ++g) {
            float acc[COLS_PER_THREAD][MT];
#pragma unroll
            for (int c = 0; c < COLS_PER_THREAD; ++c)
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[c][m] = 0.0f;
#pragma unroll
            for (int half = 0; half < CHUNKS_PER_GROUP; half += 8) {
                uint4 wv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) wv[i] = ld_stream(wp + (size_t)(g * CHUNKS_PER_GROUP + half + i) * row_stride);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int kk = g * GROUP + (half + i) * 8;   // k offset inside this CTA's slice
                    uint16_t xv[MT][8];
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint4 x4 = *reinterpret_cast<const uint4*>(xs + m * p.k_per_split + kk);
                        xv[m][0] = (uint16_t)(x4.x & 0xFFFF); xv[m][1] = (uint16_t)(x4.x >> 16);
                        xv[m][2] = (uint16_t)(x4.y & 0xFFFF); xv[m][3] = (uint16_t)(x4.y >> 16);
                        xv[m][4] = (uint16_t)(x4.z & 0xFFFF); xv[m][5] = (uint16_t)(x4.z >> 16);
                        xv[m][6] = (uint16_t)(x4.w & 0xFFFF); xv[m][7] = (uint16_t)(x4.w >> 16);
                    }
                    accumulate_word<MT>(wv[i].x, xv, acc[0]);
                    accumulate_word<MT>(wv[i].y, xv, acc[1]);
                    accumulate_word<MT>(wv[i].z, xv, acc[2]);
                    accumulate_word<MT>(wv[i].w, xv, acc[3]);
                }
            }
            // fold in scale and zero point of this group
            const int gg = (k0 / GROUP) + g;
            const uint2 s2 = *reinterpret_cast<const uint2*>(p.S + (size_t)gg * p.N + n0);
            const uint2 z2 = *reinterpret_cast<const uint2*>(p.Z + (size_t)gg * p.N + n0);
            const __half* sh = reinterpret_cast<const __half*>(&s2);
            const __half* zh = reinterpret_cast<const __half*>(&z2);
#pragma unroll
            for (int c = 0; c < COLS_PER_THREAD; ++c) {
                const float sc = __half2float(sh[c]);
                const float off = 136.0f + __half2float(zh[c]);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float t = fmaf(-off, xsum[m * ngroups + g], acc[c][m]);
                    y[m][c] = fmaf(sc, t, y[m][c]);
                }
            }
        }
    }

    // ---- split-K: publish the partial; the last CTA of this column block reduces.
    const int mpad = MT;
    if (p.splits == 1) {
        if (active) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= p.M) break;
                if (p.out_type == QG_OUT_F32) {
                    *reinterpret_cast<float4*>(static_cast<float*>(p.Y) + (size_t)m * p.N + n0) =
                        make_float4(y[m][0], y[m][1], y[m][2], y[m][3]);
                } else {
                    __nv_bfloat162 a = __floats2bfloat162_rn(y[m][0], y[m][1]);
                    __nv_bfloat162 b = __floats2bfloat162_rn(y[m][2], y[m][3]);
                    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.Y) + (size_t)m * p.N + n0) =
                        make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
                }
            }
        }
        return;
    }
    if (active) {
#pragma unroll
        for (int m = 0; m < MT; ++m)
            *reinterpret_cast<float4*>(p.ws + ((size_t)blockIdx.y * mpad + m) * p.N + n0) =
                make_float4(y[m][0], y[m][1], y[m][2], y[m][3]);
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned int ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(p.tickets + blockIdx.x, 1u);
    __syncthreads();
    if (ticket != (unsigned int)p.splits - 1) return;
    __threadfence();
    if (active) {
        for (int m = 0; m < p.M && m < MT; ++m) {
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sp = 0; sp < p.splits; ++sp) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(p.ws + ((size_t)sp * mpad + m) * p.N + n0));
                s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
            }
            if (p.out_type == QG_OUT_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(p.Y) + (size_t)m * p.N + n0) = s;
            } else {
                __nv_bfloat162 a = __floats2bfloat162_rn(s.x, s.y);
                __nv_bfloat162 b = __floats2bfloat162_rn(s.z, s.w);
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.Y) + (size_t)m * p.N + n0) =
                    make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
            }
        }
    }
    if (threadIdx.x == 0) p.tickets[blockIdx.x] = 0;   // ready for the next call
}

// Rows per launch template and K split for a given M.
static int m_template(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16; }

// The split depends only on the shape (sized for the 148 SMs of a B200), so the
// workspace size is a function of (M, N, K) alone.
constexpr int kSplitSms = 148;

static int choose_splits(int MT, int N, int K) {
    const int col_blocks = (N + COLS_PER_CTA - 1) / COLS_PER_CTA;
    const int groups = K / GROUP;
    // enough CTAs for several per SM; fewer, longer splits when M makes the CTA compute-heavy
    const int target_ctas = (MT <= 2 ? 12 : MT <= 4 ? 8 : 4) * kSplitSms;
    int splits = (target_ctas + col_blocks - 1) / col_blocks;
    if (splits > groups) splits = groups;
    if (splits < 1) splits = 1;
    while (groups % splits) --splits;   // equal k ranges, each a whole number of groups
    return splits;
}

} // namespace w4

uint64_t gemv_w4a16_workspace_bytes(int M, int N, int K, int sm_count) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    uint64_t total = 0;
    for (int m0 = 0; m0 < M; m0 += w4::MAX_M) {
        const int mt = w4::m_template(M - m0 < w4::MAX_M ? M - m0 : w4::MAX_M);
        const int splits = w4::choose_splits(mt, N, K);
        const uint64_t ws = (uint64_t)splits * mt * N * 4;
        if (ws > total) total = ws;
    }
    const uint64_t col_blocks = (uint64_t)(N + w4::COLS_PER_CTA - 1) / w4::COLS_PER_CTA;
    return ((total + 255) & ~255ull) + col_blocks * 4;
}

int gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int M, int N, int K,
               void* workspace, uint64_t workspace_bytes, cudaStream_t stream) {
    QG_CHECK_ARG(X && W && S && Z && Y, "qg_gemv_w4a16: null operand");
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
    const uint64_t need = gemv_w4a16_workspace_bytes(M, N, K, info->sm_count);
    QG_CHECK_ARG(workspace && workspace_bytes >= need,
                 "qg_gemv_w4a16: workspace of %llu bytes needed (got %llu)", (unsigned long long)need,
                 (unsigned long long)workspace_bytes);
    const int col_blocks = (N + w4::COLS_PER_CTA - 1) / w4::COLS_PER_CTA;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const uint64_t ws_floats_bytes = need - (uint64_t)col_blocks * 4;
    for (int m0 = 0; m0 < M; m0 += w4::MAX_M) {
        const int mrows = (M - m0) < w4::MAX_M ? (M - m0) : w4::MAX_M;
        const int mt = w4::m_template(mrows);
        const int splits = w4::choose_splits(mt, N, K);
        w4::Params p;
        p.X = static_cast<const __nv_bfloat16*>(X) + (size_t)m0 * K;
        p.W = static_cast<const uint4*>(W);
        p.S = static_cast<const __half*>(S);
        p.Z = static_cast<const __half*>(Z);
        p.Y = static_cast<uint8_t*>(Y) + (size_t)m0 * N * (out_type == QG_OUT_F32 ? 4 : 2);
        p.ws = reinterpret_cast<float*>(ws);
        p.tickets = reinterpret_cast<unsigned int*>(ws + ws_floats_bytes);
        p.M = mrows;
        p.N = N;
        p.K = K;
        p.splits = splits;
        p.k_per_split = K / splits;
        p.out_type = out_type;
        const size_t smem = (size_t)mt * p.k_per_split * 2 + (size_t)mt * (p.k_per_split / w4::GROUP) * 4;
        QG_CHECK_ARG(smem <= 200 * 1024, "qg_gemv_w4a16: K slice too large for shared memory");
        dim3 grid(col_blocks, splits);
        switch (mt) {
#define QG_W4_LAUNCH(MTV)                                                                                   \
    case MTV:                                                                                               \
        if (smem > 48 * 1024)                                                                               \
            QG_CUDA(cudaFuncSetAttribute(w4::gemv_w4a16_kernel<MTV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         (int)smem));                                                       \
        w4::gemv_w4a16_kernel<MTV><<<grid, w4::THREADS, smem, stream>>>(p);                                 \
        break;
            QG_W4_LAUNCH(1)
            QG_W4_LAUNCH(2)
            QG_W4_LAUNCH(4)
            QG_W4_LAUNCH(8)
            QG_W4_LAUNCH(16)
#undef QG_W4_LAUNCH
        }
        QG_CUDA(cudaGetLastError());
    }
    return QG_OK;
}

} // namespace qg

extern "C" int qg_gemv_w4a16_workspace_bytes(int M, int N, int K, uint64_t* bytes) {
    QG_CHECK_ARG(bytes, "qg_gemv_w4a16_workspace_bytes: null argument");
    qg::DeviceInfo* info = nullptr;
    int sm = 148;
    if (qg::current_device_info(&info) == QG_OK) sm = info->sm_count;
    *bytes = qg::gemv_w4a16_workspace_bytes(M, N, K, sm);
    return QG_OK;
}

extern "C" int qg_gemv_w4a16(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int M,
                             int N, int K, void* workspace, uint64_t workspace_bytes, void* stream) {
    return qg::gemv_w4a16(X, W, S, Z, Y, out_type, M, N, K, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
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

static __device__ __align__(256) uint8_t g_gemv_noalloc_scratch[kNoAllocScratchBytes];

namespace qg {
namespace w4 {

constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of this device's scratch array.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device, with that device current, and cached.
static int noalloc_scratch(void** out) {
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
    const uint64_t need = qg::gemv_w4a16_workspace_bytes(M, N, K, 0);
    QG_CHECK_ARG(need <= kNoAllocScratchBytes,
                 "qg_gemv_w4a16_noalloc: shape %dx%dx%d needs %llu bytes of scratch, above the built-in maximum of "
                 "%llu bytes; use qg_gemv_w4a16 with a caller-provided workspace",
                 M, N, K, (unsigned long long)need, (unsigned long long)kNoAllocScratchBytes);
    void* scratch = nullptr;
    int rc = qg::w4::noalloc_scratch(&scratch);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The array keeps whatever the previous call (of any shape) left in it,
    // and the tickets must start at zero: clear this call's part first.
    QG_CUDA(cudaMemsetAsync(scratch, 0, (size_t)need, s));
    return qg::gemv_w4a16(X, W, S, Z, Y, out_type, M, N, K, scratch, kNoAllocScratchBytes, s);
}
