// qg_gen.cu -- operand generator kernels (seeded, counter-based; see qg_gen.cuh).
// Replaces ai_initialize (kernels/common/ai_workload_template.h:85-94) and
// pantheon_gemm_fill (kernels/common/vendor_gemm.h:184-191).
#include "qg_common.cuh"
#include "qg_gen.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace qg {
namespace gen {

// Grid-stride fill, 16 int8 values per thread step (one 128-bit store).
__global__ void gen_i8_kernel(int8_t* out, uint64_t n, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nvec = n / 16;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int8_t x = i8_from_hash(hash_at(key, v * 16 + j * 4 + b));
                word |= (uint32_t)(uint8_t)x << (8 * b);
            }
            w[j] = word;
        }
        reinterpret_cast<uint4*>(out)[v] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    // tail
    const uint64_t t = nvec * 16 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = i8_from_hash(hash_at(key, t));
}

__global__ void gen_uniform_kernel(float* out, uint64_t n, float lo, float hi, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = uniform_from_hash(hash_at(key, i), lo, hi);
}

__global__ void gen_normal_kernel(float* out, uint64_t n, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = normal_from_hash(hash_at(key, i));
}

// W4A16 operands.
__global__ void gen_bf16_normal_kernel(__nv_bfloat16* out, uint64_t n, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __float2bfloat16_rn(normal_from_hash(hash_at(key, i)));
}

__global__ void gen_f16_uniform_kernel(__half* out, uint64_t n, float lo, float hi, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __float2half_rn(uniform_from_hash(hash_at(key, i), lo, hi));
}

// Word (k8, n) packs u(8*k8 + j, n) = top 4 bits of hash(k * N + n) in nibble j.
__global__ void gen_w4_kernel(uint32_t* out, uint64_t words, uint32_t N, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += stride) {
        const uint64_t k8 = i / N, n = i - k8 * N;
        uint32_t w = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint64_t k = k8 * 8 + (uint64_t)j;
            w |= (uint32_t)(hash_at(key, k * N + n) >> 60) << (4 * j);
        }
        out[i] = w;
    }
}

// FP8 e4m3 operands: values N(0,1), each block scaled so that its
// absmax maps to 448: q = e4m3_rn_satfinite(x * (448 / amax)), scale = amax / 448.
__device__ __forceinline__ uint8_t to_e4m3(float v) {
    return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// A: 1 x 128 blocks along K, one warp per block (lane l holds k = 4l .. 4l+3).
__global__ void gen_fp8_rows_kernel(uint8_t* Q, float* S, int R, int K, uint64_t key) {
    const int kb_count = K / 128;
    const uint64_t blocks = (uint64_t)R * kb_count;
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t b = (uint64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); b < blocks; b += warps) {
        const uint64_t r = b / kb_count, kb = b - r * kb_count;
        const uint64_t base = r * (uint64_t)K + kb * 128 + (uint64_t)lane * 4;
        float x[4];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[i] = normal_from_hash(hash_at(key, base + i));
            amax = fmaxf(amax, fabsf(x[i]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.0f ? __fdiv_rn(448.0f, amax) : 1.0f;
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) w |= (uint32_t)to_e4m3(__fmul_rn(x[i], inv)) << (8 * i);
        *reinterpret_cast<uint32_t*>(Q + base) = w;
        if (lane == 0) S[b] = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
    }
}

// Dense tensor-furnace operands: v = j / 32768 - 1 with j the top 16 bits of the
// element's hash (uniform on [-1, 1) in steps of 2^-15; exact in fp32), rounded
// to the operand format (nearest even; e4m3 saturating; tf32 = fp32 word with
// the low 13 mantissa bits cleared after rounding).
__device__ __forceinline__ float dense_value(uint64_t h) {
    return __fsub_rn(__fmul_rn((float)(uint32_t)(h >> 48), 3.0517578125e-05f), 1.0f);
}

__device__ __forceinline__ uint32_t tf32_rn_bits(float v) {
    uint32_t u = __float_as_uint(v);
    u += 0xFFFu + ((u >> 13) & 1u);
    return u & 0xFFFFE000u;
}

template <int FMT>
__global__ void gen_dense_kernel(void* out, uint64_t n, uint64_t key) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = dense_value(hash_at(key, i));
        if constexpr (FMT == QG_FMT_BF16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
        else if constexpr (FMT == QG_FMT_FP16) static_cast<__half*>(out)[i] = __float2half_rn(v);
        else if constexpr (FMT == QG_FMT_TF32) static_cast<uint32_t*>(out)[i] = tf32_rn_bits(v);
        else if constexpr (FMT == QG_FMT_FP32) static_cast<float*>(out)[i] = v;
        else static_cast<uint8_t*>(out)[i] = to_e4m3(v);
    }
}

// B: 128 x 128 blocks, one 256-thread CTA per block (thread t: row t/2, 64 k).
__global__ void gen_fp8_blocks_kernel(uint8_t* Q, float* S, int R, int K, uint64_t key) {
    const int kb_count = K / 128;
    const int rb = blockIdx.x / kb_count, kb = blockIdx.x - rb * kb_count;
    const int r = rb * 128 + (threadIdx.x >> 1);
    const uint64_t base = (uint64_t)r * K + (uint64_t)kb * 128 + (threadIdx.x & 1) * 64;
    const bool live = r < R;
    float x[64];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        x[i] = live ? normal_from_hash(hash_at(key, base + i)) : 0.0f;
        amax = fmaxf(amax, fabsf(x[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __shared__ float warp_max[8];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, warp_max[i]);
    const float inv = amax > 0.0f ? __fdiv_rn(448.0f, amax) : 1.0f;
    if (live) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t word = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) word |= (uint32_t)to_e4m3(__fmul_rn(x[v * 16 + j * 4 + b], inv)) << (8 * b);
                w[j] = word;
            }
            *reinterpret_cast<uint4*>(Q + base + v * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    if (threadIdx.x == 0) S[blockIdx.x] = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
}

// NVFP4 operands: values N(0,1); per-tensor scale G = amax/(448*6);
// per 16 along K an ue4m3 scale sf = e4m3(bmax/6/G); codes q = e2m1(x/(dec(sf)*G)).
__global__ void absmax_normal_kernel(uint64_t n, uint64_t key, unsigned int* amax_bits) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    float a = 0.0f;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        a = fmaxf(a, fabsf(normal_from_hash(hash_at(key, i))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(a));   // non-negative floats order as integers
}

__global__ void global_scale_kernel(const unsigned int* amax_bits, float* g) {
    const float amax = __uint_as_float(*amax_bits);
    *g = amax > 0.0f ? __fdiv_rn(amax, 448.0f * 6.0f) : 1.0f;
}

__device__ __forceinline__ float e4m3_decode(uint8_t v) {
    const int e = (v >> 3) & 0xF, m = v & 7;
    const float r = (e == 0) ? (float)m * 0.001953125f : ldexpf((float)(8 + m), e - 10);
    return (v & 0x80) ? -r : r;
}

// e2m1 code of x (round to nearest, ties to the even code, saturating at 6).
__device__ __forceinline__ uint32_t e2m1_code(float x) {
    const uint32_t sign = (__float_as_uint(x) >> 28) & 0x8u;
    const float a = fabsf(x);
    uint32_t c;
    if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return sign | c;
}

// One thread per (row, 16-element block): codes (8 bytes) and the scale byte,
// written straight into the tcgen05 scale-factor atom layout:
//   atom (row block r/128, K chunk k/64) is 512 bytes at ((r/128) * (K/64) + k/64) * 512;
//   inside it, row r's 4 scales of the chunk are bytes (r%32)*16 + ((r/32)%4)*4 + 0..3.
__global__ void quant_nvfp4_kernel(uint8_t* Q, uint8_t* SF, int R, int K, uint64_t key, const float* gscale) {
    const int nb = K / 16;
    const uint64_t total = (uint64_t)R * nb;
    const float G = *gscale;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < total; b += stride) {
        const int r = (int)(b / nb), kb = (int)(b - (uint64_t)r * nb);
        const uint64_t base = (uint64_t)r * K + (uint64_t)kb * 16;
        float x[16];
        float bmax = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            x[i] = normal_from_hash(hash_at(key, base + i));
            bmax = fmaxf(bmax, fabsf(x[i]));
        }
        float t = __fdiv_rn(bmax, 6.0f);
        t = __fdiv_rn(t, G);
        const uint8_t sf = (uint8_t)(__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3) & 0x7F);
        const float d = __fmul_rn(e4m3_decode(sf), G);
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = d > 0.0f ? e2m1_code(__fdiv_rn(x[i], d)) : 0u;
            w0 |= c << (4 * i);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = d > 0.0f ? e2m1_code(__fdiv_rn(x[8 + i], d)) : 0u;
            w1 |= c << (4 * i);
        }
        *reinterpret_cast<uint2*>(Q + base / 2) = make_uint2(w0, w1);
        const size_t atom = (size_t)(r / 128) * (K / 64) + kb / 4;
        SF[atom * 512 + (r % 32) * 16 + ((r / 32) % 4) * 4 + (kb % 4)] = sf;
    }
}

static int grid_for(uint64_t work) {
    DeviceInfo* info = nullptr;
    int blocks = 148 * 8;
    if (current_device_info(&info) == QG_OK) blocks = info->sm_count * 8;
    uint64_t need = (work + 255) / 256;
    if (need < 1) need = 1;
    return (int)(need < (uint64_t)blocks ? need : (uint64_t)blocks);
}

} // namespace gen

int gen_i8(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s) {
    QG_CHECK_ARG(out || n == 0, "qg_gen_i8: null output");
    QG_CHECK_ARG((reinterpret_cast<uintptr_t>(out) & 15u) == 0, "qg_gen_i8: output must be 16-byte aligned");
    if (n == 0) return QG_OK;
    gen::gen_i8_kernel<<<gen::grid_for(n / 16 + 1), 256, 0, s>>>(static_cast<int8_t*>(out), n, gen::stream_key(seed, tensor_id));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int gen_dense(int fmt, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s) {
    QG_CHECK_ARG(out || n == 0, "qg_gen_dense: null output");
    if (n == 0) return QG_OK;
    const uint64_t key = gen::stream_key(seed, tensor_id);
    const int grid = gen::grid_for(n);
    switch (fmt) {
        case QG_FMT_BF16: gen::gen_dense_kernel<QG_FMT_BF16><<<grid, 256, 0, s>>>(out, n, key); break;
        case QG_FMT_FP16: gen::gen_dense_kernel<QG_FMT_FP16><<<grid, 256, 0, s>>>(out, n, key); break;
        case QG_FMT_TF32: gen::gen_dense_kernel<QG_FMT_TF32><<<grid, 256, 0, s>>>(out, n, key); break;
        case QG_FMT_E4M3: gen::gen_dense_kernel<QG_FMT_E4M3><<<grid, 256, 0, s>>>(out, n, key); break;
        case QG_FMT_FP32: gen::gen_dense_kernel<QG_FMT_FP32><<<grid, 256, 0, s>>>(out, n, key); break;
        default: set_error("qg_gen_dense: format %d is not a dense format", fmt); return QG_ERR_ARG;
    }
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int gen_uniform(void* out, uint64_t n, float lo, float hi, uint64_t seed, uint32_t tensor_id, cudaStream_t s) {
    QG_CHECK_ARG(out || n == 0, "qg_gen_uniform_f32: null output");
    if (n == 0) return QG_OK;
    gen::gen_uniform_kernel<<<gen::grid_for(n), 256, 0, s>>>(static_cast<float*>(out), n, lo, hi, gen::stream_key(seed, tensor_id));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int gen_normal(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, cudaStream_t s) {
    QG_CHECK_ARG(out || n == 0, "qg_gen_normal_f32: null output");
    if (n == 0) return QG_OK;
    gen::gen_normal_kernel<<<gen::grid_for(n), 256, 0, s>>>(static_cast<float*>(out), n, gen::stream_key(seed, tensor_id));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int gen_w4a16(void* X, void* W, void* S, void* Z, int M, int N, int K, uint64_t seed, uint32_t tid0, cudaStream_t s) {
    QG_CHECK_ARG(X && W && S && Z, "qg_gen_w4a16: null output");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % 128 == 0, "qg_gen_w4a16: bad shape %dx%dx%d", M, N, K);
    const uint64_t nx = (uint64_t)M * K, nw = (uint64_t)K / 8 * N, ns = (uint64_t)K / 128 * N;
    gen::gen_bf16_normal_kernel<<<gen::grid_for(nx), 256, 0, s>>>(static_cast<__nv_bfloat16*>(X), nx,
                                                                  gen::stream_key(seed, tid0));
    gen::gen_w4_kernel<<<gen::grid_for(nw), 256, 0, s>>>(static_cast<uint32_t*>(W), nw, (uint32_t)N,
                                                         gen::stream_key(seed, tid0 + 1));
    gen::gen_f16_uniform_kernel<<<gen::grid_for(ns), 256, 0, s>>>(static_cast<__half*>(S), ns, 0.005f, 0.02f,
                                                                  gen::stream_key(seed, tid0 + 2));
    gen::gen_f16_uniform_kernel<<<gen::grid_for(ns), 256, 0, s>>>(static_cast<__half*>(Z), ns, -0.5f, 0.5f,
                                                                  gen::stream_key(seed, tid0 + 3));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int gen_fp8(void* A, void* SA, void* B, void* SB, int M, int N, int K, uint64_t seed, uint32_t tid0, cudaStream_t s) {
    QG_CHECK_ARG(A && SA && B && SB, "qg_gen_fp8: null output");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % 128 == 0, "qg_gen_fp8: bad shape %dx%dx%d (K %% 128 == 0)", M, N, K);
    const uint64_t warps_needed = (uint64_t)M * (K / 128);
    gen::gen_fp8_rows_kernel<<<gen::grid_for(warps_needed * 32), 256, 0, s>>>(
        static_cast<uint8_t*>(A), static_cast<float*>(SA), M, K, gen::stream_key(seed, tid0));
    const int bblocks = ((N + 127) / 128) * (K / 128);
    gen::gen_fp8_blocks_kernel<<<bblocks, 256, 0, s>>>(static_cast<uint8_t*>(B), static_cast<float*>(SB), N, K,
                                                       gen::stream_key(seed, tid0 + 2));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

// NVFP4 operand set: A codes/scales from tensor tid0, B from tid0 + 2.  The two
// per-tensor scales are written to gscales[0..1] (device) and also returned
// through `host_gscales` when non-null (synchronizes `s`).  `work` is 8 bytes
// of device scratch for the absmax reductions.
int gen_nvfp4(void* A, void* SFA, void* B, void* SFB, float* gscales, void* work, int M, int N, int K, uint64_t seed,
              uint32_t tid0, cudaStream_t s) {
    QG_CHECK_ARG(A && SFA && B && SFB && gscales && work, "qg_gen_nvfp4: null output");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0 && K % 256 == 0, "qg_gen_nvfp4: bad shape %dx%dx%d (K %% 256 == 0)", M, N, K);
    unsigned int* amax = static_cast<unsigned int*>(work);
    QG_CUDA(cudaMemsetAsync(amax, 0, 8, s));
    const uint64_t keyA = gen::stream_key(seed, tid0), keyB = gen::stream_key(seed, tid0 + 2);
    const uint64_t na = (uint64_t)M * K, nbv = (uint64_t)N * K;
    gen::absmax_normal_kernel<<<gen::grid_for(na), 256, 0, s>>>(na, keyA, amax);
    gen::absmax_normal_kernel<<<gen::grid_for(nbv), 256, 0, s>>>(nbv, keyB, amax + 1);
    gen::global_scale_kernel<<<1, 1, 0, s>>>(amax, gscales);
    gen::global_scale_kernel<<<1, 1, 0, s>>>(amax + 1, gscales + 1);
    // scale atoms of rows past M / N (the last partial 128-row block) stay zero
    const size_t sfa_bytes = (size_t)((M + 127) / 128) * (K / 64) * 512;
    const size_t sfb_bytes = (size_t)((N + 127) / 128) * (K / 64) * 512;
    QG_CUDA(cudaMemsetAsync(SFA, 0, sfa_bytes, s));
    QG_CUDA(cudaMemsetAsync(SFB, 0, sfb_bytes, s));
    gen::quant_nvfp4_kernel<<<gen::grid_for((uint64_t)M * (K / 16)), 256, 0, s>>>(
        static_cast<uint8_t*>(A), static_cast<uint8_t*>(SFA), M, K, keyA, gscales);
    gen::quant_nvfp4_kernel<<<gen::grid_for((uint64_t)N * (K / 16)), 256, 0, s>>>(
        static_cast<uint8_t*>(B), static_cast<uint8_t*>(SFB), N, K, keyB, gscales + 1);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace qg

extern "C" int qg_gen_nvfp4(void* A, void* SFA, void* B, void* SFB, void* gscales, void* work, int M, int N, int K,
                            uint64_t seed, uint32_t tid0, void* stream) {
    return qg::gen_nvfp4(A, SFA, B, SFB, static_cast<float*>(gscales), work, M, N, K, seed, tid0,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_fp8(void* A, void* SA, void* B, void* SB, int M, int N, int K, uint64_t seed, uint32_t tid0,
                          void* stream) {
    return qg::gen_fp8(A, SA, B, SB, M, N, K, seed, tid0, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_w4a16(void* X, void* W, void* S, void* Z, int M, int N, int K, uint64_t seed, uint32_t tid0,
                            void* stream) {
    return qg::gen_w4a16(X, W, S, Z, M, N, K, seed, tid0, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_i8(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream) {
    return qg::gen_i8(out, n, seed, tensor_id, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_uniform_f32(void* out, uint64_t n, float lo, float hi, uint64_t seed, uint32_t tensor_id,
                                  void* stream) {
    return qg::gen_uniform(out, n, lo, hi, seed, tensor_id, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_normal_f32(void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream) {
    return qg::gen_normal(out, n, seed, tensor_id, static_cast<cudaStream_t>(stream));
}

extern "C" int qg_gen_dense(int format, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id, void* stream) {
    return qg::gen_dense(format, out, n, seed, tensor_id, static_cast<cudaStream_t>(stream));
}
