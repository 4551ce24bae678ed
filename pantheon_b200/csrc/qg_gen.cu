// qg_gen.cu -- operand generator kernels (seeded, counter-based; see qg_gen.cuh).
// Replaces ai_initialize (kernels/common/ai_workload_template.h:85-94) and
// pantheon_gemm_fill (kernels/common/vendor_gemm.h:184-191).
#include "qg_common.cuh"
#include "qg_gen.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

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

} // namespace qg

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
