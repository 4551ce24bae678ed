// qg_gen.cu -- operand generator kernels (seeded, counter-based; see qg_gen.cuh).
// Replaces ai_initialize (kernels/common/ai_workload_template.h:85-94) and
// pantheon_gemm_fill (kernels/common/vendor_gemm.h:184-191).
#include "qg_common.cuh"
#include "qg_gen.cuh"

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

} // namespace qg

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
