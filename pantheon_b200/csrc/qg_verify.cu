// qg_verify.cu -- on-device verification: compare an output against the golden
// result computed once per run, word by word.
//
// Replaces ai_verify_output (kernels/common/ai_workload_template.h:343-349) and
// verify_mma_kernel (kernels/mma_virus/mma_virus.cpp:156-173).  Differences
// from those: each thread compares 128 bits per step with 128-bit loads; the
// mismatch count is aggregated per warp (one atomic per warp, not one per bad
// word); and the first `log_cap` mismatches are recorded with their index and
// both values, as the reference's fault log does (kernels/common/fault_log.h:36-50).
#include "qg_common.cuh"
#include "qg_gen.cuh"

namespace qg {
namespace ver {

// counters[0] = mismatching words, counters[1] = log entries written.
__global__ void verify_words_kernel(const uint32_t* __restrict__ actual, const uint32_t* __restrict__ expected,
                                    uint64_t nwords, unsigned long long* counters, qg_mismatch* log, int log_cap) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nvec = nwords / 4;
    uint32_t local = 0;
    const uint4* a4 = reinterpret_cast<const uint4*>(actual);
    const uint4* e4 = reinterpret_cast<const uint4*>(expected);
    for (uint64_t v = tid; v < nvec; v += stride) {
        const uint4 a = __ldcs(a4 + v);
        const uint4 e = __ldcs(e4 + v);
        const uint32_t av[4] = {a.x, a.y, a.z, a.w};
        const uint32_t ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (av[j] != ev[j]) {
                ++local;
                if (log && log_cap > 0) {
                    const unsigned long long slot = atomicAdd(&counters[1], 1ull);
                    if (slot < (unsigned long long)log_cap) log[slot] = qg_mismatch{v * 4 + j, ev[j], av[j]};
                }
            }
        }
    }
    for (uint64_t w = nvec * 4 + tid; w < nwords; w += stride) {
        const uint32_t a = actual[w], e = expected[w];
        if (a != e) {
            ++local;
            if (log && log_cap > 0) {
                const unsigned long long slot = atomicAdd(&counters[1], 1ull);
                if (slot < (unsigned long long)log_cap) log[slot] = qg_mismatch{w, e, a};
            }
        }
    }
    const uint32_t warp_total = __reduce_add_sync(0xffffffffu, local);
    if ((threadIdx.x & 31) == 0 && warp_total) atomicAdd(&counters[0], (unsigned long long)warp_total);
}

// Digest of a word array: the sum (mod 2^64) of splitmix64(i * GAMMA + w_i +
// salt) over the words w_i.  A sum is independent of the order the atomics
// land in, so the digest is reproducible; each term is a bijection of w_i, so
// a change of any single word always changes it.
__global__ void digest_words_kernel(const uint32_t* __restrict__ words, uint64_t nwords, uint64_t salt,
                                    unsigned long long* out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t local = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords; i += stride)
        local += gen::splitmix64(i * gen::GAMMA + (uint64_t)__ldcs(words + i) + salt);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0 && local) atomicAdd(out, (unsigned long long)local);
}

__global__ void flip_bit_kernel(uint32_t* word) { word[0] ^= 0x00000080u; }

__global__ void flip_bit_at_kernel(uint8_t* base, uint64_t byte, uint32_t bit) { base[byte] ^= (uint8_t)(1u << bit); }

} // namespace ver

int verify_words(const void* actual, const void* expected, uint64_t nwords, void* counters, void* log, int log_cap,
                 cudaStream_t s) {
    QG_CHECK_ARG(actual && expected && counters, "qg_verify_words: null argument");
    QG_CHECK_ARG((reinterpret_cast<uintptr_t>(actual) & 15u) == 0 && (reinterpret_cast<uintptr_t>(expected) & 15u) == 0,
                 "qg_verify_words: arrays must be 16-byte aligned");
    if (nwords == 0) return QG_OK;
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    uint64_t need = (nwords / 4 + 255) / 256 + 1;
    const uint64_t cap = (uint64_t)info->sm_count * 8;
    const int grid = (int)(need < cap ? need : cap);
    ver::verify_words_kernel<<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(actual),
                                                  static_cast<const uint32_t*>(expected), nwords,
                                                  static_cast<unsigned long long*>(counters),
                                                  static_cast<qg_mismatch*>(log), log_cap);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int digest_words(const void* words, uint64_t nwords, uint64_t salt, void* out, cudaStream_t s) {
    QG_CHECK_ARG(words && out, "digest_words: null argument");
    if (nwords == 0) return QG_OK;
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    const uint64_t need = (nwords + 255) / 256;
    const uint64_t cap = (uint64_t)info->sm_count * 8;
    ver::digest_words_kernel<<<(int)(need < cap ? need : cap), 256, 0, s>>>(
        static_cast<const uint32_t*>(words), nwords, salt, static_cast<unsigned long long*>(out));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int flip_bit(void* word, cudaStream_t s) {
    ver::flip_bit_kernel<<<1, 1, 0, s>>>(static_cast<uint32_t*>(word));
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

int flip_bit_at(void* base, uint64_t byte, int bit, cudaStream_t s) {
    ver::flip_bit_at_kernel<<<1, 1, 0, s>>>(static_cast<uint8_t*>(base), byte, (uint32_t)bit);
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace qg

extern "C" int qg_verify_words(const void* actual, const void* expected, uint64_t nwords, void* count, void* log,
                               int log_cap, void* stream) {
    return qg::verify_words(actual, expected, nwords, count, log, log_cap, static_cast<cudaStream_t>(stream));
}
