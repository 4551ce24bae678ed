// qg_check.cuh -- verification of every launch, inside the kernels.
//
// The workload compares the output of the LAST launch of each batch with the
// golden result bitwise (qg_verify), but a batch is ~200 ms of launches that
// overwrite one output buffer, so a corruption in an earlier launch of the
// batch would be overwritten unseen.  Each launch therefore checks itself
// where its results are still in registers:
//   GEMMs   every epilogue thread folds the output words it stores for its row
//           segment (256 columns in the INT8 / dense kernels, 128 in the FP8
//           and NVFP4 kernels) into a fingerprint -- the INT8 kernel also folds
//           its INT32 accumulators, so a flipped low accumulator bit that
//           rounds away in bf16 still shows -- and, in the golden launch,
//           records it; in every later launch it compares it with the recorded
//           one;
//   GEMV    the CUDA-core (1 row) and warp-MMA (2-12 rows) kernels compare each
//           output word they write with the golden output; the tcgen05 kernel
//           (13-16 rows) folds the words of each output column into a
//           fingerprint, recorded by
//           the golden launch and compared by later launches, with the
//           expected value loaded when the column's tile starts (a compare at
//           the end would put a memory round trip per row on the fold's path).
// Differences are counted with one atomic per warp (ballot + popc).  The
// fingerprint folds the words in a fixed order, fp = fp * kCheckMul + word
// (mod 2^32, one multiply-add per word): word i enters multiplied by an odd
// power of kCheckMul, so a change of any single word always changes it.
#pragma once

#include <cstdint>

namespace qg {

struct LaunchCheck {
    uint32_t* record = nullptr;             // golden launch: fingerprints written here
    const uint32_t* expect = nullptr;       // checked launch: fingerprints recorded by the golden launch
    unsigned long long* count = nullptr;    // checked launch: differences found
    const void* golden = nullptr;           // checked GEMV launch: the golden output (CUDA-core kernel)
};

// Odd multiplier of the fold (odd: multiplication by it is invertible mod 2^32).
constexpr uint32_t kCheckMul = 0x9E3779B1u;

// Record or compare the fingerprint of segment `idx` (only where `valid`).  Every
// lane of the warp calls it with the same `c`; at most one atomic per warp.
__device__ __forceinline__ void check_segment(const LaunchCheck& c, bool valid, uint64_t idx, uint32_t fp) {
    if (c.record) {
        if (valid) c.record[idx] = fp;
    } else if (c.expect) {
        const bool bad = valid && __ldcg(c.expect + idx) != fp;
        const unsigned mask = __ballot_sync(0xffffffffu, bad);
        if (mask && (threadIdx.x & 31) == 0) atomicAdd(c.count, (unsigned long long)__popc(mask));
    }
}

// Add `n` differences found by this lane to the warp's count (one atomic per warp).
// Every lane of the warp calls it.
__device__ __forceinline__ void check_count_warp(unsigned long long* count, uint32_t n) {
    const uint32_t total = __reduce_add_sync(0xffffffffu, n);
    if (total && (threadIdx.x & 31) == 0) atomicAdd(count, (unsigned long long)total);
}

} // namespace qg
