// qg_gemv.cuh -- what the three W4A16 GEMV kernels share: the SM count their
// work split is sized for, and the entries of the tcgen05 kernel (13..16
// activation rows) and the warp-MMA kernel (2..12 rows), used by the C entry
// points in qg_gemv_w4a16.cu.
#pragma once

#include "qg_common.cuh"

#include <utility>

namespace qg {

// Launch with programmatic stream serialization (PDL): the kernel's CTAs may
// start while the previous kernel on the stream drains; the kernels call
// griddepcontrol.wait before any global memory access and
// griddepcontrol.launch_dependents once all their CTAs are resident, so
// back-to-back GEMV calls overlap one call's tail with the next one's launch.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

// The split of the work depends only on the shape (sized for the 148 SMs of a
// B200), so workspace sizes are functions of (M, N, K) alone.
constexpr int kGemvSms = 148;

// fp32 partial-sum bytes and ticket count of the tcgen05 GEMV for N x K.
uint64_t gemv_w4a16_tc_partial_bytes(int N, int K);
uint64_t gemv_w4a16_tc_ticket_count(int N);

// Bytes of the prepared-X area (quantised activation tiles and their scales).
uint64_t gemv_w4a16_tc_xprep_bytes(int K);

// One call for `mrows` (1..16) activation rows (two launches: the X pre-pass,
// then the GEMV); `partials`, `tickets` and `xprep` come from the caller's
// workspace, tickets zero on entry (and on return).  Per-launch check
// (qg_check.cuh): with `fp_record` the writer of each output column stores the
// column's fingerprint (N entries); with `fp_expect` it compares it with the
// recorded one and counts differing columns into `check_count`.  With
// QG_GEMV_ACTIVATIONS_CONST in `flags` the pre-pass quantises X before waiting
// for the kernel ahead on the stream (it waits only before its stores).
int gemv_w4a16_tc(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                  int K, float* partials, unsigned int* tickets, void* xprep, cudaStream_t stream,
                  uint32_t* fp_record = nullptr, const uint32_t* fp_expect = nullptr,
                  unsigned long long* check_count = nullptr, unsigned int flags = 0);

// The warp-MMA GEMV for up to 8 rows (qg_gemv_w4a16_mma.cu): workspace parts
// for `mrows` rows of N x K (fp32 partials, tickets).
uint64_t gemv_w4a16_mma_partial_bytes(int mrows, int N, int K);
uint64_t gemv_w4a16_mma_ticket_count(int N);

// One call (one launch) for `mrows` (1..16) activation rows.  `partials`
// (16-byte aligned) and `tickets` (zero on entry and on return) come from the
// caller's workspace; `flags` are the QG_GEMV_* declarations about the kernel
// ahead on the stream (QG_GEMV_WEIGHTS_CONST: it writes no W, S or Z;
// QG_GEMV_ACTIVATIONS_CONST: it writes no X).  With `golden` (a checked launch)
// every stored output word is compared with the golden output and
// differences are counted into `check_count`.
int gemv_w4a16_mma(const void* X, const void* W, const void* S, const void* Z, void* Y, int out_type, int mrows, int N,
                   int K, float* partials, unsigned int* tickets, unsigned int flags, cudaStream_t stream,
                   const void* golden = nullptr, unsigned long long* check_count = nullptr);

} // namespace qg
