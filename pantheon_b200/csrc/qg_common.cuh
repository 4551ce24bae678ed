// qg_common.cuh -- host-side helpers shared by the kernels' launchers:
// error recording, device properties, TMA tensor-map encoding (through the
// runtime's driver entry point, so the library needs no link-time libcuda),
// and the per-device status word of the bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "qg_ptx.cuh"
#include "../../include/pantheon_qgemm.h"

namespace qg {

// Last library-level error (thread-local: one host thread drives one GPU).
void set_error(const char* fmt, ...);
const char* last_error();

#define QG_CUDA(call)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            ::qg::set_error("%s failed: %s (%d) at %s:%d", #call, cudaGetErrorString(e_), \
                            (int)e_, __FILE_NAME__, __LINE__);                         \
            return QG_ERR_CUDA;                                                        \
        }                                                                              \
    } while (0)

#define QG_CHECK_ARG(cond, ...)                 \
    do {                                        \
        if (!(cond)) {                          \
            ::qg::set_error(__VA_ARGS__);       \
            return QG_ERR_ARG;                  \
        }                                       \
    } while (0)

struct DeviceInfo {
    int sm_count = 0;
    int major = 0, minor = 0;
    size_t smem_optin = 0;
};

// Cached properties of the current device; fails on anything but sm_100.
int current_device_info(DeviceInfo** out);

// Device address of this device's bounded-wait status word.
int device_status_ptr(DeviceStatus** out);

// Encode a 2D row-major tensor map: `rows` x `cols` elements of `elem_bytes`,
// row stride `row_bytes`, box `box_cols` x `box_rows`, with `swizzle`.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                 uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

} // namespace qg
