// qg_common.cu -- shared host helpers (see qg_common.cuh).
#include "qg_common.cuh"

#include <cstdarg>
#include <mutex>

namespace qg {

static thread_local char g_err[512];

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

const char* last_error() { return g_err; }

constexpr int kMaxDevices = 64;
static DeviceInfo g_info[kMaxDevices];
static bool g_info_ok[kMaxDevices];
static DeviceStatus* g_status_ptr[kMaxDevices];
static std::mutex g_mu;

// One status word per device (each device that loads the library has its own
// copy of this variable).
__device__ DeviceStatus g_device_status;

int current_device_info(DeviceInfo** out) {
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    QG_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_info_ok[dev]) {
        cudaDeviceProp p;
        QG_CUDA(cudaGetDeviceProperties(&p, dev));
        if (p.major != 10 || p.minor != 0) {
            set_error("device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev, p.major, p.minor);
            return QG_ERR_UNSUPPORTED;
        }
        g_info[dev].sm_count = p.multiProcessorCount;
        g_info[dev].major = p.major;
        g_info[dev].minor = p.minor;
        g_info[dev].smem_optin = p.sharedMemPerBlockOptin;
        g_info_ok[dev] = true;
    }
    *out = &g_info[dev];
    return QG_OK;
}

int device_status_ptr(DeviceStatus** out) {
    int dev = 0;
    QG_CUDA(cudaGetDevice(&dev));
    QG_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status_ptr[dev]) {
        void* p = nullptr;
        QG_CUDA(cudaGetSymbolAddress(&p, g_device_status));
        g_status_ptr[dev] = static_cast<DeviceStatus*>(p);
    }
    *out = g_status_ptr[dev];
    return QG_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                 uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled is not available from the driver"); return QG_ERR_CUDA; }
    QG_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15u) == 0, "tensor base %p is not 16-byte aligned", base);
    QG_CHECK_ARG(row_bytes % 16 == 0, "row stride %llu bytes is not a multiple of 16", (unsigned long long)row_bytes);
    QG_CHECK_ARG((uint64_t)box_cols * elem_bytes <= 128 || swizzle == CU_TENSOR_MAP_SWIZZLE_NONE,
                 "box inner extent exceeds the swizzle span");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d): dims %llux%llu box %ux%u", (int)r,
                  (unsigned long long)cols, (unsigned long long)rows, box_cols, box_rows);
        return QG_ERR_CUDA;
    }
    return QG_OK;
}

} // namespace qg

extern "C" int qg_device_status_detail(int device, uint32_t* site, uint32_t* waits_expired, uint32_t* ctas_drained) {
    QG_CUDA(cudaSetDevice(device));
    qg::DeviceStatus* p = nullptr;
    int rc = qg::device_status_ptr(&p);
    if (rc) return rc;
    qg::DeviceStatus h{};
    QG_CUDA(cudaMemcpy(&h, p, sizeof(h), cudaMemcpyDeviceToHost));
    if (site) *site = h.code;
    if (waits_expired) *waits_expired = h.count;
    if (ctas_drained) *ctas_drained = h.drained;
    if (h.code == 0 && h.drained == 0) return QG_OK;
    qg::set_error("device wait expired: site 0x%08x (%u waits gave up, %u CTAs drained and freed TMEM)", h.code,
                  h.count, h.drained);
    qg::DeviceStatus z{};
    QG_CUDA(cudaMemcpy(p, &z, sizeof(z), cudaMemcpyHostToDevice));
    return h.code ? QG_ERR_DEVICE_TIMEOUT : QG_OK;
}

extern "C" int qg_device_status(int device) { return qg_device_status_detail(device, nullptr, nullptr, nullptr); }
