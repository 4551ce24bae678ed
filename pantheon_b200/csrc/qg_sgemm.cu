// qg_sgemm.cu -- FP32 GEMM on the CUDA cores: the tensor furnace's fp32 type.
//
//   C[m,n] = out(alpha * sum_k A[m,k] * B[n,k]),  A fp32 [M,K], B fp32 [N,K], K contiguous.
//
// The reference furnace's fp32 GEMM is cuBLASLt's SGEMM (kernels/common/
// vendor_gemm.h:296-316: R_32F operands, COMPUTE_32F), i.e. the FP32 pipes,
// not the tensor cores (fp32 operands on the tensor cores are the tf32 type).
//
// 128 x 128 tile per CTA of 256 threads, each thread an 8 x 8 block of C held
// in registers: rows 4ty..4ty+3 and 64+4ty..64+4ty+3, columns 4tx..4tx+3 and
// 64+4tx..64+4tx+3 (tx = thread % 16, ty = thread / 16), the split that lets
// the inner loop read its 8 A and 8 B values with two 128-bit shared loads
// each.  K advances 16 at a time: each slab of A and B (128 rows x 16 K) is
// read from global memory as float4 along K one step ahead into registers,
// then stored transposed ([k][row]) into the other half of a double-buffered
// shared-memory tile (warp w stores K offset 4(w % 4) of 32 consecutive rows:
// conflict-free).  Per k the inner loop issues 32 paired fp32 FMAs
// (fma.rn.f32x2): 64 multiply-adds per 4 shared loads.
#include "qg_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qg {
namespace sg {

constexpr int TM = 128, TN = 128, TK = 16;
constexpr int THREADS = 256;
constexpr int LDS = TM + 4;                   // padded row of the transposed tiles (floats)

__device__ __forceinline__ void ffma2(float& a0, float& a1, float b0, float b1, float s) {
    asm("{\n\t.reg .b64 a, b, s;\n\t"
        "mov.b64 a, {%0, %1};\n\t"
        "mov.b64 b, {%2, %3};\n\t"
        "mov.b64 s, {%4, %4};\n\t"
        "fma.rn.f32x2 a, b, s, a;\n\t"
        "mov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1), "f"(s));
}

// The slab rows this thread moves: warp w covers K offset 4 (w % 4) of rows
// 32 (w / 4) + lane and 64 more.
struct SlabMap {
    int k4, r0;
    __device__ SlabMap() {
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        k4 = (w & 3) * 4;
        r0 = (w >> 2) * 32 + lane;
    }
};

__device__ __forceinline__ float4 ld_row4(const float* X, int rows, int K, int r, int k) {
    if (r < rows && k < K) return __ldg(reinterpret_cast<const float4*>(X + (size_t)r * K + k));
    return make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int OUT>
__device__ __forceinline__ void store4(void* C, int N, int m, int n, float4 v, bool full) {
    if (OUT == QG_OUT_F32) {
        float* d = static_cast<float*>(C) + (size_t)m * N + n;
        if (full) { *reinterpret_cast<float4*>(d) = v; return; }
        const float f[4] = {v.x, v.y, v.z, v.w};
        for (int j = 0; j < 4 && n + j < N; ++j) d[j] = f[j];
    } else if (OUT == QG_OUT_F16) {
        __half* d = static_cast<__half*>(C) + (size_t)m * N + n;
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        if (full) {
            *reinterpret_cast<uint2*>(d) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            return;
        }
        const float f[4] = {v.x, v.y, v.z, v.w};
        for (int j = 0; j < 4 && n + j < N; ++j) d[j] = __float2half_rn(f[j]);
    } else {
        __nv_bfloat16* d = static_cast<__nv_bfloat16*>(C) + (size_t)m * N + n;
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
        if (full) {
            *reinterpret_cast<uint2*>(d) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            return;
        }
        const float f[4] = {v.x, v.y, v.z, v.w};
        for (int j = 0; j < 4 && n + j < N; ++j) d[j] = __float2bfloat16_rn(f[j]);
    }
}

template <int OUT>
__global__ void __launch_bounds__(THREADS, 2)
sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B, float alpha, void* __restrict__ C, int M,
             int N, int K) {
    __shared__ __align__(16) float As[2][TK][LDS];
    __shared__ __align__(16) float Bs[2][TK][LDS];
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const SlabMap sm;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    float4 ra[2], rb[2];
    auto load_slab = [&](int k0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            ra[h] = ld_row4(A + (size_t)m0 * K, M - m0, K, sm.r0 + 64 * h, k0 + sm.k4);
            rb[h] = ld_row4(B + (size_t)n0 * K, N - n0, K, sm.r0 + 64 * h, k0 + sm.k4);
        }
    };
    auto store_slab = [&](int buf) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = sm.r0 + 64 * h;
            As[buf][sm.k4 + 0][r] = ra[h].x; As[buf][sm.k4 + 1][r] = ra[h].y;
            As[buf][sm.k4 + 2][r] = ra[h].z; As[buf][sm.k4 + 3][r] = ra[h].w;
            Bs[buf][sm.k4 + 0][r] = rb[h].x; Bs[buf][sm.k4 + 1][r] = rb[h].y;
            Bs[buf][sm.k4 + 2][r] = rb[h].z; Bs[buf][sm.k4 + 3][r] = rb[h].w;
        }
    };

    const int kt = (K + TK - 1) / TK;
    load_slab(0);
    store_slab(0);
    __syncthreads();
    for (int t = 0; t < kt; ++t) {
        const int cur = t & 1;
        if (t + 1 < kt) load_slab((t + 1) * TK);   // in flight during this step's math
#pragma unroll
        for (int k = 0; k < TK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][4 * ty]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][64 + 4 * ty]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][4 * tx]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][64 + 4 * tx]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; j += 2) ffma2(acc[i][j], acc[i][j + 1], b[j], b[j + 1], a[i]);
        }
        if (t + 1 < kt) {
            store_slab(cur ^ 1);   // the other buffer: nobody reads it this step
            __syncthreads();
        }
    }

    // epilogue: 8 rows x two 4-column chunks per thread
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
        if (m >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int n = n0 + 64 * h + 4 * tx;
            if (n >= N) continue;
            const float4 v = make_float4(alpha * acc[i][4 * h + 0], alpha * acc[i][4 * h + 1], alpha * acc[i][4 * h + 2],
                                         alpha * acc[i][4 * h + 3]);
            store4<OUT>(C, N, m, n, v, n + 4 <= N && (N % 4) == 0);
        }
    }
}

} // namespace sg

int gemm_f32(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
             cudaStream_t stream) {
    QG_CHECK_ARG(A && B && C, "qg_gemm_f32: null operand or output");
    QG_CHECK_ARG(M > 0 && N > 0 && K > 0, "qg_gemm_f32: empty shape %dx%dx%d", M, N, K);
    QG_CHECK_ARG(K % 4 == 0, "qg_gemm_f32: K=%d: rows must be a multiple of 16 bytes", K);
    QG_CHECK_ARG(((uintptr_t)A & 15) == 0 && ((uintptr_t)B & 15) == 0 && ((uintptr_t)C & 15) == 0,
                 "qg_gemm_f32: A, B, C must be 16-byte aligned");
    DeviceInfo* info = nullptr;
    int rc = current_device_info(&info);
    if (rc) return rc;
    const dim3 grid((N + sg::TN - 1) / sg::TN, (M + sg::TM - 1) / sg::TM);
    QG_CHECK_ARG(grid.y <= 65535, "qg_gemm_f32: M=%d too large", M);
    const float* a = static_cast<const float*>(A);
    const float* b = static_cast<const float*>(B);
    switch (out_type) {
        case QG_OUT_F32: sg::sgemm_kernel<QG_OUT_F32><<<grid, sg::THREADS, 0, stream>>>(a, b, alpha, C, M, N, K); break;
        case QG_OUT_F16: sg::sgemm_kernel<QG_OUT_F16><<<grid, sg::THREADS, 0, stream>>>(a, b, alpha, C, M, N, K); break;
        case QG_OUT_BF16: sg::sgemm_kernel<QG_OUT_BF16><<<grid, sg::THREADS, 0, stream>>>(a, b, alpha, C, M, N, K); break;
        default: set_error("qg_gemm_f32: out_type %d (bf16, f16 or f32)", out_type); return QG_ERR_ARG;
    }
    QG_CUDA(cudaGetLastError());
    return QG_OK;
}

} // namespace qg

extern "C" int qg_gemm_f32(const void* A, const void* B, float alpha, void* C, int out_type, int M, int N, int K,
                           void* stream) {
    return qg::gemm_f32(A, B, alpha, C, out_type, M, N, K, static_cast<cudaStream_t>(stream));
}
