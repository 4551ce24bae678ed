// qg_gen.cuh -- device side of the counter-based operand generator.
//
// The reference fills its operands from a hash of the element index
// (ai_initialize, kernels/common/ai_workload_template.h:85-94;
// pantheon_gemm_fill, kernels/common/vendor_gemm.h:184-191).  Here the hash is
// splitmix64 (Steele, Lea & Flood, OOPSLA 2014), output i of the stream keyed by
// (seed, tensor id), so A and B never share a stream and every element can be
// produced independently by any thread.  All fp32 arithmetic uses explicit
// round-to-nearest intrinsics, one rounding per operation, so the host test
// oracle (compiled with -ffp-contract=off) reproduces every bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace qg {
namespace gen {

constexpr uint64_t GAMMA = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint32_t tensor_id) {
    return splitmix64(seed + GAMMA * ((uint64_t)tensor_id + 1ull));
}

__host__ __device__ __forceinline__ uint64_t hash_at(uint64_t key, uint64_t index) {
    return splitmix64(key + GAMMA * (index + 1ull));
}

__device__ __forceinline__ int8_t i8_from_hash(uint64_t h) {
    return (int8_t)((int)((uint32_t)(h >> 32) % 255u) - 127);
}

__device__ __forceinline__ float uniform_from_hash(uint64_t h, float lo, float hi) {
    const float u = __fmul_rn((float)(uint32_t)(h >> 40), 5.9604644775390625e-08f);
    const float d = __fsub_rn(hi, lo);
    const float t = __fmul_rn(d, u);
    return __fadd_rn(lo, t);
}

// log x for normal x > 0 from log m = 2 atanh((m-1)/(m+1)) (odd power series).
__device__ __forceinline__ float log_series(float x) {
    const uint32_t b = __float_as_uint(x);
    int e = (int)((b >> 23) & 0xFF) - 127;
    float m = __uint_as_float((b & 0x007FFFFFu) | 0x3F800000u);
    if (m > 1.41421356f) { m = __fmul_rn(m, 0.5f); e = e + 1; }
    const float num = __fsub_rn(m, 1.0f);
    const float den = __fadd_rn(m, 1.0f);
    const float s = __fdiv_rn(num, den);
    const float s2 = __fmul_rn(s, s);
    float p = 0.0909090936f;
    p = __fadd_rn(__fmul_rn(p, s2), 0.111111112f);
    p = __fadd_rn(__fmul_rn(p, s2), 0.142857149f);
    p = __fadd_rn(__fmul_rn(p, s2), 0.200000003f);
    p = __fadd_rn(__fmul_rn(p, s2), 0.333333343f);
    p = __fadd_rn(__fmul_rn(p, s2), 1.0f);
    const float lm = __fmul_rn(__fadd_rn(s, s), p);
    const float el = __fmul_rn((float)e, 0.693147182f);
    return __fadd_rn(el, lm);
}

// Standard normal deviate by P. J. Acklam's rational inverse-CDF approximation.
__device__ __forceinline__ float normal_from_hash(uint64_t h) {
    const float p = __fmul_rn((float)(2u * (uint32_t)(h >> 41) + 1u), 5.9604644775390625e-08f);
    const float plow = 0.02425f;
    const float phigh = __fsub_rn(1.0f, plow);
    float x;
    if (p < plow || p > phigh) {
        const float pp = p < plow ? p : __fsub_rn(1.0f, p);
        const float l = log_series(pp);
        const float t = __fmul_rn(-2.0f, l);
        const float q = __fsqrt_rn(t);
        float n = -7.78489400e-03f;
        n = __fadd_rn(__fmul_rn(n, q), -3.22396458e-01f);
        n = __fadd_rn(__fmul_rn(n, q), -2.40075827e+00f);
        n = __fadd_rn(__fmul_rn(n, q), -2.54973254e+00f);
        n = __fadd_rn(__fmul_rn(n, q), 4.37466414e+00f);
        n = __fadd_rn(__fmul_rn(n, q), 2.93816398e+00f);
        float d = 7.78469571e-03f;
        d = __fadd_rn(__fmul_rn(d, q), 3.22467129e-01f);
        d = __fadd_rn(__fmul_rn(d, q), 2.44513414e+00f);
        d = __fadd_rn(__fmul_rn(d, q), 3.75440866e+00f);
        d = __fadd_rn(__fmul_rn(d, q), 1.0f);
        x = __fdiv_rn(n, d);
        if (p > plow) x = -x;
    } else {
        const float q = __fsub_rn(p, 0.5f);
        const float r = __fmul_rn(q, q);
        float n = -3.96968303e+01f;
        n = __fadd_rn(__fmul_rn(n, r), 2.20946098e+02f);
        n = __fadd_rn(__fmul_rn(n, r), -2.75928510e+02f);
        n = __fadd_rn(__fmul_rn(n, r), 1.38357752e+02f);
        n = __fadd_rn(__fmul_rn(n, r), -3.06647981e+01f);
        n = __fadd_rn(__fmul_rn(n, r), 2.50662828e+00f);
        n = __fmul_rn(n, q);
        float d = -5.44760988e+01f;
        d = __fadd_rn(__fmul_rn(d, r), 1.61585837e+02f);
        d = __fadd_rn(__fmul_rn(d, r), -1.55698980e+02f);
        d = __fadd_rn(__fmul_rn(d, r), 6.68013119e+01f);
        d = __fadd_rn(__fmul_rn(d, r), -1.32806816e+01f);
        d = __fadd_rn(__fmul_rn(d, r), 1.0f);
        x = __fdiv_rn(n, d);
    }
    return x;
}

} // namespace gen
} // namespace qg
