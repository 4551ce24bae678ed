/*
 * qg_oracle.c -- CPU restatement of the quantized-GEMM workload's arithmetic.
 * TEST INFRASTRUCTURE ONLY (see qg_oracle.h for scope, pins and provenance).
 *
 * Every function cites the workload text or reference convention it follows.
 * Compiled with -ffp-contract=off: each fp32 expression is one IEEE operation
 * with round-to-nearest-even, in the order written.
 */
#include "qg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int qgo_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Use n OpenMP threads from now on (a launcher may have set OMP_NUM_THREADS=1). */
void qgo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------
 * Generator.  The reference fills operands from a hash of the element index
 * (ai_initialize, kernels/common/ai_workload_template.h:85-94;
 * pantheon_gemm_fill, kernels/common/vendor_gemm.h:184-191).  Here the hash
 * is splitmix64 (Steele, Lea & Flood, "Fast splittable pseudorandom number
 * generators", OOPSLA 2014): output i of the stream keyed by (seed, tensor).
 * A and B use different tensor ids, so they never share a stream.
 * ---------------------------------------------------------------------- */
#define QG_GAMMA 0x9E3779B97F4A7C15ull

uint64_t qgo_splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t qgo_hash64(uint64_t seed, uint32_t tensor_id, uint64_t index) {
    uint64_t key = qgo_splitmix64(seed + QG_GAMMA * ((uint64_t)tensor_id + 1ull));
    return qgo_splitmix64(key + QG_GAMMA * (index + 1ull));
}

/* uniform integer in [-127, 127] (configs: "INT8 operands uniform over [-127,127]") */
int8_t qgo_i8_from_hash(uint64_t h) {
    return (int8_t)((int)((uint32_t)(h >> 32) % 255u) - 127);
}

/* lo + (hi - lo) * u, u = top 24 bits / 2^24, three fp32 roundings */
float qgo_uniform_from_hash(uint64_t h, float lo, float hi) {
    float u = (float)(uint32_t)(h >> 40) * 5.9604644775390625e-08f; /* 2^-24, exact */
    float d = hi - lo;
    float t = d * u;
    return lo + t;
}

/* Natural log for x > 0 normal: x = m 2^e with m in [sqrt(1/2), sqrt(2)),
 * log m = 2 atanh(s), s = (m-1)/(m+1), atanh by its odd power series to s^11.
 * Written from the series; fp32, one rounding per operation. */
float qgo_logf(float x) {
    uint32_t b = f2u(x);
    int e = (int)((b >> 23) & 0xFF) - 127;
    float m = u2f((b & 0x007FFFFFu) | 0x3F800000u);
    if (m > 1.41421356f) { m = m * 0.5f; e = e + 1; }
    float num = m - 1.0f;
    float den = m + 1.0f;
    float s = num / den;
    float s2 = s * s;
    float p = 0.0909090936f;              /* 1/11 */
    p = p * s2; p = p + 0.111111112f;     /* 1/9  */
    p = p * s2; p = p + 0.142857149f;     /* 1/7  */
    p = p * s2; p = p + 0.200000003f;     /* 1/5  */
    p = p * s2; p = p + 0.333333343f;     /* 1/3  */
    p = p * s2; p = p + 1.0f;
    float twos = s + s;
    float lm = twos * p;
    float ef = (float)e;
    float el = ef * 0.693147182f;         /* ln 2 */
    return el + lm;
}

/* Inverse normal CDF, P. J. Acklam's rational approximation (2003), in fp32
 * with one rounding per operation; p = (2 j + 1) / 2^24 for the top 23 bits j
 * of h, so p is exact and strictly inside (0, 1). */
float qgo_normal_from_hash(uint64_t h) {
    float p = (float)(2u * (uint32_t)(h >> 41) + 1u) * 5.9604644775390625e-08f; /* 2^-24 */
    const float plow = 0.02425f;
    float x;
    if (p < plow || p > 1.0f - plow) {
        float pp = p < plow ? p : 1.0f - p;
        float l = qgo_logf(pp);
        float t = -2.0f * l;
        float q = sqrtf(t);
        float n = -7.78489400e-03f;
        n = n * q; n = n + -3.22396458e-01f;
        n = n * q; n = n + -2.40075827e+00f;
        n = n * q; n = n + -2.54973254e+00f;
        n = n * q; n = n + 4.37466414e+00f;
        n = n * q; n = n + 2.93816398e+00f;
        float d = 7.78469571e-03f;
        d = d * q; d = d + 3.22467129e-01f;
        d = d * q; d = d + 2.44513414e+00f;
        d = d * q; d = d + 3.75440866e+00f;
        d = d * q; d = d + 1.0f;
        x = n / d;
        if (p > plow) x = -x;
    } else {
        float q = p - 0.5f;
        float r = q * q;
        float n = -3.96968303e+01f;
        n = n * r; n = n + 2.20946098e+02f;
        n = n * r; n = n + -2.75928510e+02f;
        n = n * r; n = n + 1.38357752e+02f;
        n = n * r; n = n + -3.06647981e+01f;
        n = n * r; n = n + 2.50662828e+00f;
        n = n * q;
        float d = -5.44760988e+01f;
        d = d * r; d = d + 1.61585837e+02f;
        d = d * r; d = d + -1.55698980e+02f;
        d = d * r; d = d + 6.68013119e+01f;
        d = d * r; d = d + -1.32806816e+01f;
        d = d * r; d = d + 1.0f;
        x = n / d;
    }
    return x;
}

void qgo_gen_i8(int8_t* out, uint64_t n, uint64_t seed, uint32_t tensor_id) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) out[i] = qgo_i8_from_hash(qgo_hash64(seed, tensor_id, (uint64_t)i));
}

void qgo_gen_uniform_f32(float* out, uint64_t n, float lo, float hi, uint64_t seed, uint32_t tensor_id) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        out[i] = qgo_uniform_from_hash(qgo_hash64(seed, tensor_id, (uint64_t)i), lo, hi);
}

void qgo_gen_normal_f32(float* out, uint64_t n, uint64_t seed, uint32_t tensor_id) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        out[i] = qgo_normal_from_hash(qgo_hash64(seed, tensor_id, (uint64_t)i));
}

/* ------------------------------------------------------------------------
 * Format conversions, round to nearest even.
 * ---------------------------------------------------------------------- */
uint16_t qgo_f32_to_bf16(float x) {
    uint32_t b = f2u(x);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x0040u);
    uint32_t r = b + 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(r >> 16);
}

float qgo_bf16_to_f32(uint16_t v) { return u2f((uint32_t)v << 16); }

uint16_t qgo_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u);
    if (ax >= 0x477FF000u) return sign | 0x7C00u;              /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                     /* below 2^-14: subnormal */
        float q = u2f(ax) * 16777216.0f;                        /* quantum 2^-24, exact scaling */
        return sign | (uint16_t)rintf(q);
    }
    uint32_t e = ((ax >> 23) - 127u + 15u);
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t r = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return sign | (uint16_t)r;
}

float qgo_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    float v;
    if (e == 0) v = ldexpf((float)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexpf((float)(m | 0x400u), (int)e - 25);
    return s ? -v : v;
}

/* OCP FP8 E4M3 ("fn": no infinities, 0x7F/0xFF NaN, max 448), satfinite. */
uint8_t qgo_f32_to_e4m3(float x) {
    uint8_t sign = (uint8_t)((f2u(x) >> 24) & 0x80u);
    float a = fabsf(x);
    if (isnan(x)) return (uint8_t)(sign | 0x7F);
    if (a == 0.0f) return sign;
    if (a > 448.0f) return (uint8_t)(sign | 0x7E);
    int e;
    (void)frexpf(a, &e);
    int E = e - 1;                                   /* a in [2^E, 2^(E+1)) */
    if (E < -6) {                                    /* subnormal: quantum 2^-9 */
        int mi = (int)rintf(a * 512.0f);             /* 8 -> encodes 2^-6 exactly */
        return (uint8_t)(sign | mi);
    }
    int mi = (int)rintf(ldexpf(a, 3 - E));           /* in [8, 16] */
    if (mi == 16) { mi = 8; E += 1; }
    if (E > 8 || (E == 8 && mi > 14)) return (uint8_t)(sign | 0x7E);
    return (uint8_t)(sign | ((E + 7) << 3) | (mi - 8));
}

float qgo_e4m3_to_f32(uint8_t v) {
    int e = (v >> 3) & 0xF, m = v & 7;
    float r;
    if (e == 15 && m == 7) r = NAN;
    else if (e == 0) r = ldexpf((float)m, -9);
    else r = ldexpf((float)(8 + m), e - 10);
    return (v & 0x80) ? -r : r;
}

/* OCP FP4 E2M1: {0, 0.5, 1, 1.5, 2, 3, 4, 6}, satfinite, ties to even code. */
uint8_t qgo_f32_to_e2m1(float x) {
    uint8_t sign = (uint8_t)((f2u(x) >> 28) & 0x8u);
    float a = fabsf(x);
    uint8_t c;
    if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return (uint8_t)(sign | c);
}

float qgo_e2m1_to_f32(uint8_t v) {
    static const float tbl[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float r = tbl[v & 7];
    return (v & 8) ? -r : r;
}

/* ------------------------------------------------------------------------
 * INT8 W8A8 (configs[0..1]): exact INT32 accumulate, then
 * out = f32(acc) * sa[m] * sb[n] (two fp32 roundings, this order).
 * ---------------------------------------------------------------------- */
uint32_t qgo_cksum_weight(uint32_t m, uint32_t n) {
    return (m * 0x9E3779B1u + n * 0x85EBCA77u) | 1u;
}

void qgo_gemm_i8(const int8_t* A, const int8_t* B, const float* sa, const float* sb,
                 int M, int N, int K, const int32_t* rows, int nrows,
                 int out_type, void* C, int32_t* acc, uint32_t* row_cksum) {
    if (!rows) nrows = M;
    /* work items are (row, 256-column tile) so that a sample of a few rows
     * still spreads over every host thread; the row checksum is a wrapping
     * u32 sum, so adding the tiles' parts in any order gives the same bits */
    const int TN = 256;
    int ntn = (N + TN - 1) / TN;
    if (row_cksum) for (int r = 0; r < nrows; ++r) row_cksum[r] = 0;
    #pragma omp parallel for schedule(dynamic, 1)
    for (long it = 0; it < (long)nrows * ntn; ++it) {
        int r = (int)(it / ntn);
        int n0 = (int)(it % ntn) * TN, n1 = n0 + TN < N ? n0 + TN : N;
        int m = rows ? rows[r] : r;
        const int8_t* a = A + (size_t)m * K;
        uint32_t ck = 0;
        for (int n = n0; n < n1; ++n) {
            const int8_t* b = B + (size_t)n * K;
            int32_t s = 0;
            for (int k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
            size_t o = (size_t)r * N + n;
            if (acc) acc[o] = s;
            ck += (uint32_t)s * qgo_cksum_weight((uint32_t)m, (uint32_t)n);
            if (C) {
                if (out_type == 2) { ((int32_t*)C)[o] = s; continue; }
                float f = (float)s;
                f = f * sa[m];
                f = f * sb[n];
                if (out_type == 1) ((float*)C)[o] = f;
                else ((uint16_t*)C)[o] = qgo_f32_to_bf16(f);
            }
        }
        if (row_cksum) {
            #pragma omp atomic
            row_cksum[r] += ck;
        }
    }
}

/* ------------------------------------------------------------------------
 * Tensor-furnace operands (the mma_virus workload; the reference fills them
 * uniform on [-1, 1) in steps of 2^-15, kernels/common/vendor_gemm.h:184-191):
 * v = j / 32768 - 1 with j the top 16 bits of the element's hash (exact in
 * fp32), rounded to the operand format.  tf32 is kept as an fp32 word rounded
 * to nearest even at 10 mantissa bits with the low 13 bits cleared.
 * ---------------------------------------------------------------------- */
uint32_t qgo_f32_to_tf32_bits(float x) {
    uint32_t u = f2u(x);
    if (isnan(x)) return u | 0x00400000u;
    u += 0xFFFu + ((u >> 13) & 1u);
    return u & 0xFFFFE000u;
}

float qgo_dense_value(uint64_t h) {
    return (float)(uint32_t)(h >> 48) * 3.0517578125e-05f - 1.0f;
}

void qgo_gen_dense(int fmt, void* out, uint64_t n, uint64_t seed, uint32_t tensor_id) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        float v = qgo_dense_value(qgo_hash64(seed, tensor_id, (uint64_t)i));
        switch (fmt) {
            case QGO_FMT_BF16: ((uint16_t*)out)[i] = qgo_f32_to_bf16(v); break;
            case QGO_FMT_FP16: ((uint16_t*)out)[i] = qgo_f32_to_f16(v); break;
            case QGO_FMT_TF32: ((uint32_t*)out)[i] = qgo_f32_to_tf32_bits(v); break;
            case QGO_FMT_FP32: ((float*)out)[i] = v; break;
            default: ((uint8_t*)out)[i] = qgo_f32_to_e4m3(v); break;
        }
    }
}

/* ------------------------------------------------------------------------
 * Tensor-furnace GEMMs: C = alpha * A B^T with bf16 (kind 1), e4m3 (kind 2),
 * fp16 (kind 3), tf32 (kind 4, fp32 words holding tf32 values) or fp32
 * (kind 5) operands;
 * the exact products are summed in double, rounded to fp32, scaled by alpha
 * in fp32, then stored as bf16 (out_type 0), fp32 (1) or fp16 (3).  Rows
 * rows[0..nrows) of C (all when rows is NULL), compact.
 * ---------------------------------------------------------------------- */
static float dense_operand(int kind, const void* X, size_t i, const float* lut) {
    switch (kind) {
        case 1: return qgo_bf16_to_f32(((const uint16_t*)X)[i]);
        case 3: return qgo_f16_to_f32(((const uint16_t*)X)[i]);
        case 4: case 5: return u2f(((const uint32_t*)X)[i]);
        default: return lut[((const uint8_t*)X)[i]];
    }
}

void qgo_gemm_dense(int kind, const void* A, const void* B, float alpha, int M, int N, int K,
                    const int32_t* rows, int nrows, int out_type, void* C) {
    if (!rows) nrows = M;
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = qgo_e4m3_to_f32((uint8_t)i);
    #pragma omp parallel for schedule(dynamic, 1)
    for (int r = 0; r < nrows; ++r) {
        int m = rows ? rows[r] : r;
        double* av = (double*)malloc(sizeof(double) * (size_t)K);
        for (int k = 0; k < K; ++k) av[k] = dense_operand(kind, A, (size_t)m * K + k, lut);
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += av[k] * (double)dense_operand(kind, B, (size_t)n * K + k, lut);
            float f = (float)s;
            f = f * alpha;
            size_t o = (size_t)r * N + n;
            if (out_type == 1) ((float*)C)[o] = f;
            else if (out_type == 3) ((uint16_t*)C)[o] = qgo_f32_to_f16(f);
            else ((uint16_t*)C)[o] = qgo_f32_to_bf16(f);
        }
        free(av);
    }
}

/* ------------------------------------------------------------------------
 * FP8 e4m3 block-128: "values drawn N(0,1) then scaled so that
 * each block's absmax maps to 448"; scale s = absmax / 448 so x ~ q * s.
 * A blocks are 1x128 along K, B blocks 128x128.
 * ---------------------------------------------------------------------- */
static void quant_fp8_block(const float* X, int K, int r0, int r1, int k0, uint8_t* Q, float* s_out) {
    float amax = 0.0f;
    for (int r = r0; r < r1; ++r)
        for (int k = k0; k < k0 + 128; ++k) { float a = fabsf(X[(size_t)r * K + k]); if (a > amax) amax = a; }
    float inv = amax > 0.0f ? 448.0f / amax : 1.0f;
    float s = amax > 0.0f ? amax / 448.0f : 1.0f;
    for (int r = r0; r < r1; ++r)
        for (int k = k0; k < k0 + 128; ++k) {
            float v = X[(size_t)r * K + k] * inv;
            Q[(size_t)r * K + k] = qgo_f32_to_e4m3(v);
        }
    *s_out = s;
}

void qgo_quant_fp8_rows(const float* X, int R, int K, uint8_t* Q, float* S) {
    int kb = K / 128;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < R; ++r)
        for (int b = 0; b < kb; ++b) quant_fp8_block(X, K, r, r + 1, b * 128, Q, &S[(size_t)r * kb + b]);
}

void qgo_quant_fp8_blocks(const float* X, int R, int K, uint8_t* Q, float* S) {
    int kb = K / 128, rb = (R + 127) / 128;   /* a last partial block of rows is its own block */
    #pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < rb; ++i)
        for (int b = 0; b < kb; ++b) {
            int r1 = i * 128 + 128 < R ? i * 128 + 128 : R;
            quant_fp8_block(X, K, i * 128, r1, b * 128, Q, &S[(size_t)i * kb + b]);
        }
}

/* Per 128-wide K block: exact partial sum (products of e4m3 values are exact in
 * fp32 and 128 of them sum exactly in double), rounded once to fp32, then
 * acc = fma(partial, sa[m,kb] * sb[n/128,kb], acc) in fp32, K blocks in order
 * (the promotion the GPU epilogue performs per K block). */
void qgo_gemm_fp8_b128(const uint8_t* A, const uint8_t* B, const float* sa, const float* sb,
                       int M, int N, int K, const int32_t* rows, int nrows,
                       int out_type, void* C) {
    if (!rows) nrows = M;
    int kb = K / 128;
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = qgo_e4m3_to_f32((uint8_t)i);
    #pragma omp parallel for schedule(dynamic, 1)
    for (int r = 0; r < nrows; ++r) {
        int m = rows ? rows[r] : r;
        const uint8_t* a = A + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const uint8_t* b = B + (size_t)n * K;
            float acc = 0.0f;
            for (int j = 0; j < kb; ++j) {
                double p = 0.0;
                for (int k = j * 128; k < j * 128 + 128; ++k) p += (double)(lut[a[k]] * lut[b[k]]);
                float pf = (float)p;
                float sc = sa[(size_t)m * kb + j] * sb[(size_t)(n / 128) * kb + j];
                acc = fmaf(pf, sc, acc);
            }
            size_t o = (size_t)r * N + n;
            if (out_type == 1) ((float*)C)[o] = acc;
            else ((uint16_t*)C)[o] = qgo_f32_to_bf16(acc);
        }
    }
}

/* ------------------------------------------------------------------------
 * NVFP4: per-tensor scale G = amax / (448 * 6); per 16-element
 * block along K an ue4m3 scale sf = e4m3(bmax / 6 / G); codes
 * q = e2m1(x / (dec(sf) * G)); x ~ q * dec(sf) * G.
 * ---------------------------------------------------------------------- */
float qgo_nvfp4_global_scale(const float* X, uint64_t n) {
    float amax = 0.0f;
    for (uint64_t i = 0; i < n; ++i) { float a = fabsf(X[i]); if (a > amax) amax = a; }
    if (amax == 0.0f) return 1.0f;
    float d = 448.0f * 6.0f;
    return amax / d;
}

void qgo_quant_nvfp4(const float* X, int R, int K, float G, uint8_t* Q, uint8_t* SF) {
    int nb = K / 16;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < R; ++r) {
        for (int b = 0; b < nb; ++b) {
            const float* x = X + (size_t)r * K + b * 16;
            float bmax = 0.0f;
            for (int i = 0; i < 16; ++i) { float a = fabsf(x[i]); if (a > bmax) bmax = a; }
            float t = bmax / 6.0f;
            t = t / G;
            uint8_t sf = qgo_f32_to_e4m3(t) & 0x7F;
            SF[(size_t)r * nb + b] = sf;
            float d = qgo_e4m3_to_f32(sf) * G;
            for (int i = 0; i < 16; i += 2) {
                uint8_t c0 = 0, c1 = 0;
                if (d > 0.0f) { c0 = qgo_f32_to_e2m1(x[i] / d); c1 = qgo_f32_to_e2m1(x[i + 1] / d); }
                Q[((size_t)r * K + b * 16 + i) / 2] = (uint8_t)(c0 | (c1 << 4));
            }
        }
    }
}

/* acc = sum_k (q_a sfa) (q_b sfb) accumulated in double, rounded to fp32,
 * out = acc * (GA * GB) (fp32). */
void qgo_gemm_nvfp4(const uint8_t* A, const uint8_t* SFA, float GA,
                    const uint8_t* B, const uint8_t* SFB, float GB,
                    int M, int N, int K, const int32_t* rows, int nrows,
                    int out_type, void* C) {
    if (!rows) nrows = M;
    int nb = K / 16;
    float g = GA * GB;
    #pragma omp parallel for schedule(dynamic, 1)
    for (int r = 0; r < nrows; ++r) {
        int m = rows ? rows[r] : r;
        float* av = (float*)malloc(sizeof(float) * (size_t)K);
        for (int k = 0; k < K; ++k) {
            uint8_t byte = A[((size_t)m * K + k) / 2];
            uint8_t c = (k & 1) ? (byte >> 4) : (byte & 0xF);
            av[k] = qgo_e2m1_to_f32(c) * qgo_e4m3_to_f32(SFA[(size_t)m * nb + k / 16]);
        }
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int b = 0; b < nb; ++b) {
                double bs = (double)qgo_e4m3_to_f32(SFB[(size_t)n * nb + b]);
                double ps = 0.0;
                for (int i = 0; i < 16; ++i) {
                    int k = b * 16 + i;
                    uint8_t byte = B[((size_t)n * K + k) / 2];
                    uint8_t c = (k & 1) ? (byte >> 4) : (byte & 0xF);
                    ps += (double)av[k] * (double)qgo_e2m1_to_f32(c);
                }
                s += ps * bs;
            }
            float accf = (float)s;
            float out = accf * g;
            size_t o = (size_t)r * N + n;
            if (out_type == 1) ((float*)C)[o] = out;
            else ((uint16_t*)C)[o] = qgo_f32_to_bf16(out);
        }
        free(av);
    }
}

/* ------------------------------------------------------------------------
 * W4A16 group-128: w = (q - z) * s, accumulated in double,
 * rounded to fp32 then bf16.  Computed for columns cols[0..ncols) (all when NULL);
 * Y is [M, ncols] compact.
 * ---------------------------------------------------------------------- */
void qgo_gemv_w4a16(const uint16_t* X, const uint32_t* W, const uint16_t* S, const uint16_t* Z,
                    int M, int N, int K, const int32_t* cols, int ncols,
                    int out_type, void* Y) {
    if (!cols) ncols = N;
    int ng = K / 128;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int c = 0; c < ncols; ++c) {
        int n = cols ? cols[c] : c;
        for (int m = 0; m < M; ++m) {
            double acc = 0.0;
            for (int g = 0; g < ng; ++g) {
                double s = (double)qgo_f16_to_f32(S[(size_t)g * N + n]);
                double z = (double)qgo_f16_to_f32(Z[(size_t)g * N + n]);
                double part = 0.0;
                for (int k = g * 128; k < g * 128 + 128; ++k) {
                    uint32_t w = W[(size_t)(k / 8) * N + n];
                    int q = (int)((w >> (4 * (k % 8))) & 0xF) - 8;
                    double x = (double)qgo_bf16_to_f32(X[(size_t)m * K + k]);
                    part += x * ((double)q - z);
                }
                acc += part * s;
            }
            float f = (float)acc;
            size_t o = (size_t)m * ncols + c;
            if (out_type == 1) ((float*)Y)[o] = f;
            else ((uint16_t*)Y)[o] = qgo_f32_to_bf16(f);
        }
    }
}

/* W4A16 operands: X = bf16(N(0,1)); u = top 4 bits of hash(k*N+n)
 * packed 8 per word along K; S = f16(U[0.005,0.02]); Z = f16(U[-0.5,0.5]). */
void qgo_gen_w4a16(uint16_t* X, uint32_t* W, uint16_t* S, uint16_t* Z, int M, int N, int K,
                   uint64_t seed, uint32_t tid0) {
    uint64_t nx = (uint64_t)M * K, nw = (uint64_t)K / 8 * N, ns = (uint64_t)K / 128 * N;
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)nx; ++i)
        X[i] = qgo_f32_to_bf16(qgo_normal_from_hash(qgo_hash64(seed, tid0, (uint64_t)i)));
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)nw; ++i) {
        uint64_t k8 = (uint64_t)i / (uint64_t)N, n = (uint64_t)i - k8 * (uint64_t)N;
        uint32_t w = 0;
        for (int j = 0; j < 8; ++j) {
            uint64_t k = k8 * 8 + (uint64_t)j;
            w |= (uint32_t)(qgo_hash64(seed, tid0 + 1, k * (uint64_t)N + n) >> 60) << (4 * j);
        }
        W[i] = w;
    }
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)ns; ++i) {
        S[i] = qgo_f32_to_f16(qgo_uniform_from_hash(qgo_hash64(seed, tid0 + 2, (uint64_t)i), 0.005f, 0.02f));
        Z[i] = qgo_f32_to_f16(qgo_uniform_from_hash(qgo_hash64(seed, tid0 + 3, (uint64_t)i), -0.5f, 0.5f));
    }
}

/* ------------------------------------------------------------------------
 * Verification helpers (word compare as ai_verify_output,
 * kernels/common/ai_workload_template.h:343-349).
 * ---------------------------------------------------------------------- */
uint64_t qgo_count_mismatch_u32(const uint32_t* a, const uint32_t* b, uint64_t n) {
    uint64_t c = 0;
    for (uint64_t i = 0; i < n; ++i) c += a[i] != b[i];
    return c;
}

double qgo_max_rel_err(const void* y, const void* r, uint64_t n, int kind) {
    double ss = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        double rv = kind ? (double)((const float*)r)[i] : (double)qgo_bf16_to_f32(((const uint16_t*)r)[i]);
        ss += rv * rv;
    }
    double rms = n ? sqrt(ss / (double)n) : 0.0;
    if (rms == 0.0) rms = 1e-30;
    double worst = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        double rv = kind ? (double)((const float*)r)[i] : (double)qgo_bf16_to_f32(((const uint16_t*)r)[i]);
        double yv = kind ? (double)((const float*)y)[i] : (double)qgo_bf16_to_f32(((const uint16_t*)y)[i]);
        double den = fabs(rv) > rms ? fabs(rv) : rms;
        double e = fabs(yv - rv) / den;
        if (!(e <= worst)) worst = e;   /* NaN propagates as worst */
    }
    return worst;
}
