// RN(x / s) for the FP8 quantizer without a division: Markstein's
// correction of the product by the reciprocal (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; the same step as in Cornea, Harrison and Tang,
// "Scientific Computing on Itanium-based Systems", 2002):
//
//   r = RN(1 / s)            once per row
//   y = RN(x * r)            within an ulp of x / s
//   e = RN(x - y * s)        an FMA; the residual is exact
//   q = RN(y + e * r)        an FMA; the correctly rounded quotient
//
// for rows whose s (at least 2^-60) and r are positive normal f32 values and
// whose products x * r stay far from overflow, while the residual is a
// normal f32 (|x| >= 2^-102).  The sign of x is put on q, so -0 / s is -0
// and a NaN weight's NaN keeps the weight's sign, as the reference's x86
// division does.  Smaller weights' quotients (below 2^-42) may differ from
// the division in the last place; they encode to a signed FP8 zero either
// way.
//
// tests/test_fp8_product.py checks q against IEEE division on the CPU, and
// the FP8 codes through the C restatement's encoder, for every bf16 weight
// against every per-channel scale the reference can form at backoff 1 (and
// strided samples at other backoffs).
//
// Shared by the CUDA quantizer and that CPU check: plain C++ on the host,
// __host__ __device__ under nvcc.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define RENG_HD __host__ __device__ __forceinline__
#else
#define RENG_HD inline
#endif

namespace reng {

RENG_HD uint32_t fp_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

RENG_HD float fp_from_bits(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

RENG_HD float fp_mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);  // never contracted into an FMA
#else
    volatile float p = a * b;
    return p;
#endif
}

RENG_HD float fp_fma_rn(float a, float b, float c) {
#ifdef __CUDA_ARCH__
    return __fmaf_rn(a, b, c);
#else
    return fmaf(a, b, c);
#endif
}

// Whether elements of magnitude at most `xmax` (NaN weights aside) take the
// product path for scale s with r = RN(1 / s): s at least 2^-60 and finite,
// r positive normal, and xmax * r below 2^126, so nothing overflows.  The
// residual x - y * s is exact while |x| >= 2^-102 (it stays a normal f32);
// a smaller weight's quotient is below 2^-42 for such s and encodes to a
// signed zero whatever its last place.
RENG_HD bool fp8_product_ok(float s, float r, float xmax) {
    const uint32_t es = fp_bits(s) >> 23, er = fp_bits(r) >> 23;  // sign bit included: must be 0
    return es >= 67u && es <= 254u && er >= 1u && er <= 254u && xmax * r < 8.507059e37f;  // 2^-60, 2^126
}

// RN(x / s) given r = RN(1 / s), for a row that fp8_product_ok admits.
RENG_HD float fp_quotient(float x, float s, float r) {
    const float y = fp_mul_rn(x, r);
    const float e = fp_fma_rn(-y, s, x);
    const float q = fp_fma_rn(e, r, y);
    return fp_from_bits(fp_bits(q) | (fp_bits(x) & 0x80000000u));
}

}  // namespace reng
