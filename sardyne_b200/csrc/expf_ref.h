// expf as the reference computes it on its host: the reference calls libm's expf (softmax,
// ops.c:353-364; SiLU, ops.c:366-371; attention through op_softmax), and glibc (2.28 and later;
// the image's is 2.39) implements it with the published table-driven method of ARM's
// optimized-routines expf (Szabolcs Nagy): with N = 32,
//     x = (k + r) ln2 / N,  k integer, |r| <= 1/2,   exp(x) = 2^(k/N) * 2^(r/N),
// 2^(k/N) = 2^(k div N) * T[k mod N] with T[i] = 2^(i/N) rounded to double, and 2^(r/N) by a cubic
// in r evaluated in double, rounded once to float at the end. glibc's x86-64 build of it fuses
// r = x*N/ln2 - k into one multiply-add. Restated here in double with explicitly rounded
// operations so that the GPU gets glibc's float for every input (checked exhaustively over all
// 2^32 inputs against the host's expf by tests/test_expf_ref.py). The correctly rounded exp
// differs from glibc's on 170,648 inputs, and on these synthetic models one differing exp in an
// attention softmax flips int8 roundings downstream, so the end-to-end logits would drift.
//
// Shared by the CUDA kernels (device) and the CPU check (plain C/C++, compiled with
// -ffp-contract=off so that only the fma() calls fuse).
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define SDY_EXPF_FN __device__ __forceinline__
#else
#define SDY_EXPF_FN static inline
#endif

namespace sdy {

// Bit patterns of 2^(i/32) rounded to nearest double, minus i << 47 (the table entry is added to
// k << 47, which puts k div 32 into the exponent field). On the GPU the table sits in global
// memory and is read through the read-only L1 path: the lanes of a warp index different entries,
// which the constant cache would serve one address at a time.
#if defined(__CUDACC__)
__device__
#endif
static const uint64_t kExp2Tab32[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

SDY_EXPF_FN float expf_ref(float x) {
    // Minimax cubic for 2^(r/32), |r| <= 1/2, coefficients as published with the method.
    const double C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 C2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double INV_LN2_N = 0x1.71547652b82fep+0 * 32;  // N / ln 2
    const double SHIFT = 0x1.8p+52;                      // rounds to an integer in the low bits
    uint32_t ux;
    memcpy(&ux, &x, 4);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) {  // |x| >= 88, inf or nan
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double xd = (double)x;
#if defined(__CUDACC__)
    const double z = __dmul_rn(INV_LN2_N, xd);
    const double kd_shifted = __dadd_rn(z, SHIFT);
    uint64_t ki;
    memcpy(&ki, &kd_shifted, 8);
    const double kd = __dsub_rn(kd_shifted, SHIFT);
    const double r = __fma_rn(INV_LN2_N, xd, -kd);
    uint64_t t = __ldg((const unsigned long long *)&kExp2Tab32[ki % 32]) + (ki << 47);
    double s;
    memcpy(&s, &t, 8);
    const double p = __fma_rn(C0, r, C1), r2 = __dmul_rn(r, r);
    double y = __fma_rn(C2, r, 1.0);
    y = __fma_rn(p, r2, y);
    return (float)__dmul_rn(y, s);
#else
    const double z = INV_LN2_N * xd;
    const double kd_shifted = z + SHIFT;
    uint64_t ki;
    memcpy(&ki, &kd_shifted, 8);
    const double kd = kd_shifted - SHIFT;
    const double r = fma(INV_LN2_N, xd, -kd);
    uint64_t t = kExp2Tab32[ki % 32] + (ki << 47);
    double s;
    memcpy(&s, &t, 8);
    const double p = fma(C0, r, C1), r2 = r * r;
    double y = fma(C2, r, 1.0);
    y = fma(p, r2, y);
    return (float)(y * s);
#endif
}

}  // namespace sdy
