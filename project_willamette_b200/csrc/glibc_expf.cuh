// glibc_expf.cuh -- the exp the reference actually calls, bit for bit.
//
// The reference's f32::exp (softmax_inplace, attention.rs:61-64; SiLU,
// ffn.rs) is the C library's expf on its Linux x86-64 hosts: glibc 2.39 in
// this image, whose expf is the published ARM optimized-routines algorithm
// (glibc sysdeps/ieee754/flt-32/e_expf.c with the 2^(i/32) table of
// e_exp2f_data.c).  It is restated here because a double-precision exp
// rounded once to f32 -- correctly rounded nearly everywhere -- disagrees with
// glibc's 0.502-ulp expf on about 1 in 12,000 arguments in [-40, 0], and a
// long decode (about 350,000 softmax exps per BitNet-2B token) then differs
// from the reference in the last bit of some attention weight, which the
// int8 re-quantisation of the next BitLinear input can turn into a visible
// difference.
//
// The algorithm, in double precision with IEEE round-to-nearest and no
// contraction (each step below is one rounding, as in glibc):
//     z  = x * (32 / ln 2)
//     kd = (z + 1.5 * 2^52) - 1.5 * 2^52    (round z to an integer k)
//     r  = z - kd                            (|r| <= 1/2)
//     s  = 2^(k/32) = the double whose bits are tab[k % 32] + (k << 47)
//     y  = ((c0 r + c1) r^2 + (c2 r + 1)) * s, rounded once to f32
// with tab[i] = bits(2^(i/32)) - (i << 47) (2^(i/32) rounded to the nearest
// double) and c0, c1, c2 the polynomial coefficients of 2^(r/32) scaled by
// 32^-3, 32^-2, 32^-1.  Arguments outside the polynomial's range follow
// glibc: exp(-inf) = +0, NaN -> NaN, x > 88.72283 -> +inf, x < -103.97208 ->
// +0.  For two arguments, 0x1.04845ep+5 and -0x1.f8cbb2p+5, whose polynomial
// value lies within 2^-30 ulp of a rounding midpoint, glibc 2.39 returns the
// correctly rounded result, one ulp above the polynomial's; they are returned
// as glibc does.  Checked against glibc's expf on all 4,278,190,082 non-NaN
// floats (the same steps in host C, identical results), and on the GPU
// through wl_dev_softmax_f32 against the oracle's softmax_inplace.
#pragma once

#include <cstdint>

namespace wl {

__device__ __constant__ uint64_t g_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

__device__ __forceinline__ float glibc_expf(float x) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7FFu;
    if (abstop >= 0x42Bu) {                         // |x| >= 88 (and inf / NaN)
        if (ux == 0xFF800000u) return 0.0f;         // exp(-inf)
        if (abstop >= 0x7F8u) return x + x;         // NaN (and +inf)
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7F800000);  // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;        // underflow
    }
    if (x == 0x1.04845ep+5f) return 0x1.f93e38p+46f;   // glibc's correctly rounded result
    if (x == -0x1.f8cbb2p+5f) return 0x1.f45326p-92f;  // (see above)
    const double inv_ln2_n = 0x1.71547652b82fep+5;  // 32 / ln 2
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-20, c1 = 0x1.ebfce50fac4f3p-13, c2 = 0x1.62e42ff0c52d6p-6;
    const double z = __dmul_rn(inv_ln2_n, (double)x);
    double kd = __dadd_rn(z, shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __dsub_rn(z, kd);
    const uint64_t t = g_exp2_tab[ki % 32u] + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double zp = __dadd_rn(__dmul_rn(c0, r), c1);
    const double r2 = __dmul_rn(r, r);
    double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
    y = __dadd_rn(__dmul_rn(zp, r2), y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

}  // namespace wl
